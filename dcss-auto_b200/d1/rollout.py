"""Rollout buffer and collection loop of gpu-d1/scripts/run_ring_ablations.py:332-353
on the B200 kernels.

Every step the policy reads observation slot t and writes action/log-prob/value
slot t; the env step writes its next observation and legal mask straight into
slot t+1 and its outcome row into out[t]. Nothing is copied between kernels.
"""
import torch

OBS = 1832


class Rollout:
    def __init__(self, env, policy, horizon, seed=0, sample_seed=None):
        self.env, self.policy, self.T = env, policy, horizon
        B, dev = env.batch, env.device
        self.seed = seed
        self.sample_seed = seed if sample_seed is None else sample_seed
        self.obs = torch.empty((horizon + 1, B, OBS), dtype=torch.bfloat16, device=dev)
        self.legal = torch.empty((horizon + 1, B), dtype=torch.int16, device=dev)
        self.actions = torch.empty((horizon, B), dtype=torch.int64, device=dev)
        self.logp = torch.empty((horizon, B), device=dev)
        self.values = torch.empty((horizon + 1, B), device=dev)
        self.out = torch.zeros((horizon, B, env.out.shape[1]), device=dev)
        self.global_step = 0
        env.reset(seed, obs_out=self.obs[0], legal_out=self.legal[0])

    def step(self, t):
        self.policy.act(self.obs[t], self.legal[t], self.sample_seed, self.global_step, self.env.first_env,
                        action=self.actions[t], logp=self.logp[t], value=self.values[t])
        self.env.step(self.actions[t], obs_out=self.obs[t + 1], legal_out=self.legal[t + 1], out_out=self.out[t])
        self.global_step += 1

    def bootstrap(self):
        self.policy.value(self.obs[self.T], out=self.values[self.T])

    def collect(self):
        for t in range(self.T):
            self.step(t)
        self.bootstrap()

    def roll(self):
        """Start the next rollout from the last observation."""
        self.obs[0].copy_(self.obs[self.T])
        self.legal[0].copy_(self.legal[self.T])

    @property
    def rewards(self):
        return self.out[:, :, 0]

    @property
    def dones(self):
        return self.out[:, :, 1]
