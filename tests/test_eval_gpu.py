"""Evaluation harness, greedy heads, frame stack and exact checkpoint/resume on
the GPU (reference: gpu-d1/scripts/train_clear.py:42-76,
run_ring_ablations.py:231-309, scripts/test_resume.py, vision15-centered-map-v1/
scripts/frame_stack.py):

* the evaluation loop (active mask, terminal rows, returns, Wilson interval)
  gives exactly the metrics of the same loop run on the CPU -- the oracle for
  the spec task with the random baseline, the reference's own host build for
  the reference-compatible task with the wait and pursuit baselines;
* greedy heads pick the argmax of the masked distribution;
* the frame-stack kernel equals a torch restatement of the reference wrapper;
* a PPO run saved after two iterations and resumed for two more ends bit-for-bit
  where the uninterrupted run ends.
"""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def d1mods():
    from d1 import evaluate, spec_env, learn_env, policy, conv_policy, frame_stack, checkpoint, ppo, rollout
    oracle.build()
    return dict(evaluate=evaluate, spec_env=spec_env, learn_env=learn_env, policy=policy, conv_policy=conv_policy,
                frame_stack=frame_stack, checkpoint=checkpoint, ppo=ppo, rollout=rollout)


def host_loop(env, pick, limit):
    """The reference's evaluation loop (train_clear.py:47-58) on a CPU env."""
    n = env.batch
    active = np.ones(n, bool)
    terminal = np.zeros((n, 8), np.float32)
    returns = np.zeros(n, np.float32)
    for k in range(limit):
        _, out = env.step(pick(env, k), active)
        returns[active] += out[active, 0]
        ended = active & (out[:, 1] > 0)
        terminal[ended] = out[ended, :8]
        active &= ~ended
        if not active.any():
            break
    assert not active.any()
    return terminal, returns


class OracleSpecActive:
    """OracleSpec with the GPU's active-mask semantics: inactive envs keep their
    state, observation, legal bits and outcome row."""

    def __init__(self, n, config, seed):
        self.env = oracle.OracleSpec(n, config, seed=seed)
        self.batch = n

    @property
    def legal(self):
        return self.env.legal

    def step(self, actions, active):
        e = self.env
        saved = [a.copy() for a in (e.state, e.obs, e.legal, e.out)]
        e.step(actions)
        keep = ~active
        for arr, old in zip((e.state, e.obs, e.legal, e.out), saved):
            arr[keep] = old[keep]
        return e.obs, e.out


def test_random_baseline_eval_matches_oracle(d1mods):
    ev, spec_env = d1mods['evaluate'], d1mods['spec_env']
    n, seed = 128, 900000
    got = ev.evaluate(spec_env.SpecEnv(n, seed=1), mode='random', seed=seed)
    cpu = OracleSpecActive(n, spec_env.DEFAULT, seed)
    pick = lambda env, k: oracle.sample_uniform_legal(env.legal, 12, seed, k)
    terminal, returns = host_loop(cpu, pick, spec_env.DEFAULT['limit'])
    ref = ev.metrics(torch.from_numpy(terminal), torch.from_numpy(returns), 'random', seed)
    assert got == ref


@pytest.mark.parametrize('mode', ['wait', 'pursuit'])
def test_reference_task_eval_matches_the_reference_build(d1mods, mode):
    ev, learn_env = d1mods['evaluate'], d1mods['learn_env']
    try:
        ref_env = oracle.ReferenceV1(96, 6, seed=0)
    except FileNotFoundError:
        pytest.skip('reference build oracle/_ref/learn_v1.so not present')
    ref_env.reset(900000)
    got = ev.evaluate(learn_env.Env(96, 6, seed=0), mode=mode)
    pick = (lambda env, k: np.full(env.batch, 8, np.int64)) if mode == 'wait' else (lambda env, k: env.heuristic())
    terminal, returns = host_loop(ref_env, pick, 256)
    assert got == ev.metrics(torch.from_numpy(terminal), torch.from_numpy(returns), mode, 900000, 6)


def test_greedy_heads_take_the_masked_argmax(d1mods):
    spec_env, policy, conv_policy = d1mods['spec_env'], d1mods['policy'], d1mods['conv_policy']
    from d1._lib import library
    lib = library()
    n = 512
    env = spec_env.SpecEnv(n, seed=3)
    pol = policy.Policy(seed=2)
    _, h2 = pol.hidden_layers(env.obs)
    logits = torch.empty((n, 12), device='cuda')
    pol.head(h2, env.legal, 0, 0, 0, None, None, None, logits)
    act = torch.empty(n, dtype=torch.int64, device='cuda')
    s = torch.cuda.current_stream().cuda_stream
    assert lib.d1_policy_head_greedy(h2.data_ptr(), n, 256, pol.bf16['wh'].data_ptr(), pol.params['bh'].data_ptr(),
                                     env.legal.data_ptr(), act.data_ptr(), None, None, s) == 0
    mask = ((env.legal.to(torch.int64)[:, None] & 0xffff) >> torch.arange(12, device='cuda')) & 1
    assert torch.equal(act, logits.masked_fill(mask == 0, -1e9).argmax(-1))
    # autoregressive head: argmax verb, then argmax target of that verb
    cp = conv_policy.ConvPolicy(seed=5, chunk=256)
    buf = cp.buffers(n)
    dbg = cp.act(env.state, env.legal, n, buf, 1, 1, debug=True)
    joint = torch.empty(n, dtype=torch.int64, device='cuda')
    p = cp.params
    assert lib.d1_ar_head_greedy(buf['hb'].data_ptr(), n, cp.cond.data_ptr(), p['wt'].data_ptr(), p['bt'].data_ptr(),
                                 env.legal.data_ptr(), joint.data_ptr(), None, None, None, s) == 0
    from test_conv_gpu import ReferenceActionDistribution, masks
    tvalid, vmask = masks(env.legal)
    dist = ReferenceActionDistribution(dbg['verb_logits'], dbg['target_logits'], tvalid, vmask)
    kind = dist.types.probs.argmax(-1)
    direction = dist.directions.probs.argmax(-1).gather(1, kind.clamp_max(1)[:, None]).squeeze(1)
    assert torch.equal(joint, torch.where(kind < 2, 9 * kind + direction, kind + 16))


class ReferenceFrameStack:
    """Torch restatement of vision15-centered-map-v1/scripts/frame_stack.py:5-32."""

    def __init__(self, base, frames):
        self.base, self.frames = base, frames
        self.width = base.obs.shape[1]
        self.obs = base.obs.repeat(1, frames)

    def step(self, actions, active=None):
        _, out = self.base.step(actions) if active is None else self.base.step(actions, active=active)
        self.obs[:, :-self.width].copy_(self.obs[:, self.width:].clone())
        self.obs[:, -self.width:].copy_(self.base.obs)
        ended = out[:, 1] > 0
        if active is not None:
            ended &= active
        self.obs[ended] = self.base.obs[ended].repeat(1, self.frames)
        return self.obs, out


def test_frame_stack_matches_the_reference_wrapper(d1mods):
    spec_env, fs = d1mods['spec_env'], d1mods['frame_stack']
    from golden.schedule import random_actions
    n = 256
    a = fs.FrameStack(spec_env.SpecEnv(n, seed=9), frames=4)
    b = ReferenceFrameStack(spec_env.SpecEnv(n, seed=9), frames=4)
    assert torch.equal(a.obs, b.obs)
    acts = torch.from_numpy(random_actions(3, 80, n, 12)).cuda()
    g = torch.Generator(device='cuda').manual_seed(1)
    for k in range(80):
        active = None if k % 3 else (torch.rand(n, device='cuda', generator=g) > 0.2)
        a.step(acts[k].contiguous(), active)
        b.step(acts[k].contiguous(), active)
        assert torch.equal(a.obs.view(torch.int16), b.obs.view(torch.int16)), k


@pytest.mark.parametrize('torch_order', [False, True])
def test_checkpoint_resume_is_exact(d1mods, tmp_path, torch_order):
    """The epoch order from d1_ppo_permute (device epoch count in the
    checkpoint) or from torch.randperm on a generator (its state saved)."""
    spec_env, policy, rollout, ppo, ckpt = (d1mods[k] for k in ('spec_env', 'policy', 'rollout', 'ppo', 'checkpoint'))

    def make():
        env = spec_env.SpecEnv(256, seed=1)
        pol = policy.Policy(seed=0)
        roll = rollout.Rollout(env, pol, 16, seed=1)
        tr = ppo.PPO(pol, roll, minibatch=1024, epochs=2, perm_seed=11)
        return tr, (torch.Generator(device='cuda').manual_seed(5) if torch_order else None)

    full, g_full = make()
    for _ in range(4):
        full.iteration(g_full)
    half, g_half = make()
    for _ in range(2):
        half.iteration(g_half)
    ckpt.save(tmp_path / 'latest.pt', half, g_half, extra={'iterations': 2})
    resumed, g_res = make()
    assert ckpt.load(tmp_path / 'latest.pt', resumed, g_res) == {'iterations': 2}
    for _ in range(2):
        resumed.iteration(g_res)
    torch.cuda.synchronize()
    a, b = ckpt.state_dict(full, g_full), ckpt.state_dict(resumed, g_res)
    keys = ['params', 'adam_m', 'adam_v', 'adam_step', 'perm_epoch', 'env_state', 'obs', 'cobs', 'legal']
    for key in keys + (['generator'] if torch_order else []):
        assert torch.equal(a[key], b[key]), key
    assert a['global_step'] == b['global_step']
    # a different job is refused
    other, _ = make()
    other.lr = 1e-3
    with pytest.raises(ValueError):
        ckpt.load(tmp_path / 'latest.pt', other)
