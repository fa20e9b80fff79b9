"""Evaluation harness of the reference (gpu-d1/scripts/train_clear.py:42-76 and
run_ring_ablations.py:231-267) on the B200 kernels.

Every env plays one episode from the evaluation seed; an `active` mask freezes
envs whose episode has ended (d1_spec_step / learn_step_active leave them
untouched), their outcome row is kept, and the loop ends when no env is active.
Modes: 'greedy' and 'sampled' (a policy), 'wait', 'random' (uniform over the
legal actions, d1_sample_uniform_legal) and, on the reference-compatible task,
'pursuit' (learn_heuristic). Per-step bookkeeping is one kernel
(d1_eval_accumulate); the host checks the active set every `check_every` steps.

Metrics follow train_clear.py:62-76: clear rate with its Wilson 95 % interval,
kills, final hp, episode length, death and timeout rates, mean shaped return.
Outcome columns 0-7 mean the same on both tasks (reward, done, clear, kills, hp,
length, death, timeout).
"""
import math

import torch

from ._lib import check, library, launch_stream


def wilson(successes, n, z=1.96):
    """Wilson score interval for successes / n (train_clear.py:63-66)."""
    phat = successes / n
    center = (phat + z * z / (2 * n)) / (1 + z * z / n)
    half = z * math.sqrt(phat * (1 - phat) / n + z * z / (4 * n * n)) / (1 + z * z / n)
    return center - half, center + half


def _legal_bits(env):
    if hasattr(env, 'legal'):
        return env.legal, 12
    mask = env.mask > 0  # reference-compatible task: float mask [n, 9]
    weights = 1 << torch.arange(mask.shape[1], device=mask.device)
    return (mask.to(torch.int64) * weights).sum(1).to(torch.int16), mask.shape[1]


@torch.no_grad()
def evaluate(env, policy=None, mode='greedy', seed=900000, steps=None, check_every=32):
    lib = library()
    dev, n = env.device, env.batch
    stream = launch_stream(dev)
    spec = hasattr(env, 'values')
    if mode in ('greedy', 'sampled') and policy is None:
        raise ValueError(f'mode {mode!r} needs a policy')
    if mode == 'pursuit' and spec:
        raise ValueError('the pursuit baseline exists for the reference-compatible task only')
    conv = policy is not None and hasattr(policy, 'act_from_features')
    env.reset(seed)
    first_env = getattr(env, 'first_env', 0)
    active = torch.ones(n, dtype=torch.bool, device=dev)
    terminal = torch.zeros((n, 8), device=dev)
    returns = torch.zeros(n, device=dev)
    action = torch.empty(n, dtype=torch.int64, device=dev)
    limit = steps or (env.values['limit'] if spec else env.limit)
    buf = policy.buffers(n) if conv else None
    cout = None
    for k in range(limit):
        if mode == 'wait':
            action.fill_(8)
        elif mode == 'random':
            bits, nact = _legal_bits(env)
            check(lib.d1_sample_uniform_legal(bits.data_ptr(), nact, n, seed, k, first_env, action.data_ptr(),
                                              stream), 'd1_sample_uniform_legal')
        elif mode == 'pursuit':
            action = env.heuristic()
        elif conv:
            policy.encode(env.state, n, buf)
            policy.features(buf, n)
            if mode == 'greedy':
                p = policy.params
                check(lib.d1_ar_head_greedy(buf['hb'].data_ptr(), n, policy.cond.data_ptr(), p['wt'].data_ptr(),
                                            p['bt'].data_ptr(), env.legal.data_ptr(), None, action.data_ptr(),
                                            None, None, stream), 'd1_ar_head_greedy')
            else:
                cout = policy.act_from_features(env.legal, n, buf, seed, k, first_env, out=cout)
                action = cout['env_action']
        else:
            _, h2 = policy.hidden_layers(env.obs)
            if mode == 'greedy':
                check(lib.d1_policy_head_greedy(h2.data_ptr(), n, policy.hidden, policy.bf16['wh'].data_ptr(),
                                                policy.params['bh'].data_ptr(), env.legal.data_ptr(),
                                                action.data_ptr(), None, None, stream), 'd1_policy_head_greedy')
            else:
                policy.head(h2, env.legal, seed, k, first_env, action, None, None)
        env.step(action, active=active)
        check(lib.d1_eval_accumulate(env.out.data_ptr(), env.out.shape[1], n, active.data_ptr(), returns.data_ptr(),
                                     terminal.data_ptr(), 8, stream), 'd1_eval_accumulate')
        if (k + 1) % check_every == 0 and not active.any().item():
            break
    if active.any().item():
        raise RuntimeError('episodes still running after the step limit')
    return metrics(terminal.cpu(), returns.cpu(), mode, seed, getattr(env, 'enemies', None))


def metrics(t, returns, mode, seed, enemies=None):
    n = t.shape[0]
    successes = float(t[:, 2].sum())
    lo, hi = wilson(successes, n)
    cleared = t[:, 2] > 0
    kills = float(t[:, 3].mean())
    return dict(mode=mode, eval_seed=seed, episodes=n, clear_rate=successes / n, clear_ci95=[lo, hi],
                enemies_killed=kills, killed_fraction=kills / enemies if enemies else None,
                mean_hp=float(t[:, 4].mean()), mean_length=float(t[:, 5].mean()),
                clear_length=float(t[cleared, 5].mean()) if successes else None,
                death_rate=float(t[:, 6].mean()), timeout_rate=float(t[:, 7].mean()),
                mean_return=float(returns.mean()))
