#!/usr/bin/env python3
"""Throughput of the batched D:1 env step feeding the policy.

A step is one decision for every env of the job: MLP policy forward and masked
sampling on observation slot t, then the env step that writes slot t+1 (the
rollout loop of gpu-d1/scripts/run_ring_ablations.py:346-352). Weak scaling:
each rank owns 65,536 envs (global env ids rank*65536 + i). Data is synthetic:
every env plays its own seeded generated map.

  python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Prints one JSON line on rank 0.
"""
import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / 'dcss-auto_b200'))

METRIC = 'env decisions/sec (sim+policy, device-timed)'
ENV_TRAFFIC_BYTES = 357.6e6  # step_kernel DRAM bytes per 65,536-env launch (ncu: 139.5 MB read + 218.1 MB write)
UNIT = 'decisions/s'
ENVS, HORIZON = 65536, 128
# Algorithmic bytes per decision of the env step (sim + bf16 observation write):
# 2*128 B compact state + 700 B bit-packed map + 8 B action + 5 B reward/done
# + 3,664 B observation.
ENV_BYTES_PER_DECISION = 969 + 3664
POLICY_FLOPS_PER_DECISION = 2 * (1832 * 256 + 256 * 256 + 256 * 13)
# Route-cue task (the reference's headline build): algorithmic bytes per decision
# = 2 x (64 B header + 280 B monster table + 840 B remembered plane) state read and
# written + 700 B bit-packed map + 8 B action + (421 + 9 + 8) x 4 B observation,
# mask and outcome row. The frontier list (read as far as it is long) is extra.
ROUTE_BYTES_PER_DECISION = 2 * (64 + 280 + 840) + 700 + 8 + (421 + 9 + 8) * 4


_T0 = time.perf_counter()


def progress(msg):
    """One line per phase on stderr (stdout carries only the JSON result)."""
    print(f'[bench {time.perf_counter() - _T0:7.1f}s] {msg}', file=sys.stderr, flush=True)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=128)
    ap.add_argument('--warmup', type=int, default=8)
    ap.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    ap.add_argument('--envs', type=int, default=ENVS, help='envs per GPU')
    ap.add_argument('--horizon', type=int, default=HORIZON, help='rollout slots (profiling runs shrink it)')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-ppo', action='store_true', help='skip the PPO-update measurement')
    ap.add_argument('--minibatch', type=int, default=16384)
    ap.add_argument('--exchange', choices=('auto', 'oneshot', 'twophase', 'nvls'), default='auto',
                    help='peer gradient exchange of the PPO update on several GPUs')
    ap.add_argument('--epochs', type=int, default=4)
    ap.add_argument('--no-cpu', action='store_true')
    ap.add_argument('--no-conv', action='store_true', help='skip the config-3 conv-policy rollout line')
    ap.add_argument('--conv-envs', type=int, default=131072, help='envs per GPU of the config-3 line')
    ap.add_argument('--conv-steps', type=int, default=16)
    ap.add_argument('--no-c4', action='store_true', help='skip the config-4 ogre-pressure iteration line')
    ap.add_argument('--c4-envs', type=int, default=131072, help='envs per GPU of the config-4 line')
    ap.add_argument('--c4-horizon', type=int, default=10,
                    help='rollout steps per config-4 iteration (131,072 x 10 x 8 GPUs = 10.5M decisions)')
    ap.add_argument('--no-ref-tasks', action='store_true',
                    help="skip the reference-task lines (route-cue and v1 on the GPU beside the reference's own "
                         'host build)')
    ap.add_argument('--no-route-ppo', action='store_true',
                    help="skip the route-cue task's PPO pipeline (the reference's benchmark loop) in the "
                         'reference-task lines')
    ap.add_argument('--no-ref-gpu', action='store_true',
                    help="skip timing the reference's own learn.cu GPU build in the reference-task lines")
    ap.add_argument('--route-envs', type=int, default=65536, help='envs per GPU of the route-cue line')
    ap.add_argument('--route-maps', type=int, default=16, help='maps in the route-cue corpus')
    ap.add_argument('--ref-cpu-envs', type=int, default=8192, help="envs of the reference build's host sample")
    ap.add_argument('--kernels', action='store_true',
                    help='run every hot kernel twice at bench sizes for profiler captures, print nothing else')
    return ap.parse_args()


class Clocks:
    """Sample SM clocks and throttle reasons with nvidia-smi during the timed region."""
    Q = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,'
         'clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,'
         'clocks_event_reasons.sw_power_cap')

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def start(self):
        try:
            self.proc = subprocess.Popen(['nvidia-smi', f'--id={self.index}', f'--query-gpu={self.Q}',
                                          '--format=csv,noheader,nounits', '-lms', '100'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(',')])

    def stop(self):
        if self.proc is None:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['nvidia-smi unavailable']}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:  # a sampler stuck in the driver must not hold the bench
            self.proc.kill()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                pass
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace('.', '').isdigit()]
        smax = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace('.', '').isdigit()]
        reasons = set()
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        for r in self.rows:
            if len(r) > 8:
                for name, v in zip(names, r[5:9]):
                    if v.strip().lower() == 'active':
                        reasons.add(name)
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(smax) if smax else None,
                'reasons': sorted(reasons), 'samples': len(sm)}


def peaks():
    try:
        return json.loads((REPO / 'MEASURED_PEAKS.json').read_text()), 'measured'
    except Exception:
        return {'hbm_gbs': 6650.0, 'bf16_tflops': 1590.0, 'bf16_tflops_sustained': 1400.0}, 'fallback'


# ---------------------------------------------------------------- CPU legs
def cpu_rollout(n_envs, steps, threads, warmup=1):
    """The oracle's spec env (C, one slice per thread) + a CPU torch policy of the
    same architecture: `warmup` untimed decisions, then `steps` timed ones.
    Returns (decisions/s, seconds)."""
    import numpy as np
    import torch
    sys.path.insert(0, str(REPO / 'oracle'))
    import oracle
    from d1.spec_env import DEFAULT
    oracle.build()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    w1 = torch.randn(256, 1832, generator=g) / 1832 ** 0.5
    w2 = torch.randn(256, 256, generator=g) / 16.0
    wh = torch.randn(13, 256, generator=g) / 16.0
    per = (n_envs + threads - 1) // threads
    envs = [oracle.OracleSpec(min(per, n_envs - i * per), DEFAULT, seed=0, first_env=i * per)
            for i in range(threads) if i * per < n_envs]
    from concurrent.futures import ThreadPoolExecutor
    pool = ThreadPoolExecutor(len(envs))
    actions = [np.zeros(e.batch, np.int64) for e in envs]

    def one_step(step):
        obs = torch.from_numpy(np.concatenate([e.obs for e in envs]))
        legal = np.concatenate([e.legal for e in envs])
        h = torch.relu(torch.relu(obs @ w1.T) @ w2.T) @ wh.T
        a, _ = oracle.sample_actions(h[:, :12].numpy(), legal, 0, step)
        off = 0
        for i, e in enumerate(envs):
            actions[i][:] = a[off:off + e.batch]
            off += e.batch
        list(pool.map(lambda i: envs[i].step(actions[i]), range(len(envs))))

    for s in range(warmup):
        one_step(s)
    t0 = time.perf_counter()
    for s in range(warmup, warmup + steps):
        one_step(s)
    dt = time.perf_counter() - t0
    pool.shutdown()
    return n_envs * steps / dt, dt


def legal_bits(mask):
    import numpy as np
    return ((np.asarray(mask) > 0) * (1 << np.arange(mask.shape[1]))).sum(1).astype(np.uint16)


def reference_host_rate(env, warmup, steps, threads, seed=7):
    """The reference's own learn.cu build (host path, learn_step(..., gpu=0)) over
    contiguous env slices on `threads` host threads (ctypes drops the GIL), with
    uniform legal actions from the oracle's sampler; warm-up steps, then `steps`
    timed steps. Returns (decisions/s, seconds)."""
    from concurrent.futures import ThreadPoolExecutor
    sys.path.insert(0, str(REPO / 'oracle'))
    import oracle
    n = env.batch
    per = (n + threads - 1) // threads
    slices = [(lo, min(n, lo + per)) for lo in range(0, n, per)]
    pool = ThreadPoolExecutor(len(slices))

    def one(k):
        a = oracle.sample_uniform_legal(legal_bits(env.mask), env.mask.shape[1], seed, k)
        list(pool.map(lambda sl: env.step(a, lo=sl[0], hi=sl[1]), slices))

    for k in range(warmup):
        one(k)
    t0 = time.perf_counter()
    for k in range(warmup, warmup + steps):
        one(k)
    dt = time.perf_counter() - t0
    pool.shutdown()
    return n * steps / dt, dt


def reference_tasks(args, dev, rank, world, stream):
    """The reference's own tasks on the GPU beside the reference's own host build
    of the same task on the host cores: the route-cue task (its headline PPO
    build, gpu-d1/PERFORMANCE.md:16) on a generated corpus, and the default v1
    task on the fixture map. A step = uniform legal actions (d1_sample_uniform_legal)
    + the env step, device-timed like the main line."""
    import torch
    import torch.distributed as dist
    from d1._lib import check, library
    from d1.learn_env import Env
    from d1.route_env import RouteEnv, generated_corpus
    lib = library()
    pk, pk_kind = peaks()
    cores = len(os.sched_getaffinity(0))
    out = {}
    maps = generated_corpus(args.route_maps, seed=11, device=dev)
    for name in ('route', 'v1'):
        n = args.route_envs
        if name == 'route':
            env = RouteEnv(n, 40, seed=1, maps=maps, device=dev)
            legal = env.legal
        else:
            env = Env(n, 8, seed=1, device=dev)
            legal = torch.zeros(n, dtype=torch.int16, device=dev)
        act = torch.zeros(n, dtype=torch.int64, device=dev)
        pow2 = (2 ** torch.arange(9, device=dev)).to(torch.float32)

        def step(k):
            if name == 'v1':  # the v1 wrapper returns a float mask only
                legal.copy_((env.mask @ pow2).to(torch.int16))
            check(lib.d1_sample_uniform_legal(legal.data_ptr(), 9, n, 7, k, rank * n, act.data_ptr(),
                                              stream.cuda_stream), 'd1_sample_uniform_legal')
            env.step(act)

        for k in range(args.warmup):
            step(k)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(args.warmup, args.warmup + args.steps):
            step(k)
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        # the env kernel alone, on its launching stream
        kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(8)]
        for a, b in kev:
            a.record(stream)
            env.step(act)
            b.record(stream)
        torch.cuda.synchronize()
        kms = sum(a.elapsed_time(b) for a, b in kev) / len(kev)
        line = {'decisions_per_s': n * world * args.steps / (t.item() / 1e3), 'unit': UNIT,
                'ms_per_step': t.item() / args.steps, 'envs_per_gpu': n, 'window_steps': [args.warmup,
                                                                                        args.warmup + args.steps],
                'kernel': 'd1::route::step_kernel' if name == 'route' else 'd1::v1::step_kernel',
                'kernel_ms': kms}
        if name == 'route':
            line['workload'] = ('route-cue task (reference flags of run_ring_ablations.py:141-157): 40 sleeping '
                                f'monsters, {args.route_maps}-map corpus (fixture + generated), uniform legal actions')
            ach = ROUTE_BYTES_PER_DECISION * n / (kms / 1e3) / 1e9
            line['roofline'] = {'bound': 'hbm', 'achieved': ach, 'peak': pk['hbm_gbs'], 'unit': 'GB/s',
                                'frac': ach / pk['hbm_gbs'], 'peak_kind': pk_kind,
                                'algorithmic_bytes_per_decision': ROUTE_BYTES_PER_DECISION}
        else:
            line['workload'] = 'v1 task (reference default build): fixture map, 8 monsters, uniform legal actions'
        if rank == 0 and not args.no_ref_gpu:
            r = reference_gpu_rate(name, env, args, dev, stream, n)
            if r is not None:
                line['reference_gpu_build'] = {
                    'value': r[0], 'unit': UNIT, 'ms_per_step': r[1],
                    'what': "the reference's own learn.cu of this task compiled for sm_100a (oracle/_ref), "
                            'its GPU path on this B200, same tables, envs and steps'}
                line['over_reference_gpu_build'] = (n / (t.item() / args.steps / 1e3)) / r[0]
        if rank == 0 and not args.no_cpu:
            sys.path.insert(0, str(REPO / 'oracle'))
            import oracle
            lib_ok = oracle.route_library() if name == 'route' else oracle.reference_library()
            if lib_ok is None:
                line['cpu_reference'] = {'unavailable': 'oracle/_ref was not built with the reference sources'}
            else:
                m = args.ref_cpu_envs
                if name == 'route':
                    ref = oracle.ReferenceRoute(m, oracle.route_corpus(args.route_maps, _spec_default(), seed=11),
                                                seed=1)
                else:
                    ref = oracle.ReferenceV1(m, 8, seed=1)
                rate, dt = reference_host_rate(ref, args.warmup, args.steps, cores)
                line['cpu_reference'] = {
                    'value': rate, 'unit': UNIT, 'cores': cores, 'kind': 'reference',
                    'sample': f'{m} envs x decisions {args.warmup}-{args.warmup + args.steps} ({dt:.1f} s), '
                              "the reference's learn.cu host path (oracle/_ref)"}
                line['gpu_over_cpu_reference'] = line['decisions_per_s'] / rate
        if name == 'route' and rank == 0 and not args.no_route_ppo:
            progress("route-cue PPO pipeline (the reference's benchmark loop)")
            pipe = {'what': "the reference's PPO benchmark loop restated (gpu-d1/scripts/benchmark_pipeline.py): "
                            'torch fp32 MLP 421-128-128 tanh, T=64 turns, 4 epochs of minibatch 4096; the env '
                            "under it is ours or the reference's own learn.cu GPU build on this B200; random "
                            'initialisation (the mature checkpoint is not available)',
                    'published_rtx5000_decisions_per_s': 153123, 'published_source': 'gpu-d1/PERFORMANCE.md:16'}
            for worlds in (512, 8192):
                for kind in ('ours', 'reference'):
                    r = route_ppo_pipeline(kind, maps, worlds, 64, 4, 2, dev)
                    if r is not None:
                        pipe[f'{kind}_{worlds}_worlds'] = r
            line['ppo_pipeline'] = pipe
        out[name] = line
        del env
    return out


def reference_gpu_rate(name, env, args, dev, stream, n):
    """The reference's own learn.cu of the task, compiled for sm_100a from the
    reference sources (oracle/_ref, the route build with its selected
    LEARN_BLOCK_SIZE=4), run through its own GPU path (learn_step(..., gpu=1))
    on this B200 with the same tables and uniform legal actions. Returns
    (decisions/s, ms per step) or None when the build is absent."""
    import ctypes as C
    import torch
    sys.path.insert(0, str(REPO / 'oracle'))
    import oracle
    from d1._lib import check, library
    lib = oracle.route_library() if name == 'route' else oracle.reference_library()
    if lib is None:
        return None
    if name == 'route':
        a = env.arrays
        tables = oracle.RouteTables(a[0].data_ptr(), a[1].data_ptr(), a[2].data_ptr(), a[3].data_ptr(),
                                    env.tables.ncells, a[4].data_ptr(), a[5].data_ptr(), env.n_maps, -1)
        nobs, limit = 421, 1024
    else:
        a = env.arrays
        tables = oracle.Tables(a[0].data_ptr(), a[1].data_ptr(), a[2].data_ptr(), a[3].data_ptr(), a[1].shape[0])
        nobs, limit = 206, 256
    state = torch.zeros((n, lib.learn_state_bytes()), dtype=torch.uint8, device=dev)
    obs = torch.empty((n, nobs), device=dev)
    mask = torch.empty((n, 9), device=dev)
    out = torch.empty((n, 8), device=dev)
    act = torch.zeros(n, dtype=torch.int64, device=dev)
    legal = torch.zeros(n, dtype=torch.int16, device=dev)
    pow2 = (2 ** torch.arange(9, device=dev)).to(torch.float32)
    s = stream.cuda_stream
    code = lib.learn_init(state.data_ptr(), n, C.byref(env.config), C.byref(tables), 1, obs.data_ptr(),
                          mask.data_ptr(), s, 1)
    if code:
        return None
    ulib = library()

    def step(k):
        legal.copy_((mask @ pow2).to(torch.int16))
        check(ulib.d1_sample_uniform_legal(legal.data_ptr(), 9, n, 7, k, 0, act.data_ptr(), s),
              'd1_sample_uniform_legal')
        lib.learn_step(state.data_ptr(), n, C.byref(env.config), C.byref(tables), act.data_ptr(), limit,
                       obs.data_ptr(), mask.data_ptr(), out.data_ptr(), s, 1)

    for k in range(args.warmup):
        step(k)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.warmup, args.warmup + args.steps):
        step(k)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    return n / (ms / 1e3), ms


def route_ppo_pipeline(kind, maps, B, T, updates, warmup, dev):
    """The reference's own PPO benchmark loop for the route-cue task, restated
    (gpu-d1/scripts/benchmark_pipeline.py; the loop of run_ring_ablations.py:
    332-372): its MLP policy (421 -> 128 tanh -> 128 tanh, actor 9, critic 1,
    fp32, TF32 off), T-turn rollouts of B worlds, GAE, 4 epochs of minibatch
    4096, clip 0.2, 0.25 MSE, entropy 0.01, grad-norm 0.5, Adam 3e-4. `kind`
    picks the env under it: 'ours' (libd1's route kernel) or 'reference' (the
    reference's own learn.cu of the task compiled for sm_100a, its GPU path).
    The mature checkpoint that benchmark starts from is not available, so the
    policy starts from the reference's initialisation. Returns the median
    decisions/s over `updates` timed updates."""
    import ctypes as C
    import math
    import torch
    from torch import nn
    from torch.distributions import Categorical, Distribution
    sys.path.insert(0, str(REPO / 'oracle'))
    import oracle
    from d1.route_env import RouteEnv
    Distribution.set_default_validate_args(False)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.manual_seed(0)
    env = RouteEnv(B, 40, seed=17, maps=maps, device=dev)
    if kind == 'reference':
        lib = oracle.route_library()
        if lib is None:
            return None
        a = env.arrays
        tables = oracle.RouteTables(a[0].data_ptr(), a[1].data_ptr(), a[2].data_ptr(), a[3].data_ptr(),
                                    env.tables.ncells, a[4].data_ptr(), a[5].data_ptr(), env.n_maps, -1)
        state = torch.zeros((B, lib.learn_state_bytes()), dtype=torch.uint8, device=dev)
        obs, mask, out = env.obs.clone(), env.mask.clone(), env.out.clone()
        s = torch.cuda.current_stream(dev).cuda_stream
        assert lib.learn_init(state.data_ptr(), B, C.byref(env.config), C.byref(tables), 17, obs.data_ptr(),
                              mask.data_ptr(), s, 1) == 0

        def step(act):
            lib.learn_step(state.data_ptr(), B, C.byref(env.config), C.byref(tables), act.data_ptr(), 1024,
                           obs.data_ptr(), mask.data_ptr(), out.data_ptr(), s, 1)
            return obs, out
    else:
        obs, mask = env.obs, env.mask
        step = env.step

    class Policy(nn.Module):
        def __init__(self):
            super().__init__()
            self.body = nn.Sequential(nn.Linear(421, 128), nn.Tanh(), nn.Linear(128, 128), nn.Tanh())
            self.actor, self.critic = nn.Linear(128, 9), nn.Linear(128, 1)
            for layer in self.modules():
                if isinstance(layer, nn.Linear):
                    nn.init.orthogonal_(layer.weight, math.sqrt(2))
                    nn.init.zeros_(layer.bias)
            nn.init.orthogonal_(self.actor.weight, .01)
            nn.init.orthogonal_(self.critic.weight, 1)

        def forward(self, o, m):
            h = self.body(o)
            return Categorical(logits=self.actor(h).masked_fill(m == 0, -1e9)), self.critic(h).squeeze(-1)

    model = Policy().to(dev)
    opt = torch.optim.Adam(model.parameters(), lr=3e-4, eps=1e-5)
    observations = torch.empty((T, B, 421), device=dev)
    masks = torch.empty((T, B, 9), device=dev)
    actions = torch.empty((T, B), dtype=torch.int64, device=dev)
    oldlp, values, rewards, dones, advantages = [torch.empty((T, B), device=dev) for _ in range(5)]

    def update():
        with torch.no_grad():
            for t in range(T):
                observations[t].copy_(obs)
                masks[t].copy_(mask)
                dist, v = model(obs, mask)
                act = dist.sample()
                actions[t] = act
                oldlp[t] = dist.log_prob(act)
                values[t] = v
                _, o = step(act)
                rewards[t] = o[:, 0]
                dones[t] = o[:, 1]
            _, nextv = model(obs, mask)
            gae = torch.zeros(B, device=dev)
            for t in reversed(range(T)):
                live = 1 - dones[t]
                delta = rewards[t] + .99 * nextv * live - values[t]
                gae = delta + .99 * .95 * live * gae
                advantages[t], nextv = gae, values[t]
            returns = (advantages + values).flatten()
            adv = advantages.flatten()
            adv = (adv - adv.mean()) / (adv.std() + 1e-8)
        for _ in range(4):
            for inds in torch.randperm(T * B, device=dev).split(4096):
                dist, v = model(observations.flatten(0, 1)[inds], masks.flatten(0, 1)[inds])
                ratio = (dist.log_prob(actions.flatten()[inds]) - oldlp.flatten()[inds]).exp()
                pg = -torch.minimum(ratio * adv[inds], ratio.clamp(.8, 1.2) * adv[inds]).mean()
                loss = pg + .25 * (v - returns[inds]).square().mean() - .01 * dist.entropy().mean()
                if not torch.isfinite(loss).item():
                    raise RuntimeError('Non-finite PPO loss')
                opt.zero_grad(set_to_none=True)
                loss.backward()
                nn.utils.clip_grad_norm_(model.parameters(), .5)
                opt.step()

    times = []
    for i in range(warmup + updates):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        update()
        torch.cuda.synchronize()
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return T * B / statistics.median(times)


def _spec_default():
    from d1.spec_env import DEFAULT
    return DEFAULT


def run_reference(args, rank, world):
    """`--impl reference`: the CPU implementation of this path timed on the host
    cores. The reference has no code for the BASELINE task, so this is the oracle
    port of it (the reference's own learn.cu host path covers only the fixture
    task); every host thread is used."""
    if rank != 0:
        return
    cores = len(os.sched_getaffinity(0))
    n = min(args.envs, 8192)
    rate, dt = cpu_rollout(n, args.steps, cores, warmup=args.warmup)
    line = {'impl': 'reference', 'metric': METRIC, 'value': rate, 'unit': UNIT, 'n_gpus': args.gpus,
            'steps': args.steps, 'warmup': args.warmup, 'higher_is_better': True, 'scaling': 'weak',
            'vs_baseline': None, 'dtype': 'f32', 'data': 'synthetic',
            'config': {'workload': 'config1 rollout: generated D:1 maps, MLP 1832-256-256-13, host CPU',
                       'envs_sampled': n},
            'cpu_baseline': {'value': rate, 'unit': UNIT, 'cores': cores, 'kind': 'port',
                             'sample': f'{n} envs x decisions {args.warmup}-{args.warmup + args.steps} '
                                       f'({dt:.1f} s)'},
            'e2e': {'value': rate, 'unit': UNIT, 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU leg
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from d1.policy import Policy
    from d1.rollout import Rollout
    from d1.spec_env import SpecEnv

    dev = torch.device('cuda', local_rank)
    torch.cuda.set_device(dev)
    B, T = args.envs, args.horizon
    env = SpecEnv(B, seed=1, first_env=rank * B, device=dev)
    policy = Policy(device=dev, seed=0)
    roll = Rollout(env, policy, T, seed=1)
    stream = torch.cuda.current_stream(dev)

    def step(k):
        t = k % T
        if t == 0 and k > 0:
            roll.roll()
        roll.step(t)

    progress('env + policy built; warm-up')
    for k in range(args.warmup):
        step(k)
    clocks = Clocks(local_rank)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(args.warmup, args.warmup + args.steps):
        step(k)
    roll.join()  # the env ranges' streams
    stop.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(stop)
    # Kernel-level timing of the env step for the roofline: the rollout's env
    # ranges overlap the policy on other streams, so the kernel is timed alone
    # here, whole batch per launch, with events on its launching stream,
    # continuing the same episodes with the rollout's last actions.
    def env_kernel_ms(k0):
        n_env = min(16, args.steps)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_env)]
        for i in range(n_env):
            ev[i][0].record(stream)
            env.step(roll.actions[(k0 + i) % T])
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev) / n_env

    env_ms = env_kernel_ms(args.warmup + args.steps)
    # A later window of the same rollout (episodes under way, many envs past
    # their first reset); the main window above is the driver's early one.
    k = args.warmup + args.steps
    k_late = max(k, 2 * T)
    while k < k_late:
        step(k)
        k += 1
    late_k = args.steps
    l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    l0.record(stream)
    for j in range(late_k):
        step(k + j)
    roll.join()
    l1.record(stream)
    torch.cuda.synchronize()
    tl = torch.tensor([l0.elapsed_time(l1)], device=dev)
    if world > 1:
        dist.all_reduce(tl, op=dist.ReduceOp.MAX)
    late_line = {'value': B * world * late_k / (tl.item() / 1e3), 'unit': UNIT, 'window_steps': [k, k + late_k],
                 'ms_per_step': tl.item() / late_k, 'env_kernel_ms': env_kernel_ms(k + late_k)}
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
    ms = t.item()
    value = B * world * args.steps / (ms / 1e3)

    # End to end through the public API with host buffers: every step copies the
    # actions in from pinned host memory, steps the env, runs the policy and
    # copies the outcome rows and the next actions back (d1.rollout.DecisionGraph:
    # the decision is one captured CUDA graph, replayed and synchronised per step).
    e2e = None
    if not args.no_e2e:
        from d1.rollout import DecisionGraph
        env.reset(2)
        dg = DecisionGraph(env, policy, seed=3, first_env=rank * B, step=0)
        # the same step range as the device-timed rollout: W warm-up decisions
        # after a reset, then K timed ones
        for k in range(max(3, args.warmup)):
            dg.replay()
            torch.cuda.synchronize()
            dg.h_act.copy_(dg.h_next)
        e2e_steps = args.steps
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for k in range(e2e_steps):
            dg.replay()
            torch.cuda.synchronize()
            dg.h_act.copy_(dg.h_next)
        e2e_s = torch.tensor([time.perf_counter() - t0], device=dev)
        if world > 1:
            dist.all_reduce(e2e_s, op=dist.ReduceOp.MAX)
        e2e = {'value': B * world * e2e_steps / e2e_s.item(), 'unit': UNIT,
               'h2d_bytes_per_step': B * 8, 'd2h_bytes_per_step': B * (env.out.shape[1] * 4 + 8),
               'steps': e2e_steps, 'streams': len(dg.ranges),
               'path': 'd1.rollout.DecisionGraph (captured decision, host copies inside)'}
        del dg
    progress('e2e done')
    from d1 import gemm as G
    x = roll.obs
    w1, b1 = policy.bf16['w1'], policy.params['b1']
    h1 = torch.empty((B, 256), dtype=torch.bfloat16, device=dev)
    for _ in range(3):
        G.gemm(x, w1, bias=b1, relu=True, out=h1)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    g0.record(stream)
    for i in range(reps):
        G.gemm(roll.obs, w1, bias=b1, relu=True, out=h1)  # 240 MB, larger than L2
    g1.record(stream)
    torch.cuda.synchronize()
    gemm_ms = g0.elapsed_time(g1) / reps
    gemm_tflops = 2.0 * B * 1832 * 256 / (gemm_ms / 1e3) / 1e12
    # PPO samples/s: full iteration = rollout of T steps +
    # GAE + epochs x (T*B / minibatch) minibatch updates, NCCL all-reduce of the
    # advantage statistics and of every minibatch gradient when world > 1.
    ppo_line = None
    if not args.no_ppo:
        from d1.ppo import PPO
        group = dist.group.WORLD if world > 1 else None
        trainer = PPO(policy, roll, minibatch=args.minibatch, epochs=args.epochs, group=group, exchange=args.exchange,
                      perm_seed=1234 + rank)
        roll.roll()
        progress('PPO warm-up iteration')
        trainer.iteration()  # warm-up iteration
        progress('PPO timed iteration')
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        p0, p1, p2, p3 = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        p0.record(stream)
        roll.collect()
        p1.record(stream)
        trainer.advantages()
        p2.record(stream)
        trainer.update()
        p3.record(stream)
        torch.cuda.synchronize()
        roll.roll()
        peer_error = trainer.lib.d1_peer_error() if trainer.peer is not None else 0
        exchange = None
        if world > 1:
            exchange = exchange_label(trainer)
        trainer.release()  # graph and exchange buffers go before the process group does
        it_ms = torch.tensor([p0.elapsed_time(p3)], device=dev)
        if world > 1:
            dist.all_reduce(it_ms, op=dist.ReduceOp.MAX)
        updates = args.epochs * (T * B // args.minibatch)
        ppo_line = {'samples_per_s': T * B * world / (it_ms.item() / 1e3), 'ms_per_iteration': it_ms.item(),
                    'rollout_ms': p0.elapsed_time(p1), 'gae_ms': p1.elapsed_time(p2),
                    'update_ms': p2.elapsed_time(p3), 'minibatch_ms': p2.elapsed_time(p3) / updates,
                    'samples_per_iteration': T * B * world, 'minibatch': args.minibatch, 'epochs': args.epochs,
                    'finite': bool(torch.isfinite(policy.flat).all().item()),
                    'gradient_exchange': exchange, 'peer_error': int(peer_error)}
    # centered-map conv policy with the autoregressive head,
    # 131,072 envs per GPU; a step = crop + conv stack + FC + head + AR sampling
    # + env step (no 1832-feature observation is written).
    conv_line = None
    if not args.no_conv:
        from d1.conv_policy import ConvPolicy, conv_error
        progress('config 3 conv rollout')
        n3 = args.conv_envs
        env3 = SpecEnv(n3, seed=3, first_env=rank * n3, device=dev, observe=False)
        pol3 = ConvPolicy(device=dev, seed=0)
        buf3 = pol3.buffers(n3)
        out3 = None
        for k in range(3):
            out3 = pol3.act(env3.state, env3.legal, n3, buf3, 3, k, rank * n3, out=out3)
            env3.step(out3['env_action'])
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        c0.record(stream)
        for k in range(args.conv_steps):
            last = k == args.conv_steps - 1
            pol3.encode(env3.state, n3, buf3)
            if last:
                f0.record(stream)
            pol3.features(buf3, n3)
            if last:
                f1.record(stream)
            out3 = pol3.act_from_features(env3.legal, n3, buf3, 3, 100 + k, rank * n3, out=out3)
            env3.step(out3['env_action'])
        c1.record(stream)
        torch.cuda.synchronize()
        t3 = torch.tensor([c0.elapsed_time(c1)], device=dev)
        if world > 1:
            dist.all_reduce(t3, op=dist.ReduceOp.MAX)
        feat_ms = f0.elapsed_time(f1)
        conv_flop = (5535360 + 8294400 + 3612672 + 3211264) * n3
        pk3, _ = peaks()
        conv_line = {'metric': 'env decisions/sec, centered-map conv policy + autoregressive head (config 3)',
                     'value': n3 * world * args.conv_steps / (t3.item() / 1e3), 'unit': UNIT,
                     'ms_per_step': t3.item() / args.conv_steps, 'envs_per_gpu': n3, 'steps': args.conv_steps,
                     'roofline': {'kernels': 'd1::conv::conv_kernel<1..3> + FC/head d1::tc::gemm_kernel',
                                  'bound': 'tensor', 'achieved': conv_flop / (feat_ms / 1e3) / 1e12,
                                  'peak': pk3['bf16_tflops'], 'unit': 'TFLOP/s',
                                  'frac': conv_flop / (feat_ms / 1e3) / 1e12 / pk3['bf16_tflops'],
                                  'flop_per_decision': conv_flop // n3, 'features_ms': feat_ms},
                     'conv_error': conv_error()}
        del env3, pol3, buf3, out3
    # the ogre-pressure scale-out scenario -- 131,072 envs per
    # GPU on maps with one sleeping ogre, the config-1 MLP, and a full iteration
    # (rollout of c4-horizon steps + GAE + 4-epoch PPO update with the gradient
    # exchange and global advantage statistics); decisions/s over the whole
    # iteration, all ranks.
    c4_line = None
    if not args.no_c4:
        from d1.ppo import PPO
        from d1.spec_env import OGRE
        progress('config 4 iteration')
        n4, t4 = args.c4_envs, args.c4_horizon
        env4 = SpecEnv(n4, config=OGRE, seed=4, first_env=rank * n4, device=dev)
        pol4 = Policy(device=dev, seed=0)
        roll4 = Rollout(env4, pol4, t4, seed=4)
        tr4 = PPO(pol4, roll4, minibatch=args.minibatch, epochs=args.epochs,
                  group=dist.group.WORLD if world > 1 else None, exchange=args.exchange, perm_seed=4321 + rank)
        tr4.iteration()  # warm-up iteration (also captures the update graph)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        q0, q1, q2 = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        q0.record(stream)
        roll4.collect()
        q1.record(stream)
        tr4.advantages()
        tr4.update()
        q2.record(stream)
        torch.cuda.synchronize()
        roll4.roll()
        peer_error4 = tr4.lib.d1_peer_error() if tr4.peer is not None else 0
        exchange4 = None
        if world > 1:
            exchange4 = exchange_label(tr4)
        tr4.release()
        t_it = torch.tensor([q0.elapsed_time(q2), q0.elapsed_time(q1)], device=dev)
        if world > 1:
            dist.all_reduce(t_it, op=dist.ReduceOp.MAX)
        decisions = n4 * t4 * world
        c4_line = {'metric': 'env decisions/sec over full rollout + GAE + PPO iterations (config 4, ogre maps)',
                   'value': decisions / (t_it[0].item() / 1e3), 'unit': UNIT,
                   'rollout_decisions_per_s': decisions / (t_it[1].item() / 1e3),
                   'ms_per_iteration': t_it[0].item(), 'rollout_ms': t_it[1].item(),
                   'decisions_per_iteration': decisions, 'envs_per_gpu': n4, 'horizon': t4,
                   'minibatch': args.minibatch, 'epochs': args.epochs,
                   'gradient_exchange': exchange4, 'peer_error': int(peer_error4),
                   'finite': bool(torch.isfinite(pol4.flat).all().item())}
        del env4, pol4, roll4, tr4
    ref_tasks = None
    if not args.no_ref_tasks:
        progress('reference tasks (route-cue, v1) beside the reference host build')
        ref_tasks = reference_tasks(args, dev, rank, world, stream)
    if rank != 0:
        return
    pk, pk_kind = peaks()
    achieved = ENV_BYTES_PER_DECISION * B / (env_ms / 1e3) / 1e9
    line = {
        'metric': METRIC, 'value': value, 'unit': UNIT, 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': ms / args.steps, 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'workload': 'config1 rollout: 65,536 envs/GPU on seeded generated 80x70 D:1 maps, '
                               'obs 1832 bf16, MLP 1832-256-256-13 (random N(0,1/fan_in)), masked sampling',
                   'envs_per_gpu': B, 'horizon': T, 'parallelism': f'dp{world} (env shards)',
                   'window_steps': [args.warmup, args.warmup + args.steps],
                   'rollout_streams': roll.parts,
                   'l2': 'inputs larger than L2 (240 MB obs slot + 134 MB env state per step)'},
        'roofline': {'kernel': 'd1::spec::step_kernel', 'bound': 'hbm', 'achieved': achieved,
                     'peak': pk['hbm_gbs'], 'unit': 'GB/s', 'frac': achieved / pk['hbm_gbs'],
                     # DRAM read + write of one launch at 65,536 envs, from one ncu
                     # capture of the kernel
                     'traffic': ENV_TRAFFIC_BYTES * B / 65536, 'traffic_unit': 'bytes per launch (ncu)',
                     'peak_kind': pk_kind,
                     'algorithmic_bytes_per_decision': ENV_BYTES_PER_DECISION,
                     'kernel_ms_per_step': env_ms},
        'roofline_policy_gemm': {'kernel': 'd1::tc::gemm_pair_kernel<2> (layer 1: M=%d, N=256, K=1832; 512-row 2-SM pair tiles)' % B,
                                 'bound': 'tensor', 'achieved': gemm_tflops, 'peak': pk['bf16_tflops'],
                                 'unit': 'TFLOP/s', 'frac': gemm_tflops / pk['bf16_tflops'],
                                 'ms_per_launch': gemm_ms, 'peak_kind': pk_kind + ' burst'},
        'late_window': late_line,
        'reference_tasks': ref_tasks,
        'ppo': ppo_line,
        'config3': conv_line,
        'config4': c4_line,
        'clocks': clk,
        'e2e': e2e,
        'gpu_launches': args.steps * 4 * roll.parts,
    }
    if not args.no_cpu:
        progress('CPU baseline')
        cores = len(os.sched_getaffinity(0))
        rate, dt = cpu_rollout(8192, args.steps, cores, warmup=args.warmup)
        line['cpu_baseline'] = {'value': rate, 'unit': UNIT, 'cores': cores, 'kind': 'port',
                                'sample': f'8192 envs x decisions {args.warmup}-{args.warmup + args.steps} of the '
                                          f'same workload ({dt:.1f} s)'}
    print(json.dumps(line), flush=True)


def exchange_label(trainer):
    """How a multi-GPU trainer exchanged its gradients."""
    pr = trainer.peer
    if pr is None:
        return 'NCCL'
    if pr.get('mc'):
        return 'peer memory (NVLink), one-shot read through NVLS multicast'
    return 'peer memory (NVLink), two-phase' if pr['two_phase'] else 'peer memory (NVLink), one-shot'


def run_kernels(args):
    """Every hot kernel once for warm-up and once more to be captured (ncu -k
    <kernel> -s <skip> -c <count>), at the bench's sizes, ~4 GB on the device.
    Launch order: an 8-step rollout of 65,536 envs (8 x (step_kernel, layer 1 on
    gemm_pair_kernel, layer 2 on gemm_kernel, head_sample_kernel), then the same
    two GEMMs + head_sample_kernel for the bootstrap value) and GAE; then per
    pass: rollout layer 1 (gemm_pair_kernel<2, 0>), one PPO minibatch of 16,384
    (layer 1 from compact rows gemm_pair_kernel<1, 1>; tail_kernel: layer 2,
    head, loss, dh2 and dh1; dW2 gemm_kernel; dW1 from compact rows
    gemm_pair_kernel<1, 2>; grad_reduce_kernel, adam_update_kernel), layer 2
    (gemm_kernel), head_sample_kernel, step_kernel, gae_scan_kernel, and the
    config-3 policy on 16,384 envs (crop_kernel, conv_kernel<1..3>, FC
    gemm_pair_kernel, head gemm_kernel, ar_kernel), then GAE over a [128, B]
    rollout of synthetic rewards and dones in the rollout's plane layout
    (gae_scan_kernel) and one route-cue env step of B envs on a 16-map
    corpus (d1::route::step_kernel, after 8 warm-up steps and their heuristic
    launches), and last the fused rollout policy (policy_tail_kernel: layer 2,
    head and draw from the pass's h1). A `gemm` regex therefore sees 18
    launches in the rollout and 7 per pass; `tail_kernel` (the PPO tail) one
    per pass; `policy_tail` one per pass; `gae_scan` one before the passes
    (the setup's, T = 8) and two per pass (T = 8, then T = 128); `route.*step`
    8 before the passes and one per pass."""
    import torch
    from d1 import gemm as G
    from d1.conv_policy import ConvPolicy
    from d1.policy import Policy
    from d1.ppo import PPO
    from d1.rollout import Rollout
    from d1.spec_env import SpecEnv
    torch.cuda.set_device(0)
    B = args.envs
    env = SpecEnv(B, seed=1)
    # the unfused layer 2 + head in the rollout part, so that the launch order
    # (and the -s offsets of the captures summarised in profiles/) stays fixed;
    # the fused policy tail runs once at the end of every pass
    pol = Policy(seed=0, tail=False)
    roll = Rollout(env, pol, 8, seed=1, parts=1)  # one stream: the launch order below is fixed
    roll.collect()
    tr = PPO(pol, roll, minibatch=args.minibatch, epochs=1, graph=False)
    tr.advantages()
    idx = torch.randperm(tr.total, device='cuda', generator=torch.Generator(device='cuda').manual_seed(0))[:tr.mb]
    x = roll.obs
    h1 = torch.empty((B, 256), dtype=torch.bfloat16, device='cuda')
    h2 = torch.empty((B, 256), dtype=torch.bfloat16, device='cuda')
    act = torch.empty(B, dtype=torch.int64, device='cuda')
    lp, val = torch.empty(B, device='cuda'), torch.empty(B, device='cuda')
    n3 = 16384
    env3 = SpecEnv(n3, seed=3, observe=False)
    cp = ConvPolicy(seed=0, chunk=n3)
    buf = cp.buffers(n3)
    from d1._lib import check, library
    from d1.route_env import RouteEnv, generated_corpus
    lib = library()
    g = torch.Generator(device='cuda').manual_seed(3)
    gae_out = torch.zeros((128, 10, B), device='cuda')
    gae_out[:, 0] = torch.randn((128, B), device='cuda', generator=g)
    gae_out[:, 1] = (torch.rand((128, B), device='cuda', generator=g) < 0.01).float()
    gae_val = torch.randn((129, B), device='cuda', generator=g)
    gae_adv, gae_ret = torch.empty((128, B), device='cuda'), torch.empty((128, B), device='cuda')
    gae_stats = torch.zeros(2, dtype=torch.float64, device='cuda')
    renv = RouteEnv(B, 40, seed=1, maps=generated_corpus(16, seed=11))
    for _ in range(8):
        renv.step(renv.heuristic().clone())
    torch.cuda.synchronize()
    for rep in range(2):
        G.gemm(x, pol.bf16['w1'], bias=pol.params['b1'], relu=True, out=h1)
        tr.minibatch(idx)
        G.gemm(h1, pol.bf16['w2'], bias=pol.params['b2'], relu=True, out=h2)
        pol.head(h2, env.legal, 1, rep, 0, act, lp, val)
        env.step(act)
        tr.advantages()
        cp.act(env3.state, env3.legal, n3, buf, 1, rep)
        check(lib.d1_gae(gae_out.data_ptr(), gae_out[:, 1].data_ptr(), gae_out.stride(0), 1, gae_val.data_ptr(),
                         128, B, 0.999, 0.95, gae_adv.data_ptr(), gae_ret.data_ptr(), gae_stats.data_ptr(), 1,
                         torch.cuda.current_stream().cuda_stream), 'd1_gae')
        renv.step(renv.heuristic().clone())
        pol.tail_sample(h1, env.legal, 1, rep, 0, act, lp, val)
        torch.cuda.synchronize()


def main():
    args = parse()
    if args.kernels:
        run_kernels(args)
        return
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    if args.impl == 'reference':
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=120))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    main()
