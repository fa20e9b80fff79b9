"""Multi-rank host logic on CPU with the gloo backend (world size 2).

The GPU path shards envs by global id and all-reduces two things: the
advantage statistics once per rollout and the flat gradient once per
minibatch. These tests check the three facts that design relies on, with the
CPU oracle and CPU torch standing in for the kernels:

* a shard of env ids [r*n, (r+1)*n) reproduces exactly those envs of one
  unsharded run (every env's stream is keyed by its global id);
* the mean of the ranks' per-minibatch mean gradients equals the gradient of
  the union minibatch when every rank uses the same minibatch size;
* all-reduced (sum, sum of squares, count) give the global mean and torch's
  unbiased std.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from golden.schedule import random_actions

SPEC = dict(hp=15, ac100=200, ev100=794, sh100=906, shield_limit=2, regen=23, gdr=(19, 21),
            min_monsters=3, max_monsters=10, min_mhp=2, max_mhp=8, ogre=1, ogre_hp=30, ogre_min_damage=2,
            limit=512, explore_milli=2, kill_milli=1000, descend_milli=3000, death_milli=1000,
            kinds=[(10, 3, 19, 15), (14, 3, 19, 15), (10, 1, 19, 15), (10, 4, 19, 15), (5, 17, 30, 25)])
N_PER, STEPS = 24, 60


def free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def worker(rank, world, port, results):
    import sys
    from pathlib import Path
    here = Path(__file__).resolve().parent
    for p in (here, here.parent / 'oracle'):
        sys.path.insert(0, str(p))
    import oracle as O
    from golden.schedule import random_actions as ra
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        # 1. env shards
        env = O.OracleSpec(N_PER, SPEC, seed=9, first_env=rank * N_PER)
        acts = ra(21, STEPS, N_PER * world, 12)
        for k in range(STEPS):
            env.step(acts[k][rank * N_PER:(rank + 1) * N_PER])
        rows = torch.from_numpy(env.compact())
        obs = torch.from_numpy(env.obs)
        gathered = [torch.empty_like(rows) for _ in range(world)]
        gathered_obs = [torch.empty_like(obs) for _ in range(world)]
        dist.all_gather(gathered, rows)
        dist.all_gather(gathered_obs, obs)
        # 2. gradient averaging over equal-size minibatches
        g = torch.Generator().manual_seed(0)
        w = torch.randn(16, 8, generator=g, dtype=torch.float64)
        x = torch.randn(world * 32, 8, generator=g, dtype=torch.float64)
        y = torch.randn(world * 32, 16, generator=g, dtype=torch.float64)
        wr = w.clone().requires_grad_(True)
        xs, ys = x[rank * 32:(rank + 1) * 32], y[rank * 32:(rank + 1) * 32]
        loss = ((xs @ wr.T - ys) ** 2).mean()
        loss.backward()
        grad = wr.grad.clone()
        dist.all_reduce(grad)
        grad /= world
        # 3. advantage statistics
        adv = torch.randn(world * 1000, generator=g, dtype=torch.float32)
        mine = adv[rank * 1000:(rank + 1) * 1000].double()
        stats = torch.tensor([mine.sum().item(), (mine * mine).sum().item()], dtype=torch.float64)
        dist.all_reduce(stats)
        if rank == 0:
            results['rows'] = torch.cat(gathered).numpy()
            results['obs'] = torch.cat(gathered_obs).numpy()
            results['grad'] = grad.numpy()
            results['stats'] = stats.numpy()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.fixture(scope='module')
def two_ranks(oracle_lib):
    oracle.spec_library()
    ctx = mp.get_context('spawn')
    manager = ctx.Manager()
    results = manager.dict()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    return dict(results)


def test_env_shards_reproduce_the_unsharded_run(two_ranks):
    full = oracle.OracleSpec(2 * N_PER, SPEC, seed=9)
    acts = random_actions(21, STEPS, 2 * N_PER, 12)
    for k in range(STEPS):
        full.step(acts[k])
    assert np.array_equal(two_ranks['rows'], full.compact())
    assert np.array_equal(two_ranks['obs'], full.obs)


def test_mean_of_rank_gradients_is_the_union_gradient(two_ranks):
    g = torch.Generator().manual_seed(0)
    w = torch.randn(16, 8, generator=g, dtype=torch.float64).requires_grad_(True)
    x = torch.randn(64, 8, generator=g, dtype=torch.float64)
    y = torch.randn(64, 16, generator=g, dtype=torch.float64)
    ((x @ w.T - y) ** 2).mean().backward()
    assert np.allclose(two_ranks['grad'], w.grad.numpy(), rtol=1e-12, atol=1e-12)


def test_all_reduced_advantage_statistics_give_global_normalisation(two_ranks):
    g = torch.Generator().manual_seed(0)
    torch.randn(16, 8, generator=g, dtype=torch.float64)
    torch.randn(64, 8, generator=g, dtype=torch.float64)
    torch.randn(64, 16, generator=g, dtype=torch.float64)
    adv = torch.randn(2000, generator=g, dtype=torch.float32)
    s1, s2 = two_ranks['stats']
    n = 2000.0
    mean = s1 / n
    std = np.sqrt((s2 - s1 * mean) / (n - 1))
    assert abs(mean - adv.double().mean().item()) < 1e-9
    assert abs(std - adv.double().std().item()) < 1e-9
