"""GPU parity of the reference-compatible task: CUDA kernels vs the CPU oracle.

Mirrors gpu-d1/scripts/test_learning.py (CPU/CUDA exact parity on every buffer),
with the oracle as the CPU side and the reference's own golden digests."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from golden.schedule import random_actions

pytestmark = pytest.mark.gpu
GOLDEN = oracle.REPO / 'tests' / 'golden' / 'v1_trajectories.npz'


@pytest.fixture(scope='module')
def Env():
    from d1.learn_env import Env
    oracle.build()
    return Env


def gpu_digest(env):
    h = hashlib.sha256()
    for a in (env.obs, env.mask, env.out, env.compact()):
        h.update(np.ascontiguousarray(a.cpu().numpy()).tobytes())
    return np.frombuffer(h.digest(), np.uint8)


def assert_same(gpu, cpu, what):
    for f in ('obs', 'mask', 'out'):
        g, c = getattr(gpu, f).cpu().numpy(), getattr(cpu, f)
        assert np.array_equal(g, c), (what, f, np.argwhere(g != c)[:5])
    assert np.array_equal(gpu.compact().cpu().numpy(), cpu.compact()), (what, 'state')


def test_device_semantic_checks(Env):
    assert Env(4, 6, seed=0).semantic_test() == 0


def test_distance_table_matches_oracle(Env):
    env = Env(2, 1, seed=0)
    ref = oracle.fixture()[5]
    assert np.array_equal(env.arrays[3].cpu().numpy().view(np.uint16), ref)


@pytest.mark.parametrize('name', ['e1', 'e6', 'e8', 'r8'])
def test_reference_golden_trajectories(Env, name):
    g = np.load(GOLDEN)
    batch, enemies, seed, steps, heur = map(int, g[f'{name}_meta'])
    env = Env(batch, enemies, seed=seed)
    assert np.array_equal(gpu_digest(env), g[f'{name}_init'])
    rand = torch.from_numpy(random_actions(1000 + enemies + batch, steps, batch, 9)).cuda()
    for k in range(steps):
        a = env.heuristic().clone() if (heur and k % 2 == 0) else rand[k].contiguous()
        env.step(a)
        assert np.array_equal(gpu_digest(env), g[f'{name}_digests'][k]), (name, k)


@pytest.mark.parametrize('enemies', [1, 6, 8])
def test_mixed_actions_match_oracle_every_step(Env, enemies):
    gpu, cpu = Env(37, enemies, seed=91), oracle.OracleV1(37, enemies, seed=91)
    assert_same(gpu, cpu, 'init')
    rand = random_actions(31 + enemies, 300, 37, 9)
    for k in range(300):
        if k % 2:
            a = rand[k]
        else:
            a = cpu.heuristic().copy()
            assert np.array_equal(gpu.heuristic().cpu().numpy(), a), (k, 'heuristic')
        cpu.step(a)
        gpu.step(torch.from_numpy(a).cuda())
        assert_same(gpu, cpu, k)


def test_large_batch_random_play_matches_oracle(Env):
    n, steps = 4096, 200
    gpu, cpu = Env(n, 8, seed=7), oracle.OracleV1(n, 8, seed=7)
    rand = random_actions(99, steps, n, 9)
    for k in range(steps):
        cpu.step(rand[k])
        gpu.step(torch.from_numpy(rand[k]).cuda())
        if k % 20 == 19:
            assert_same(gpu, cpu, k)
    assert_same(gpu, cpu, 'final')


def test_inactive_worlds_stay_frozen(Env):
    gpu, cpu = Env(64, 8, seed=3), oracle.OracleV1(64, 8, seed=3)
    rand = random_actions(4, 100, 64, 9)
    active = np.arange(64) % 4 != 0
    act_t = torch.from_numpy(active).cuda()
    for k in range(100):
        before = gpu.state.clone()
        obs_before = gpu.obs.clone()
        gpu.step(torch.from_numpy(rand[k]).cuda(), act_t)
        cpu.step(rand[k], active)
        frozen = ~act_t
        assert torch.equal(gpu.state[frozen], before[frozen])
        assert torch.equal(gpu.obs[frozen], obs_before[frozen])
    assert_same(gpu, cpu, 'active')


def test_kernels_honor_the_callers_stream(Env):
    """gpu-d1/scripts/test_learning.py:62-70."""
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        a = Env(37, 6, seed=91)
        a.step(torch.full((37,), 8, dtype=torch.int64, device='cuda'))
        got = a.obs.clone()
    torch.cuda.synchronize()
    b = oracle.OracleV1(37, 6, seed=91)
    b.step(np.full(37, 8, np.int64))
    assert np.array_equal(got.cpu().numpy(), b.obs)


def test_empty_batch_is_a_no_op(Env):
    from d1._lib import library
    lib = library()
    env = Env(1, 1, seed=0)
    import ctypes as C
    assert lib.learn_step(None, 0, C.byref(env.config), C.byref(env.tables), None, 256, None, None, None,
                          env.stream, 1) == 0
