"""GPU parity of the spec task: CUDA kernels vs the CPU oracle, bit-exact on
observations (bf16 bit patterns), legal masks, outcomes, compact state and the
floor/remembered bit planes. Sizes follow BASELINE config 0 (1024 envs, uniform
random actions over the 12, 1000 steps) and the ogre scenario of config 4."""
import numpy as np
import pytest
import torch

import oracle
from golden.schedule import random_actions

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def spec():
    from d1 import spec_env
    oracle.build()
    return spec_env


def bf16_bits(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).view(torch.int16).numpy()


def assert_same(gpu, cpu, what, planes=False):
    g_obs = gpu.obs.view(torch.int16).cpu().numpy()
    c_obs = bf16_bits(cpu.obs)
    if not np.array_equal(g_obs, c_obs):
        bad = np.argwhere(g_obs != c_obs)
        raise AssertionError((what, 'obs', bad[:8].tolist()))
    assert np.array_equal(gpu.legal.cpu().numpy().view(np.uint16), cpu.legal), (what, 'legal')
    g_out, c_out = gpu.out.cpu().numpy(), cpu.out
    assert np.array_equal(g_out, c_out), (what, 'out', np.argwhere(g_out != c_out)[:8].tolist())
    g_c, c_c = gpu.compact().cpu().numpy(), cpu.compact()
    assert np.array_equal(g_c, c_c), (what, 'state', np.argwhere(g_c != c_c)[:8].tolist())
    if planes:
        gf, gv = gpu.planes()
        cf, cv = cpu.planes()
        assert np.array_equal(gf.cpu().numpy().view(np.uint32), cf), (what, 'floor')
        assert np.array_equal(gv.cpu().numpy().view(np.uint32), cv), (what, 'viewed')


def test_init_matches_oracle(spec):
    gpu, cpu = spec.SpecEnv(256, seed=7), oracle.OracleSpec(256, spec.DEFAULT, seed=7)
    assert_same(gpu, cpu, 'init', planes=True)


def test_config0_random_play_1024_envs_1000_steps(spec):
    n, steps = 1024, 1000
    gpu, cpu = spec.SpecEnv(n, seed=0), oracle.OracleSpec(n, spec.DEFAULT, seed=0)
    acts = random_actions(2024, steps, n, 12)
    dev = torch.from_numpy(acts).cuda()
    for k in range(steps):
        cpu.step(acts[k])
        gpu.step(dev[k].contiguous())
        if k < 20 or k % 50 == 49:
            assert_same(gpu, cpu, k, planes=(k % 200 == 199))
    assert_same(gpu, cpu, 'final', planes=True)


def test_ogre_scenario_matches_oracle(spec):
    n = 512
    gpu, cpu = spec.SpecEnv(n, config=spec.OGRE, seed=4), oracle.OracleSpec(n, spec.OGRE, seed=4)
    acts = random_actions(44, 300, n, 12)
    for k in range(300):
        cpu.step(acts[k])
        gpu.step(torch.from_numpy(acts[k]).cuda())
        if k % 30 == 29:
            assert_same(gpu, cpu, k)


def test_heuristic_like_play_with_rest_and_attack(spec):
    """Bias the action mix towards REST, attack-nearest and descend so the macro
    loop and semantic targeting are exercised heavily."""
    n = 512
    gpu, cpu = spec.SpecEnv(n, seed=9), oracle.OracleSpec(n, spec.DEFAULT, seed=9)
    base = random_actions(91, 300, n, 24)
    acts = np.where(base >= 12, np.array([9, 10, 11, 9, 10, 11, 9, 10, 11, 9, 10, 11])[base % 12], base)
    for k in range(300):
        cpu.step(acts[k])
        gpu.step(torch.from_numpy(acts[k]).cuda())
        if k % 25 == 24:
            assert_same(gpu, cpu, k)


def test_env_ids_shard_without_changing_trajectories(spec):
    a = spec.SpecEnv(64, seed=5)
    b = spec.SpecEnv(32, seed=5, first_env=32)
    acts = torch.from_numpy(random_actions(6, 40, 64, 12)).cuda()
    for k in range(40):
        a.step(acts[k].contiguous())
        b.step(acts[k, 32:].contiguous())
    assert torch.equal(a.compact()[32:], b.compact())
    assert torch.equal(a.obs[32:], b.obs)


def test_inactive_envs_are_untouched(spec):
    gpu, cpu = spec.SpecEnv(128, seed=1), oracle.OracleSpec(128, spec.DEFAULT, seed=1)
    active = torch.arange(128, device='cuda') % 3 != 0
    acts = random_actions(8, 30, 128, 12)
    for k in range(30):
        before = gpu.state.clone()
        gpu.step(torch.from_numpy(acts[k]).cuda(), active)
        assert torch.equal(gpu.state[~active], before[~active])
    # the active subset alone follows the oracle
    sub = oracle.OracleSpec(128, spec.DEFAULT, seed=1)
    act_np = active.cpu().numpy()
    for k in range(30):
        a = acts[k].copy()
        sub.step(a)  # oracle steps all; compare only the active rows below
    rows = gpu.compact().cpu().numpy()
    assert np.array_equal(rows[act_np], sub.compact()[act_np])


def test_compact_observation_expands_to_the_one_hot_observation(spec):
    """The compact observation (a channel byte per window cell + the 32 scalars)
    carries exactly the one-hot observation: its expansion -- in torch, and by the
    update's gather kernel with the ones column -- equals the env's obs bit for bit,
    at reset and after every step."""
    from d1._lib import library
    lib = library()
    n = 512
    env = spec.SpecEnv(n, seed=13)
    cobs = torch.empty((n, spec.COBS), dtype=torch.uint8, device='cuda')
    env.reset(13, cobs_out=cobs)
    acts = torch.from_numpy(random_actions(5, 40, n, 12)).cuda()
    idx = torch.randperm(n, device='cuda')
    x = torch.empty((n, 1840), dtype=torch.bfloat16, device='cuda')
    for k in range(41):
        if k:
            env.step(acts[k - 1].contiguous(), cobs_out=cobs)
        assert torch.equal(spec.expand_cobs(cobs).view(torch.int16), env.obs.view(torch.int16)), k
        assert lib.d1_ppo_gather_cobs(cobs.data_ptr(), idx.data_ptr(), n, x.data_ptr(), 1840, 1,
                                      torch.cuda.current_stream().cuda_stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(x[:, :1832].view(torch.int16), env.obs[idx].view(torch.int16)), k
        assert torch.equal(x[:, 1832:].float(), torch.tensor([1.] + [0.] * 7, device='cuda').expand(n, 8)), k
    assert torch.equal(cobs[:, 225:256], torch.zeros_like(cobs[:, 225:256]))


def test_bare_cuda_means_the_current_device():
    import torch
    from d1._lib import resolve_device, launch_stream
    from d1.spec_env import SpecEnv
    cur = torch.cuda.current_device()
    assert resolve_device('cuda') == torch.device('cuda', cur)
    env = SpecEnv(64, seed=2)
    assert env.device == torch.device('cuda', cur)
    assert launch_stream(env.device) == torch.cuda.current_stream().cuda_stream
