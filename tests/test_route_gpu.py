"""Route-cue task on the GPU (d1_route_*, libd1_route.so) against the reference.

The oracle is the reference's own build of the task (gpu-d1/src/learn.cu with
the route-cue fast flags, oracle/_ref/learn_route.so, host path), directly where
it travelled with the repository and through its committed golden digests
otherwise. Parity is bit-exact: observations, masks, outcomes, the compact
state, the remembered plane and the frontier list in the reference's
swap-remove order, every step, with heuristic and uniform actions, 1, 8 and 40
monsters, episode ends of every kind and the multi-map draws. The route-cue
known answers of gpu-d1/src/test_route_cue.cu are mirrored on hand-built rows.
"""
import ctypes as C
import pathlib

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu
HERE = pathlib.Path(__file__).resolve().parent
GOLD = np.load(HERE / 'golden' / 'route_trajectories.npz')
W = 80


@pytest.fixture(scope='module')
def maps():
    from golden.make_golden_route import corpus
    return corpus()


def gpu_digest(env):
    from golden.make_golden_route import digest
    v, f = env.memory()
    return digest(env.obs.cpu().numpy(), env.mask.cpu().numpy(), env.out.cpu().numpy(), env.compact().cpu().numpy(),
                  v.cpu().numpy().view(np.uint32), f.cpu().numpy())


def schedule(name):
    from golden.schedule import random_actions
    batch, enemies, seed, steps, heur, mf = map(int, GOLD[f'{name}_meta'])
    return batch, enemies, seed, steps, bool(heur), mf, random_actions(2000 + enemies + batch, steps, batch, 9)


def test_generated_corpus_on_the_gpu_equals_the_oracle_corpus(maps):
    """The GPU-built corpus (spec generator floors, all-pairs BFS on the device)
    equals the host-built one the golden digests were made on."""
    from d1.route_env import generated_corpus
    from golden.make_golden_route import CORPUS
    got = generated_corpus(CORPUS['n_maps'], seed=CORPUS['seed'])
    assert len(got) == len(maps)
    for a, b in zip(got, maps):
        for x, y in zip(a, b):
            assert np.array_equal(np.asarray(x), np.asarray(y))


@pytest.mark.parametrize('name', ['h40', 'r1', 'h8'])
def test_trajectories_match_the_reference_golden_digests(maps, name):
    from d1.route_env import RouteEnv
    batch, enemies, seed, steps, heur, mf, rand = schedule(name)
    env = RouteEnv(batch, enemies, seed=seed, maps=maps, map_filter=mf)
    assert np.array_equal(gpu_digest(env), GOLD[f'{name}_init']), 'init'
    for k in range(steps):
        a = env.heuristic().clone() if (heur and k % 2 == 0) else torch.from_numpy(rand[k]).cuda()
        env.step(a)
        assert np.array_equal(gpu_digest(env), GOLD[f'{name}_digests'][k]), (name, k)


@pytest.mark.skipif(oracle.route_library() is None, reason='oracle/_ref/learn_route.so not present')
def test_stepwise_against_the_reference_build(maps):
    """Field by field against the reference build, 64 envs x 1100 steps (past
    the 1024-decision deadline), heuristic actions compared too."""
    from d1.route_env import RouteEnv
    from golden.schedule import random_actions
    n, steps = 64, 1100
    ref = oracle.ReferenceRoute(n, maps, enemies=40, seed=123)
    gpu = RouteEnv(n, 40, seed=123, maps=maps)
    rand = random_actions(77, steps, n, 9)
    kinds = np.zeros(3, np.int64)
    for k in range(steps + 1):
        np.testing.assert_array_equal(gpu.obs.cpu().numpy(), ref.obs, err_msg=f'obs step {k}')
        np.testing.assert_array_equal(gpu.mask.cpu().numpy(), ref.mask, err_msg=f'mask step {k}')
        np.testing.assert_array_equal(gpu.out.cpu().numpy(), ref.out, err_msg=f'out step {k}')
        np.testing.assert_array_equal(gpu.compact().cpu().numpy(), ref.compact(), err_msg=f'compact step {k}')
        v, f = gpu.memory()
        np.testing.assert_array_equal(v.cpu().numpy().view(np.uint32), ref.viewed_bits(), err_msg=f'viewed {k}')
        np.testing.assert_array_equal(f.cpu().numpy(), ref.frontier(), err_msg=f'frontier list step {k}')
        if k == steps:
            break
        if k % 3 == 0:
            a = ref.heuristic().copy()
            assert np.array_equal(gpu.heuristic().cpu().numpy(), a), f'heuristic step {k}'
        else:
            a = rand[k]
        ref.step(a)
        gpu.step(torch.from_numpy(a).cuda())
        kinds += ref.out[:, [2, 6, 7]].sum(0).astype(np.int64)  # clears, deaths, timeouts
    assert kinds[1] > 0 and kinds[2] > 0, kinds  # deaths and deadline ends both occurred


def test_inactive_envs_are_frozen(maps):
    """learn_step_active (learn.cu:666-670): inactive rows and buffers untouched;
    active envs step exactly as in an ordinary step (gpu-d1/scripts/
    test_fast_frontier.py:20-32)."""
    from d1.route_env import RouteEnv
    a = RouteEnv(32, 40, seed=456, maps=maps)
    b = RouteEnv(32, 40, seed=456, maps=maps)
    for _ in range(30):
        act = a.heuristic().clone()
        a.step(act)
        b.step(act)
    a.out.zero_()
    b.out.zero_()
    active = torch.arange(32, device='cuda') % 2 == 0
    before = [x.clone() for x in (b.state, b.obs, b.mask, b.out)]
    act = a.heuristic().clone()
    a.step(act)
    b.step(act, active=active)
    for old, got, want in zip(before, (b.state, b.obs, b.mask, b.out), (a.state, a.obs, a.mask, a.out)):
        assert torch.equal(got[~active], old[~active])
        assert torch.equal(got[active], want[active])


def test_route_cue_known_answers():
    """gpu-d1/src/test_route_cue.cu on hand-built rows through d1_route_observe:
    a detour around a known wall, an unseen shortcut (floor or not) that cannot
    change the cue, the same shortcut once seen, adjacent, at-target,
    unreachable and absent targets."""
    from d1._lib import library
    from d1.route_env import OBS, Tables
    lib = library()
    N = 5600
    floor = np.zeros(N, np.uint8)
    viewed = np.zeros(N, bool)
    player = 20 * W + 20

    def known(x, y):
        floor[y * W + x] = 1
        viewed[y * W + x] = True

    def row(targets):
        r = np.zeros(13312, np.uint8)
        hdr = r[24:56].view(np.int32)
        hdr[:] = [20, 0, 0, player, 0, 0, 0, len(targets)]
        bits = np.zeros((70, 3), np.uint32)
        vv = viewed.reshape(70, 80)
        for x in range(80):
            bits[:, x // 32] |= vv[:, x].astype(np.uint32) << np.uint32(x % 32)
        r[352:352 + 840] = bits.reshape(-1).view(np.uint8)
        r[2112:2112 + 2 * len(targets)] = np.asarray(targets, np.int16).view(np.uint8)
        return r

    cfg_vals = [1, 0, 20] + [0] * 32
    cfg = (C.c_int * 35)(*cfg_vals)
    zeros16 = torch.zeros(N, dtype=torch.int16, device='cuda')
    ncell = torch.tensor([N], dtype=torch.int32, device='cuda')
    off = torch.zeros(1, dtype=torch.int32, device='cuda')

    def cue(targets):
        f = torch.from_numpy(floor.copy()).cuda()
        st = torch.from_numpy(row(targets)).cuda().reshape(1, -1)
        t = Tables(f.data_ptr(), zeros16.data_ptr(), zeros16.data_ptr(), zeros16.data_ptr(), N, ncell.data_ptr(),
                   off.data_ptr(), 1, 0)
        obs = torch.zeros((1, OBS), device='cuda')
        mask = torch.zeros((1, 9), device='cuda')
        assert lib.d1_route_observe(st.data_ptr(), 1, C.byref(cfg), C.byref(t), obs.data_ptr(), mask.data_ptr(),
                                    None, torch.cuda.current_stream().cuda_stream) == 0
        return obs[0, 366 + 47:366 + 55].cpu().numpy()

    def check(target, expected):
        got = cue([target])
        want = np.array([float(d == expected) for d in range(8)], np.float32)
        assert np.array_equal(got, want), (target, expected, got)

    for x in range(18, 21):
        known(x, 20)
    for y in range(20, 25):
        known(18, y)
    for x in range(18, 25):
        known(x, 24)
    for y in range(20, 25):
        known(24, y)
    target = 20 * W + 24
    check(target, 3)
    for x in range(21, 24):
        floor[20 * W + x] = 1
    check(target, 3)
    for x in range(21, 24):
        known(x, 20)
    check(target, 1)
    check(player + 1, 1)
    check(player, -1)
    known(40, 40)
    check(40 * W + 40, -1)
    assert not cue([]).any()


def test_library_binds_like_the_reference_wrapper(maps):
    """libd1_route.so driven with the argument types of the reference's own
    wrapper (gpu-d1/scripts/learn_env_ring_multi.py:30-35, 97-111) steps
    exactly like RouteEnv."""
    from d1.route_env import RouteEnv
    path = pathlib.Path(__file__).resolve().parents[1] / 'dcss-auto_b200' / 'd1' / 'libd1_route.so'
    lib = C.CDLL(str(path))
    p, i = C.c_void_p, C.c_int
    lib.learn_init.argtypes = [p, i, p, p, C.c_uint64, p, p, p, i]
    lib.learn_step.argtypes = [p, i, p, p, p, i, p, p, p, p, i]
    lib.learn_heuristic.argtypes = [p, i, p, p, p, p, i]
    env = RouteEnv(96, 40, seed=9, maps=maps)
    # zeroed like RouteEnv's rows, so that the list slots past the count (stale
    # entries, as in the reference) compare equal too
    state = torch.zeros((96, lib.learn_state_bytes()), dtype=torch.uint8, device='cuda')
    obs = torch.empty((96, lib.learn_obs_size()), device='cuda')
    mask = torch.empty((96, lib.learn_action_size()), device='cuda')
    out = torch.empty((96, lib.learn_out_size()), device='cuda')
    act = torch.empty(96, dtype=torch.int64, device='cuda')
    s = torch.cuda.current_stream().cuda_stream
    assert lib.learn_init(state.data_ptr(), 96, C.byref(env.config), C.byref(env.tables), 9, obs.data_ptr(),
                          mask.data_ptr(), s, 1) == 0
    for k in range(200):
        assert lib.learn_heuristic(state.data_ptr(), 96, C.byref(env.config), C.byref(env.tables), act.data_ptr(),
                                   s, 1) == 0
        assert torch.equal(act, env.heuristic())
        assert lib.learn_step(state.data_ptr(), 96, C.byref(env.config), C.byref(env.tables), act.data_ptr(), 1024,
                              obs.data_ptr(), mask.data_ptr(), out.data_ptr(), s, 1) == 0
        env.step(act.clone())
        assert torch.equal(obs, env.obs) and torch.equal(out, env.out) and torch.equal(state, env.state), k
