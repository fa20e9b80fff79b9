"""CPU checks of the oracle itself: pinned to the reference before it is trusted."""
import hashlib

import numpy as np
import pytest

import oracle
from golden.schedule import random_actions

GOLDEN = oracle.REPO / 'tests' / 'golden' / 'v1_trajectories.npz'


def digest(env):
    h = hashlib.sha256()
    for a in (env.obs, env.mask, env.out, env.compact()):
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), np.uint8)


def golden_runs():
    g = np.load(GOLDEN)
    names = sorted({k.split('_')[0] for k in g.files})
    return g, names


@pytest.mark.parametrize('name', ['e1', 'e6', 'e8', 'r8'])
def test_oracle_reproduces_reference_golden_trajectories(oracle_lib, name):
    """Golden digests were produced by the reference's own learn.cu host build."""
    g = np.load(GOLDEN)
    batch, enemies, seed, steps, heur = map(int, g[f'{name}_meta'])
    env = oracle.OracleV1(batch, enemies, seed=seed)
    assert np.array_equal(digest(env), g[f'{name}_init'])
    rand = random_actions(1000 + enemies + batch, steps, batch, 9)
    for k in range(steps):
        a = env.heuristic().copy() if (heur and k % 2 == 0) else rand[k]
        env.step(a)
        assert np.array_equal(digest(env), g[f'{name}_digests'][k]), (name, k)


def test_oracle_semantic_checks(oracle_lib):
    assert oracle.OracleV1(4, 6, seed=1).semantic_test() == 0


@pytest.mark.skipif(oracle.reference_library() is None, reason='reference host build not present')
def test_oracle_matches_reference_build_with_active_mask(oracle_lib):
    """Array-level equality with the reference build, including learn_step_active."""
    ref, orc = oracle.ReferenceV1(64, 8, seed=5), oracle.OracleV1(64, 8, seed=5)
    assert ref.semantic_test() == 0
    rand = random_actions(77, 200, 64, 9)
    active = (np.arange(64) % 3 != 0)
    for k in range(200):
        act = active if k % 4 == 1 else None
        ref.step(rand[k], act)
        orc.step(rand[k], act)
        for f in ('obs', 'mask', 'out'):
            assert np.array_equal(getattr(ref, f), getattr(orc, f)), (k, f)
        assert np.array_equal(ref.compact(), orc.compact()), k


def test_distance_table_matches_native_distance(oracle_lib):
    """Row of the fixture player's cell equals the native export's distance field."""
    header, _, floor, cells, index, distance = oracle.fixture()
    import numpy as _np
    native = _np.load(oracle.DATA / 'fixture_1057.npz')['native_dist']
    row = distance[index[int(header[0])]]
    assert _np.array_equal(row, native)


def test_invariants_hold_over_random_play(oracle_lib):
    """Invariants of gpu-d1/scripts/test_learning.py:19-36 on the compact state."""
    env = oracle.OracleV1(37, 8, seed=91)
    floor = oracle.fixture()[2]
    rand = random_actions(5, 300, 37, 9)
    for k in range(300):
        env.step(rand[k])
        o = env.out
        assert np.array_equal(o[:, 1], o[:, 2] + o[:, 6] + o[:, 7])
        if k % 25 == 0:
            rows = env.compact()
            for r in rows:
                hp, regen, player, ticks, killed = r[3], r[4], r[6], r[7], r[8]
                pos, energy, mhp = r[9:17], r[17:25], r[25:33]
                live = [i for i in range(8) if mhp[i] > 0]
                assert killed == 8 - len(live)
                assert 0 < hp <= 18 and 0 <= regen < 100 and 0 <= ticks < 256
                assert floor[player] and player not in [pos[i] for i in live]
                assert len({pos[i] for i in live}) == len(live)
                for i in range(8):
                    if i in live:
                        assert floor[pos[i]] and energy[i] < 80
                    else:
                        assert energy[i] == -30000
