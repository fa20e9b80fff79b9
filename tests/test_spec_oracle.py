"""CPU checks of the spec-task oracle: its pinned parts against published or
reference vectors, its unpinned parts against their own invariants."""
import numpy as np
import pytest

import oracle
from golden.schedule import random_actions

SPEC = dict(hp=15, ac100=200, ev100=794, sh100=906, shield_limit=2, regen=23, gdr=(19, 21),
            min_monsters=3, max_monsters=10, min_mhp=2, max_mhp=8, ogre=0, ogre_hp=30, ogre_min_damage=2,
            limit=512, explore_milli=2, kill_milli=1000, descend_milli=3000, death_milli=1000,
            kinds=[(10, 3, 19, 15), (14, 3, 19, 15), (10, 1, 19, 15), (10, 4, 19, 15), (5, 17, 30, 25)])


def test_philox_known_answers(oracle_lib):
    """Random123 known-answer vectors for Philox4x32-10."""
    kat = [
        ([0, 0, 0, 0], [0, 0], [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]),
        ([0xffffffff] * 4, [0xffffffff] * 2, [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]),
        ([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0],
         [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]),
    ]
    for ctr, key, want in kat:
        assert list(oracle.philox(ctr, key)) == want


def test_los_matches_native_crawl_los_everywhere(oracle_lib):
    """The ray-fan LOS reproduces the native LOS table of the fixture map for all
    5600 origins (gpu-d1/scripts/compile_fixture.py:30-48 checks the same pairs)."""
    z = np.load(oracle.DATA / 'fixture_1057.npz')
    floor, native = z['floor'], z['native_los']
    for p in range(5600):
        assert np.array_equal(oracle.los_mask(floor, p), native[p]), p


def test_ray_fan_is_symmetric_on_the_fixture(oracle_lib):
    """Wake checks use the player's view; they equal the monster-origin view of the
    reference (semantic-actions-v1 learn.cu:199-205) because LOS is symmetric."""
    z = np.load(oracle.DATA / 'fixture_1057.npz')
    floor = z['floor']
    cells = np.flatnonzero(floor)[::7]
    masks = {int(p): oracle.los_mask(floor, int(p)) for p in cells}

    def vis(o, t):
        dx, dy = t % 80 - o % 80, t // 80 - o // 80
        if abs(dx) > 7 or abs(dy) > 7:
            return False
        b = (dy + 8) * 17 + dx + 8
        return bool((masks[o][b // 32] >> (b % 32)) & 1)
    for a in masks:
        for b in masks:
            assert vis(a, b) == vis(b, a)


def floor_cells(plane_row):
    bits = np.unpackbits(plane_row.astype('<u4').view(np.uint8), bitorder='little').reshape(70, 96)[:, :80]
    return bits.reshape(-1)


def components(fl):
    seen = np.zeros(5600, bool)
    comps = 0
    for s in np.flatnonzero(fl):
        if seen[s]:
            continue
        comps += 1
        stack = [s]
        seen[s] = True
        while stack:
            p = stack.pop()
            x, y = p % 80, p // 80
            for dx in (-1, 0, 1):
                for dy in (-1, 0, 1):
                    q = (y + dy) * 80 + x + dx
                    if 0 <= x + dx < 80 and 0 <= y + dy < 70 and fl[q] and not seen[q]:
                        seen[q] = True
                        stack.append(q)
    return comps


def test_generated_maps_are_connected_rooms_inside_a_wall_border(oracle_lib):
    env = oracle.OracleSpec(64, SPEC, seed=3)
    f, v = env.planes()
    rows = env.compact()
    for i in range(64):
        fl = floor_cells(f[i])
        grid = fl.reshape(70, 80)
        assert not grid[0].any() and not grid[-1].any() and not grid[:, 0].any() and not grid[:, -1].any()
        assert fl.sum() >= 16
        assert components(fl) == 1
        stairs, player, nmon = rows[i, 9], rows[i, 6], rows[i, 10]
        assert fl[stairs] and fl[player] and stairs != player
        assert 3 <= nmon <= 10
        pos = rows[i, 12:12 + nmon]
        assert all(fl[p] for p in pos) and len(set(pos)) == nmon and player not in pos
        hp = rows[i, 34:34 + nmon]
        assert ((hp >= 2) & (hp <= 8)).all()


def test_observation_is_one_hot_and_legal_bits_are_consistent(oracle_lib):
    env = oracle.OracleSpec(256, SPEC, seed=5)
    acts = random_actions(9, 60, 256, 12)
    for k in range(60):
        env.step(acts[k])
        cells = env.obs[:, :1800].reshape(256, 225, 8)
        assert (cells.sum(-1) == 1).all()
        assert (cells[:, 112, 3] + cells[:, 112, 4] == 1).all()  # the player's own cell is visible floor/stairs
        assert ((env.legal >> 8) & 1).all()  # wait is always legal
        o = env.out
        assert np.array_equal(o[:, 1], o[:, 2] + o[:, 6] + o[:, 7])
        assert (o[:, 8] >= 1).all()


def test_ogre_config_spawns_one_sleeping_ogre_far_away(oracle_lib):
    env = oracle.OracleSpec(64, dict(SPEC, ogre=1), seed=2)
    rows = env.compact()
    for r in rows:
        nmon = r[10]
        kinds = r[45:45 + nmon] // 2
        awake = r[45:45 + nmon] % 2
        if (kinds == 4).any():
            j = int(np.flatnonzero(kinds == 4)[0])
            p, player = r[12 + j], r[6]
            assert max(abs(p % 80 - player % 80), abs(p // 80 - player // 80)) >= 12
            assert r[34 + j] == 30 and awake[j] == 0


def test_oracle_is_deterministic_and_env_ids_are_independent(oracle_lib):
    a = oracle.OracleSpec(32, SPEC, seed=11)
    b = oracle.OracleSpec(16, SPEC, seed=11, first_env=16)
    acts = random_actions(3, 50, 32, 12)
    for k in range(50):
        a.step(acts[k])
        b.step(acts[k][16:])
    assert np.array_equal(a.compact()[16:], b.compact())
    assert np.array_equal(a.obs[16:], b.obs)


def test_oracle_slices_stepped_in_parallel_threads_match_one_run(oracle_lib):
    """The CPU baseline steps env slices from a thread pool (ctypes releases the
    GIL); the oracle must keep no shared scratch between calls."""
    from concurrent.futures import ThreadPoolExecutor
    from golden.schedule import random_actions
    n, per, steps = 128, 32, 40
    whole = oracle.OracleSpec(n, SPEC, seed=4)
    parts = [oracle.OracleSpec(per, SPEC, seed=4, first_env=i * per) for i in range(n // per)]
    acts = random_actions(8, steps, n, 12)
    with ThreadPoolExecutor(len(parts)) as pool:
        for k in range(steps):
            whole.step(acts[k])
            list(pool.map(lambda i: parts[i].step(acts[k][i * per:(i + 1) * per]), range(len(parts))))
    assert np.array_equal(np.concatenate([p.compact() for p in parts]), whole.compact())
    assert np.array_equal(np.concatenate([p.obs for p in parts]), whole.obs)
