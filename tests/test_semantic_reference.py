"""The BASELINE task's semantic rules against the reference's own semantic-actions
build (gpu-d1/branches/semantic-actions-v1/src/learn.cu, compiled for the host
with the flags of that branch's scripts/assets.py by `make -C oracle ref`),
driven from hand-built states on the fixture map through
oracle/semantic_harness.cu.

The two tasks share these rules, so each test builds the same situation in both
and compares what the rule decides:
- waking (learn.cu:199-205, 691-697): a sleeping monster wakes when the player
  is within six tiles and in the LOS seen from the monster's cell;
- attack-nearest (learn.cu:423-428): the weakest visible adjacent monster,
  first compass direction on ties;
- the legal set of wait, rest and attack-nearest (learn.cu:626-630);
- the rest macro (learn.cu:803-830): waits until full HP, an awake monster in
  view during a turn, or the end of the episode, with the physical deadline
  inside the macro; elapsed turns, HP, clock, reward, who woke, interruption;
- an invalid action costs one ordinary wait.

The reference side runs the reference's code; the other side is the CPU oracle
(and the GPU, for the cases that need no oracle-only hook). Monsters of spec
kind k sit in reference slot k + 6j, whose kind is c.kinds[slot % 6]. No roll of
either task's RNG (PCG there, Philox here) may decide anything compared: the
rest cases give every kind speed 9, so a monster that wakes (energy 70 + 9)
cannot act in the turn it wakes, and stays where it was seen; with speed 10 or
more it would take a step whose tie-break is a roll, and that step can take it
out of view.
"""
import ctypes as C

import numpy as np
import pytest

import oracle
from spec_cases import build, gpu_row, oracle_row

W, H, N = 80, 70, 5600
WAIT, REST, ATTACK = 8, 9, 10
LIMIT = 2048  # the semantic build's deadline


def reference(slow=False):
    if oracle.semantic_library() is None:
        pytest.skip('reference semantic-actions build not available (make -C oracle ref)')
    return oracle.SemanticReference(config(slow))


def config(slow=False):
    from d1.spec_env import DEFAULT
    # the semantic build's reward constants (assets.py:5) and deadline
    c = dict(DEFAULT, limit=LIMIT, kill_milli=1000, death_milli=4000, explore_milli=2)
    if slow:  # every kind at speed 9: no monster acts in the turn it wakes
        c['kinds'] = [(9,) + tuple(k[1:]) for k in c['kinds']]
    return c


def fixture_floor():
    return np.load(oracle.DATA / 'fixture_1057.npz')['floor']


def cheb(p, q):
    return max(abs(p % W - q % W), abs(p // W - q // W))


def neighbours(p):
    """Compass order N, E, S, W, NE, SE, SW, NW (sim.h:201-206)."""
    x, y = p % W, p // W
    out = []
    for dx, dy in ((0, -1), (1, 0), (0, 1), (-1, 0), (1, -1), (1, 1), (-1, 1), (-1, -1)):
        out.append((y + dy) * W + x + dx if 0 <= x + dx < W and 0 <= y + dy < H else -1)
    return out


class Ours:
    """A batch of hand-built spec-task states on the CPU oracle or on the GPU."""

    def __init__(self, backend, cases, slow=False):
        self.backend, self.n = backend, len(cases)
        cfg = config(slow)
        if backend == 'oracle':
            self.env = oracle.OracleSpec(self.n, cfg)
            self.env.state[:] = np.stack([oracle_row(c) for c in cases])
            lib = self.env.lib
            lib.oracle_spec_observe.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
            lib.oracle_spec_observe(self.env.state.ctypes.data, self.n, C.byref(self.env.config),
                                    self.env.obs.ctypes.data, self.env.legal.ctypes.data)
        else:
            import torch
            from d1.spec_env import SpecEnv
            self.torch = torch
            self.env = SpecEnv(self.n, config=cfg)
            self.env.state.copy_(torch.from_numpy(np.stack([gpu_row(c) for c in cases])).cuda())
            self.env.observe()

    @property
    def legal(self):
        if self.backend == 'oracle':
            return self.env.legal.astype(np.int64)
        return self.env.legal.cpu().numpy().astype(np.int64) & 0xffff

    def step(self, actions):
        a = np.asarray(actions, np.int64)
        if self.backend == 'oracle':
            self.env.step(a)
            return self.env.out.copy()
        self.env.step(self.torch.from_numpy(a).cuda())
        return self.env.out.cpu().numpy()

    def awake(self, i, m):
        """Awake flag of monster m of env i."""
        if self.backend == 'oracle':
            return int(self.env.state[i][137 + m])
        return int(self.env.state[i, 240 + m].item())


BACKENDS = ['oracle', pytest.param('gpu', marks=pytest.mark.gpu)]


def test_wake_rule_matches_reference_on_every_fixture_pair():
    """learn.cu:199-205: the reference asks the LOS of the monster's cell; the spec
    task asks the player's view. They agree for every floor pair within seven
    tiles of the fixture map."""
    ref = reference()
    floor = fixture_floor()
    cells = np.flatnonzero(floor)
    pairs = 0
    for p in cells:
        p = int(p)
        ref.empty(p, 10)
        los = oracle.los_mask(floor, p)
        for q in cells:
            q = int(q)
            if q == p or cheb(p, q) > 7:
                continue
            dx, dy = q % W - p % W, q // W - p // W
            bit = (dy + 8) * 17 + dx + 8
            ours = cheb(p, q) <= 6 and (int(los[bit // 32]) >> (bit % 32)) & 1 == 1
            assert ref.detects(q) == ours, (p, q)
            pairs += 1
    assert pairs > 40000


def test_wake_rule_holds_on_generated_maps():
    """On the BASELINE generator's maps the spec task's LOS is symmetric within
    six tiles, so waking from the player's view is the reference's rule (the
    LOS seen from the monster's cell) there too."""
    from d1.spec_env import DEFAULT
    fl, _ = oracle.OracleSpec(3, DEFAULT, seed=11).planes()
    for k in range(3):
        floor = oracle.floor_from_bits(fl[k])
        cells = [int(p) for p in np.flatnonzero(floor)]
        los = {p: oracle.los_mask(floor, p) for p in cells}

        def sees(a, b):
            dx, dy = b % W - a % W, b // W - a // W
            bit = (dy + 8) * 17 + dx + 8
            return (int(los[a][bit // 32]) >> (bit % 32)) & 1

        checked = 0
        for p in cells:
            for q in cells:
                if q != p and cheb(p, q) <= 6:
                    assert sees(p, q) == sees(q, p), (k, p, q)
                    checked += 1
        assert checked > 10000


def kinds_for(rng, k):
    """k spec kinds, at most four of each (reference slots kind + 6j < 24)."""
    return [int(v) for v in rng.permutation(np.repeat(np.arange(4), 4))[:k]]


def attack_cases(rng, count):
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    cases = []
    while len(cases) < count:
        p = cells[rng.integers(len(cells))]
        around = [q for q in neighbours(p) if q >= 0 and floor[q]]
        if not around:
            continue
        k = int(rng.integers(1, len(around) + 1))
        spots = [around[j] for j in rng.permutation(len(around))[:k]]
        far = [q for q in cells if cheb(p, q) == 2]
        if far and rng.random() < 0.5:
            spots.append(far[rng.integers(len(far))])
        spots = spots[:11]
        mons = [(q % W, q // W, int(rng.integers(1, 5)), kind, int(rng.random() < 0.5))
                for q, kind in zip(spots, kinds_for(rng, len(spots)))]
        cases.append((p, int(rng.integers(1, 16)), mons))
    return cases


def reference_state(ref, p, hp, mons, ticks=0):
    ref.empty(p, hp, ticks)
    used = {}
    slots = []
    for (x, y, mh, kind, awake) in mons:
        j = used.get(kind, 0)
        used[kind] = j + 1
        slot = kind + 6 * j
        assert slot < 24
        ref.put(slot, y * W + x, mh, awake)
        slots.append(slot)
    return slots


def spec_case(p, hp, mons, ticks=0):
    floor = fixture_floor()
    cells = np.flatnonzero(floor)
    taken = {p} | {y * W + x for (x, y, *_r) in mons}
    stairs = next(int(q) for q in cells[::-1] if int(q) not in taken and cheb(int(q), p) > 8)
    return build(player=(p % W, p // W), hp=hp, ticks=ticks, mons=mons, floor=floor,
                 stairs=(stairs % W, stairs // W))


def test_attack_target_matches_reference():
    """learn.cu:423-428 on 400 random neighbourhoods (HP ties are common)."""
    ref = reference()
    rng = np.random.default_rng(3)
    lib = oracle.spec_library()
    lib.oracle_spec_attack_dir.argtypes = [C.c_void_p]
    for p, hp, mons in attack_cases(rng, 400):
        reference_state(ref, p, hp, mons)
        row = oracle_row(spec_case(p, hp, mons))
        assert lib.oracle_spec_attack_dir(row.ctypes.data) == ref.attack_dir(), (p, mons)


@pytest.mark.parametrize('backend', BACKENDS)
def test_legal_wait_rest_attack_match_reference(backend):
    """learn.cu:626-630: attack legal iff a visible monster is adjacent, wait
    always, rest iff HP is below full, regeneration is on and no awake monster
    is in view -- on 400 random states with sleeping and awake monsters."""
    ref = reference()
    rng = np.random.default_rng(4)
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    cases = attack_cases(rng, 200)
    while len(cases) < 400:  # monsters anywhere within eight tiles, none adjacent
        p = cells[rng.integers(len(cells))]
        near = [q for q in cells if 2 <= cheb(p, q) <= 8]
        spots = [near[j] for j in rng.permutation(len(near))[:int(rng.integers(0, 6))]]
        mons = [(q % W, q // W, int(rng.integers(1, 9)), kind, int(rng.random() < 0.4))
                for q, kind in zip(spots, kinds_for(rng, len(spots)))]
        cases.append((p, int(rng.integers(1, 16)), mons))
    want = []
    for p, hp, mons in cases:
        reference_state(ref, p, hp, mons)
        m = ref.observe()
        want.append((int(m[0]), int(m[3]), int(m[4])))
    ours = Ours(backend, [spec_case(p, hp, mons) for p, hp, mons in cases])
    legal = ours.legal
    for i, (att, wait, rest) in enumerate(want):
        got = ((legal[i] >> ATTACK) & 1, (legal[i] >> WAIT) & 1, (legal[i] >> REST) & 1)
        assert got == (att, wait, rest), (i, cases[i])


def rest_cases(rng, count):
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    cases = []
    while len(cases) < count:
        p = cells[rng.integers(len(cells))]
        near = [q for q in cells if 2 <= cheb(p, q) <= 9]
        spots = [near[j] for j in rng.permutation(len(near))[:int(rng.integers(0, 6))]]
        mons = [(q % W, q // W, int(rng.integers(1, 9)), kind, 0) for q, kind in zip(spots, kinds_for(rng, len(spots)))]
        ticks = int(rng.integers(LIMIT - 60, LIMIT)) if rng.random() < 0.2 else int(rng.integers(0, 1000))
        cases.append((p, int(rng.integers(1, 15)), mons, ticks))
    return cases


@pytest.mark.parametrize('backend', BACKENDS)
def test_rest_macro_matches_reference(backend):
    """learn.cu:803-830 on 300 random rests among sleeping monsters at two to nine
    tiles (some within six tiles in view, which wake and interrupt), 20 % of
    them near the 2048-turn deadline: elapsed turns, total reward, HP, clock,
    done/timeout, interruption and each monster's awake flag."""
    ref = reference(slow=True)
    rng = np.random.default_rng(5)
    cases = rest_cases(rng, 300)
    want = []
    for p, hp, mons, ticks in cases:
        slots = reference_state(ref, p, hp, mons, ticks)
        o = ref.step(oracle.SEM_REST, LIMIT)
        awake = [ref.field('awake', s) for s in slots]
        want.append((o, awake))
    ours = Ours(backend, [spec_case(p, hp, mons, ticks) for p, hp, mons, ticks in cases], slow=True)
    out = ours.step([REST] * len(cases))
    woke = interrupted = deadline = 0
    for i, (o, awake) in enumerate(want):
        g = out[i]
        ctx = (i, cases[i])
        assert g[8] == o[26], ctx  # elapsed primitive turns
        assert np.float32(g[0]) == np.float32(o[0]), ctx  # total reward
        assert g[1] == o[1] and g[7] == o[7] and g[6] == o[6], ctx  # done, timeout, death
        assert g[9] == o[38], ctx  # invalid
        if not o[1]:  # a finished episode resets both states
            assert g[4] == o[4] and g[5] == o[5], ctx  # HP, clock
            assert [ours.awake(i, m) for m in range(len(awake))] == awake, ctx
        assert (not g[1] and not g[9] and g[4] < config()['hp']) == bool(o[37]), ctx  # interrupted
        woke += any(awake)
        interrupted += bool(o[37])
        deadline += bool(o[7])
    assert woke > 20 and interrupted > 20 and deadline > 10, (woke, interrupted, deadline)


@pytest.mark.parametrize('backend', BACKENDS)
def test_invalid_actions_cost_one_wait_like_reference(backend):
    """learn.cu:814-815: attack-nearest with no visible adjacent monster, and rest at
    full HP, are one ordinary wait turn (the clock, HP and reward of a wait)."""
    ref = reference()
    rng = np.random.default_rng(6)
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    cases, actions, want = [], [], []
    for k in range(100):
        p = cells[rng.integers(len(cells))]
        hp = config()['hp'] if k % 2 else int(rng.integers(1, 15))
        ticks = int(rng.integers(0, 1000))
        a, ref_a = (REST, oracle.SEM_REST) if k % 2 else (ATTACK, oracle.SEM_ATTACK)
        reference_state(ref, p, hp, [], ticks)
        o = ref.step(ref_a, LIMIT)
        want.append(o)
        cases.append(spec_case(p, hp, [], ticks))
        actions.append(a)
    out = Ours(backend, cases).step(actions)
    for i, o in enumerate(want):
        g = out[i]
        assert o[38] or actions[i] == ATTACK  # the reference flags an invalid rest
        assert g[9] == 1 and g[8] == 1 == o[26], i
        assert g[4] == o[4] and g[5] == o[5] and np.float32(g[0]) == np.float32(o[0]), i


@pytest.mark.parametrize('backend', BACKENDS)
def test_steps_and_reveal_match_reference(backend):
    """The one-turn primitive of a lone player (learn.cu:638-700): a step onto floor
    or a bump into a wall, then the LOS-gated 15x15 reveal (learn.cu:296-331) --
    every in-view cell remembered, every newly seen floor cell paying the explore
    reward. 64 players walk 150 random compass steps from random fixture cells;
    each turn's reward, the position, HP, clock and seen-floor count must agree,
    and at the end the remembered plane cell for cell."""
    ref = reference()
    rng = np.random.default_rng(7)
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    n, T = 64, 150
    starts = [cells[rng.integers(len(cells))] for _ in range(n)]
    hps = [int(rng.integers(1, 16)) for _ in range(n)]
    moves = rng.integers(0, 8, (T, n))
    want_out = np.zeros((T, n, 4), np.float64)
    want_viewed = np.zeros((n, N), np.uint8)
    for i in range(n):
        ref.empty(starts[i], hps[i])
        for t in range(T):
            o = ref.primitive(int(moves[t, i]), LIMIT)
            want_out[t, i] = (o[0], ref.field('player'), o[4], ref.field('floor_seen'))
            assert o[5] == t + 1
        want_viewed[i] = ref.viewed()
    ours = Ours(backend, [spec_case(starts[i], hps[i], []) for i in range(n)])
    moved = 0
    for t in range(T):
        out = ours.step(moves[t])
        if backend == 'oracle':
            rows = ours.env.compact()
        else:
            rows = ours.env.compact().cpu().numpy()
        got = np.stack([out[:, 0], rows[:, 6], out[:, 4], rows[:, 11]], axis=1)
        assert np.array_equal(out[:, 5], np.full(n, t + 1)), t
        for i in range(n):
            assert np.float32(got[i, 0]) == np.float32(want_out[t, i, 0]), (t, i)
            assert tuple(got[i, 1:]) == tuple(want_out[t, i, 1:]), (t, i)
        moved += int((want_out[t, :, 0] > 0).sum())
    if backend == 'oracle':
        _, viewed = ours.env.planes()
    else:
        viewed = ours.env.planes()[1].cpu().numpy().view(np.uint32)
    for i in range(n):
        assert np.array_equal(oracle.floor_from_bits(viewed[i]), want_viewed[i]), i
    assert moved > 200  # turns that revealed new floor


def test_window_channels_match_reference_observation():
    """The spec task's one-hot window (oracle_spec_observe) against the same
    information in the semantic build's observation (learn.cu:451-479): for
    every cell of the 15x15 window, unknown / remembered wall / remembered floor
    out of view / visible floor equal the build's memory value (0, -1, 1) and
    its in-view plane, and a visible monster shows as asleep or awake exactly
    where the build shows its hp and its slot's sleep flag. 48 players walk 60
    random steps from random fixture cells (memory built by the reveal both
    tasks share), then up to 10 monsters are placed within seven tiles."""
    ref = reference()
    rng = np.random.default_rng(9)
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    n, T = 48, 60
    starts = [cells[rng.integers(len(cells))] for _ in range(n)]
    moves = rng.integers(0, 8, (T, n))
    ours = Ours('oracle', [spec_case(starts[i], 15, []) for i in range(n)])
    for t in range(T):
        ours.step(moves[t])
    rows = ours.env.compact()
    env = ours.env
    checked = {0: 0, 1: 0, 2: 0, 3: 0, 5: 0, 6: 0}
    for i in range(n):
        ref.empty(starts[i], 15)
        for t in range(T):
            ref.primitive(int(moves[t, i]), LIMIT)
        p = ref.field('player')
        assert p == rows[i, 6]
        px, py = p % W, p // W
        near = [q for q in cells if 1 <= cheb(p, q) <= 7 and q != rows[i, 9]]
        spots = [near[j] for j in rng.permutation(len(near))[:int(rng.integers(0, 11))]]
        kinds = kinds_for(rng, len(spots))
        mons = [(q, int(rng.integers(1, 9)), k, int(rng.random() < 0.5)) for q, k in zip(spots, kinds)]
        used, slots = {}, []
        for q, hp, k, awake in mons:
            j = used.get(k, 0)
            used[k] = j + 1
            ref.put(k + 6 * j, q, hp, awake)
            slots.append(k + 6 * j)
        row = env.state[i]  # the oracle's row layout (tests/spec_cases.oracle_row)
        row[24 + 4 * 7:24 + 4 * 8].view(np.int32)[0] = len(mons)
        for m, (q, hp, k, awake) in enumerate(mons):
            row[60 + 2 * m:62 + 2 * m].view(np.int16)[0] = q
            row[82 + 2 * m:84 + 2 * m].view(np.int16)[0] = -30000
            row[104 + 2 * m:106 + 2 * m].view(np.int16)[0] = hp
            row[126 + m], row[137 + m] = k, awake
        env.lib.oracle_spec_observe(row.ctypes.data, 1, C.byref(env.config), env.obs[i].ctypes.data,
                                    env.legal[i:i + 1].ctypes.data)
        ref.observe()
        o = ref.obs
        mon_at = {q: (hp, awake, s) for (q, hp, k, awake), s in zip(mons, slots)}
        for dy in range(-7, 8):
            for dx in range(-7, 8):
                j = (dy + 7) * 15 + dx + 7
                x, y = px + dx, py + dy
                q = y * W + x
                if not (0 <= x < W and 0 <= y < 70) or q == rows[i, 9]:
                    continue
                ch = int(np.argmax(env.obs[i, 8 * j:8 * j + 8]))
                mem, vis, mhp = o[j], o[733 + j], o[225 + j]
                if mhp > 0:
                    hp, awake, s = mon_at[q]
                    slot = ref.field('enemy_slot', s)  # the sleep flag sits at the monster's discovery slot
                    assert mhp == np.float32(hp / 16.0) and o[959 + slot] == (-1.0 if awake else 1.0), (i, q)
                    want = 6 if awake else 5
                elif mem == 0:
                    want = 0
                elif mem == -1:
                    want = 1
                else:
                    want = 3 if vis else 2
                assert ch == want, (i, dx, dy, ch, mem, vis, mhp)
                checked[want] += 1
    assert min(checked[c] for c in (0, 1, 2, 3)) > 400 and min(checked[5], checked[6]) > 15, checked


@pytest.mark.parametrize('backend', BACKENDS)
def test_death_ends_the_episode_with_the_penalty_like_reference(backend):
    """gpu-d1/src/test_combat_ablations.cu:17-21 on both tasks: a player at -100
    HP who waits dies that turn -- done and death set, not a timeout, the
    reward one wait minus the death penalty (the semantic build's DEATH_MILLI
    4000, the spec config set to the same), HP reported as 0 -- and the episode
    resets."""
    ref = reference()
    rng = np.random.default_rng(10)
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    cases, want = [], []
    for k in range(40):
        p = cells[rng.integers(len(cells))]
        ticks = int(rng.integers(0, 1000))
        reference_state(ref, p, -100, [], ticks)
        o = ref.step(oracle.SEM_WAIT, LIMIT)
        assert o[1] == 1 and o[6] == 1 and o[7] == 0 and o[4] == 0
        assert ref.field('hp') == config()['hp'] and ref.field('ticks') == 0  # reset
        want.append(o)
        cases.append(spec_case(p, -100, [], ticks))
    out = Ours(backend, cases).step([WAIT] * len(cases))
    for i, o in enumerate(want):
        g = out[i]
        assert g[1] == 1 and g[6] == 1 and g[7] == 0 and g[4] == 0, i
        assert np.float32(g[0]) == np.float32(o[0]), (i, g[0], o[0])
