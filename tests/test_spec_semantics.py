"""The BASELINE task's semantic actions against the expected values of the
reference's own semantic self-test (gpu-d1/branches/semantic-actions-v1/src/
semantic_tests.cu:12-45), on hand-built states, on the CPU oracle and on the
GPU (the same cases; the GPU run is marked gpu).

Mapping of the reference's five actions onto the spec task's twelve:
ATTACK (0) -> attack-nearest (10), WAIT (3) -> wait (8), REST (4) -> rest (9).
EXPLORE (1) and ENGAGE (2) are not in the spec action set, so their two
assertions (semantic_tests.cu:34-38) have no counterpart here. The duration-
discounted reward out[40] has no counterpart either (the spec outcome row has
no discounted column); the undiscounted total and the elapsed turns are
checked. Every other assertion is mirrored with the reference's expected
values: the isolated player's legal set, REST equal to repeated primitive waits
(state byte for byte, reward, duration, clock scalar), a sleeping foe at seven
tiles that permits rest and stays asleep, one at six tiles that wakes and
interrupts after one turn, the physical deadline inside a rest macro, ATTACK as
one primitive with the weakest visible target and compass ties, and an invalid
action costing one ordinary wait.
"""
import numpy as np
import pytest

from spec_cases import OracleCase, GpuCase, build

REST, WAIT, ATTACK, DESCEND = 9, 8, 10, 11
W = 80


def config():
    from d1.spec_env import DEFAULT
    return dict(DEFAULT, limit=2048)  # the reference test's 2048-turn deadline


BACKENDS = ['oracle', pytest.param('gpu', marks=pytest.mark.gpu)]


def make(backend, case):
    return (GpuCase if backend == 'gpu' else OracleCase)(case, config())


def bit(legal, a):
    return (legal >> a) & 1


@pytest.mark.parametrize('backend', BACKENDS)
def test_isolated_rest_equals_primitive_waits(backend):
    cfg = config()
    base = build(hp=3)
    env = make(backend, base)
    L = env.legal
    # semantic_tests.cu:13-14: alone at 3 HP -- rest and wait legal, attack not
    assert bit(L, REST) and bit(L, WAIT) and not bit(L, ATTACK) and not bit(L, DESCEND)
    macro, manual = make(backend, base), make(backend, base)
    out = macro.step(REST)
    count, reward = 0, np.float32(0)
    while True:  # semantic_tests.cu:17
        o = manual.step(WAIT)
        count += 1
        reward = np.float32(reward + o[0])
        if manual.compact()[3] >= cfg['hp']:
            break
    # semantic_tests.cu:18-19: same reward, duration, state byte for byte
    assert out[8] == count and out[0] == reward and out[9] == 0 and out[1] == 0, (out, count, reward)
    assert np.array_equal(macro.row, manual.row)
    assert macro.compact()[7] == count
    # semantic_tests.cu:20: no rest at full HP; the clock scalar reads count / 2048
    assert not bit(macro.legal, REST)
    assert macro.obs()[1800 + 2] == np.float32(count / 2048.0)


@pytest.mark.parametrize('backend', BACKENDS)
def test_sleeping_foe_at_seven_tiles_permits_rest_and_stays_asleep(backend):
    isolated = make(backend, build(hp=3))
    isolated.step(REST)
    full = int(isolated.compact()[7])
    env = make(backend, build(hp=3, mons=[(47, 35, 8, 0, 0)]))  # semantic_tests.cu:22
    assert bit(env.legal, REST) and not bit(env.legal, ATTACK)
    out = env.step(REST)
    c = env.compact()
    assert out[8] == full and c[3] == config()['hp'] and out[1] == 0  # rested to full, not interrupted
    assert c[12 + 33] & 1 == 0  # kind * 2 + awake of monster 0: still asleep


@pytest.mark.parametrize('backend', BACKENDS)
def test_sleeping_foe_at_six_tiles_wakes_and_interrupts(backend):
    env = make(backend, build(hp=3, mons=[(46, 35, 8, 0, 0)]))  # semantic_tests.cu:24
    out = env.step(REST)
    c = env.compact()
    assert out[8] == 1 and c[3] < config()['hp']  # interrupted after one turn
    assert c[12 + 33] & 1 == 1  # awake
    assert not bit(env.legal, REST)  # semantic_tests.cu:25


@pytest.mark.parametrize('backend', BACKENDS)
def test_deadline_holds_inside_a_rest_macro(backend):
    env = make(backend, build(hp=3, ticks=2047))  # semantic_tests.cu:27
    out = env.step(REST)
    assert out[1] == 1 and out[7] == 1 and out[5] == 2048 and out[8] == 1
    assert env.compact()[7] == 0  # the episode reset after the terminal turn


@pytest.mark.parametrize('backend', BACKENDS)
def test_attack_is_one_primitive_on_the_weakest_visible_target(backend):
    hp = config()['hp']
    # semantic_tests.cu:29-32: goblin east at 8 HP, a weaker foe north at 3 HP
    case = build(hp=hp, mons=[(41, 35, 8, 2, 1), (40, 34, 3, 0, 1)])
    env = make(backend, case)
    assert bit(env.legal, ATTACK) and not bit(env.legal, REST)
    macro, manual = make(backend, case), make(backend, case)
    out = macro.step(ATTACK)
    step = manual.step(0)  # the primitive attack north
    assert out[8] == 1 and out[0] == step[0]
    assert np.array_equal(macro.row, manual.row)


@pytest.mark.parametrize('backend', BACKENDS)
@pytest.mark.parametrize('mons,direction', [
    ([(41, 35, 5, 0, 1), (40, 34, 5, 0, 1)], 0),  # N and E tied: N (compass order)
    ([(40, 36, 5, 0, 1), (41, 35, 5, 0, 1)], 1),  # E and S tied: E
    ([(39, 36, 4, 0, 1), (41, 34, 4, 0, 1)], 4),  # NE and SW tied: NE
    ([(39, 35, 6, 0, 1), (41, 36, 2, 0, 1)], 5),  # W at 6 HP, SE at 2 HP: SE
])
def test_attack_compass_ties(backend, mons, direction):
    case = build(hp=config()['hp'], mons=mons)
    macro, manual = make(backend, case), make(backend, case)
    macro.step(ATTACK)
    manual.step(direction)
    assert np.array_equal(macro.row, manual.row)


@pytest.mark.parametrize('backend', BACKENDS)
@pytest.mark.parametrize('action', [REST, ATTACK, DESCEND, 12, -1])
def test_invalid_action_costs_one_wait(backend, action):
    case = build(hp=config()['hp'])  # full HP (no rest), nobody adjacent, off the stairs
    env, wait = make(backend, case), make(backend, case)
    out = env.step(action)
    wait.step(WAIT)
    assert out[8] == 1 and out[9] == 1 and env.compact()[7] == 1  # semantic_tests.cu:40
    assert np.array_equal(env.compact(), wait.compact())


@pytest.mark.gpu
def test_gpu_and_oracle_agree_on_every_case():
    cases = [build(hp=3), build(hp=3, mons=[(47, 35, 8, 0, 0)]), build(hp=3, mons=[(46, 35, 8, 0, 0)]),
             build(hp=15, mons=[(41, 35, 8, 2, 1), (40, 34, 3, 0, 1)])]
    for case in cases:
        for a in (REST, WAIT, ATTACK, 0, 4):
            g, o = make('gpu', case), make('oracle', case)
            assert g.legal == o.legal
            np.testing.assert_array_equal(g.step(a), o.step(a))
            assert np.array_equal(g.compact(), o.compact()) and g.legal == o.legal
