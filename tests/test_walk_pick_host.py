"""The pursuit step's tie walk, restated both ways on the host: the reference's
serial rotated walk with reservoir ties (gpu-d1/src/sim.h:213-222) and the mask
form the env kernels use (walk_pick in dcss-auto_b200/csrc/d1_common.cuh: the
candidates one step closer as a bit mask in walk order, then the same draws
r(2), r(3), ...). Over every rotation and random neighbourhoods whose
distances obey the BFS bound (a free floor neighbour of a cell at distance D is
at D - 1, D or D + 1, or unreached with it), both keep the same cell and take
the same draws in the same order."""
import numpy as np

UNREACHED = 65535


def walk_serial(ok, dist, D, rotation, draw):
    best, bd, ties = -1, D, 0
    for z in range(8):
        d = (z + rotation) % 4 if z < 4 else 4 + (z + rotation) % 4
        if not ok[d]:
            continue
        if dist[d] < bd:
            bd, best, ties = dist[d], d, 1
        elif dist[d] == bd and best >= 0:
            ties += 1
            if draw(ties) == 0:
                best = d
    return best


def walk_mask(ok, dist, D, rotation, draw):
    cand = sum(1 << d for d in range(8) if ok[d] and dist[d] < D)
    if not cand:
        return -1
    lo, hi = cand & 0xF, (cand >> 4) & 0xF
    rot = lambda v: ((v >> rotation) | (v << (4 - rotation))) & 0xF
    walk = rot(lo) | (rot(hi) << 4)
    bits = [z for z in range(8) if (walk >> z) & 1]
    pick = bits[0]
    for t, z in enumerate(bits[1:], start=2):
        if draw(t) == 0:
            pick = z
    return (pick + rotation) % 4 if pick < 4 else 4 + (pick - 4 + rotation) % 4


def test_mask_form_equals_the_serial_walk():
    rng = np.random.default_rng(0)
    for case in range(20000):
        D = int(rng.integers(1, 40))
        reached = rng.random() < 0.9
        dist = [int(D + rng.integers(-1, 2)) if reached and rng.random() < 0.9 else UNREACHED for _ in range(8)]
        ok = [bool(rng.random() < 0.7) for _ in range(8)]
        rotation = int(rng.integers(4))
        stream = rng.integers(0, 1 << 30, 16)
        logs = []
        for walk in (walk_serial, walk_mask):
            log = []

            def draw(bound, log=log):
                v = int(stream[len(log)] % bound)
                log.append(bound)
                return v
            logs.append((walk(ok, dist, D, rotation, draw), log))
        assert logs[0] == logs[1], (case, ok, dist, D, rotation)
