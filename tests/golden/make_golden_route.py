#!/usr/bin/env python3
"""Generate golden trajectory digests of the route-cue task from the reference's
own host build.

Runs gpu-d1/src/learn.cu built with the route-cue fast flags (oracle/Makefile
ROUTEFLAGS -> oracle/_ref/learn_route.so, learn_step(..., gpu=0)) over a small
corpus in the reference's multi-map layout: the fixture map plus maps drawn by
the BASELINE task's generator (oracle.route_corpus; the reference's native
corpus is not available). For every step it records the SHA-256 of
obs | mask | out | compact state (171 x i64) | viewed bit plane (u32 x 210) |
frontier list (i16 x 5600, -1 past the count). Actions: the reference
heuristic on even steps and tests/golden/schedule.py's uniform actions on odd
steps, or uniform actions only. Only digests are stored.

  python tests/golden/make_golden_route.py   # writes tests/golden/route_trajectories.npz
"""
import hashlib
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / 'oracle'))
sys.path.insert(0, str(HERE.parents[1] / 'dcss-auto_b200'))
sys.path.insert(0, str(HERE))
import oracle  # noqa: E402
from schedule import random_actions  # noqa: E402

CORPUS = dict(n_maps=6, seed=11)
RUNS = [  # (name, batch, enemies, seed, steps, heuristic_on_even, map_filter)
    ('h40', 48, 40, 17, 1200, True, -1),
    ('r1', 48, 1, 5, 1200, False, -1),
    ('h8', 32, 8, 3, 600, True, -2),
]


def corpus():
    from d1.spec_env import DEFAULT
    return oracle.route_corpus(CORPUS['n_maps'], DEFAULT, seed=CORPUS['seed'])


def corpus_digest(maps):
    h = hashlib.sha256()
    for a in oracle.route_arrays(maps).values():
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), np.uint8)


def digest(obs, mask, out, compact, viewed, frontier):
    h = hashlib.sha256()
    for a, dt in ((obs, np.float32), (mask, np.float32), (out, np.float32), (compact, np.int64),
                  (viewed, np.uint32), (frontier, np.int16)):
        h.update(np.ascontiguousarray(a, dt).tobytes())
    return np.frombuffer(h.digest(), np.uint8)


def ref_digest(env):
    return digest(env.obs, env.mask, env.out, env.compact(), env.viewed_bits(), env.frontier())


def main():
    oracle.build(ref=True)
    maps = corpus()
    out = {'corpus_digest': corpus_digest(maps)}
    for name, batch, enemies, seed, steps, heur, mf in RUNS:
        rand = random_actions(2000 + enemies + batch, steps, batch, 9)
        env = oracle.ReferenceRoute(batch, maps, enemies=enemies, seed=seed, map_filter=mf)
        init = ref_digest(env)
        digs, ends = [], 0
        for k in range(steps):
            a = env.heuristic().copy() if (heur and k % 2 == 0) else rand[k]
            env.step(a)
            ends += int(env.out[:, 1].sum())
            digs.append(ref_digest(env))
        out[f'{name}_digests'] = np.stack(digs)
        out[f'{name}_init'] = init
        out[f'{name}_meta'] = np.array([batch, enemies, seed, steps, int(heur), mf], np.int64)
        print(name, 'episode ends', ends, 'last frontier count', env.compact()[:, 10].max())
    np.savez_compressed(HERE / 'route_trajectories.npz', **out)


if __name__ == '__main__':
    main()
