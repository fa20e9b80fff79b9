#!/usr/bin/env python3
"""Generate golden trajectory digests from the reference's own host build.

Runs the reference's gpu-d1/src/learn.cu default build (compiled for the host by
`make -C oracle ref`, i.e. oracle/_ref/learn_v1.so, learn_step(..., gpu=0)) on
the fixture map and records, for every step, the SHA-256 of
obs | mask | out | compact-state (compact fields: see include/d1.h). The schedule
mirrors gpu-d1/scripts/test_learning.py:41-61 -- 37 worlds, seed 91, 300 steps,
heuristic actions on even steps and uniform random actions on odd steps -- for
1, 6 and 8 enemies, plus one 512-world x 1000-step all-random run (seed 42).
Random actions come from tests/golden/schedule.py, so only digests are stored.

  python tests/golden/make_golden.py     # writes tests/golden/v1_trajectories.npz
"""
import hashlib
import pathlib
import sys

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1] / 'oracle'))
sys.path.insert(0, str(HERE))
import oracle  # noqa: E402
from schedule import random_actions  # noqa: E402

RUNS = [  # (name, batch, enemies, seed, steps, heuristic_on_even)
    ('e1', 37, 1, 91, 300, True),
    ('e6', 37, 6, 91, 300, True),
    ('e8', 37, 8, 91, 300, True),
    ('r8', 512, 8, 42, 1000, False),
]


def digest(env):
    h = hashlib.sha256()
    for a in (env.obs, env.mask, env.out, env.compact()):
        h.update(np.ascontiguousarray(a).tobytes())
    return np.frombuffer(h.digest(), np.uint8)


def run(env, actions_fn, steps):
    """Drive `env`; returns (actions used, per-step digests, initial digest)."""
    init = digest(env)
    acts, digs = [], []
    for k in range(steps):
        a = actions_fn(env, k)
        env.step(a)
        acts.append(a.copy())
        digs.append(digest(env))
    return np.stack(acts), np.stack(digs), init


def main():
    oracle.build(ref=True)
    out = {}
    for name, batch, enemies, seed, steps, heur in RUNS:
        rand = random_actions(1000 + enemies + batch, steps, batch, 9)
        env = oracle.ReferenceV1(batch, enemies, seed=seed)
        fn = (lambda e, k: e.heuristic().copy() if (heur and k % 2 == 0) else rand[k])
        acts, digs, init = run(env, fn, steps)
        out[f'{name}_digests'] = digs
        out[f'{name}_init'] = init
        out[f'{name}_meta'] = np.array([batch, enemies, seed, steps, int(heur)], np.int64)
        print(name, 'terminations', int(env.out[:, 1].sum()))
    np.savez_compressed(HERE / 'v1_trajectories.npz', **out)


if __name__ == '__main__':
    main()
