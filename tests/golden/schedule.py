"""Deterministic action schedules shared by the golden generator and the tests.

random_actions(key, steps, batch, n) draws action k of env i as
splitmix64(key * 2^32 + k * batch + i) mod n: stable across numpy versions, so
golden files need not store the actions.
"""
import numpy as np

_M = np.uint64(0xFFFFFFFFFFFFFFFF)


def splitmix64(x):
    x = np.asarray(x, np.uint64)
    with np.errstate(over='ignore'):
        x = x + np.uint64(0x9E3779B97F4A7C15)
        x = (x ^ (x >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        x = (x ^ (x >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return x ^ (x >> np.uint64(31))


def random_actions(key, steps, batch, n):
    idx = (np.uint64(key) << np.uint64(32)) + np.arange(steps * batch, dtype=np.uint64)
    return (splitmix64(idx) % np.uint64(n)).astype(np.int64).reshape(steps, batch)
