"""Host-side pieces of the evaluation harness: the Wilson interval of
train_clear.py:63-66 and the oracle of the random baseline (uniform over the
legal actions)."""
import math
import sys
from pathlib import Path

import numpy as np

import oracle

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / 'dcss-auto_b200'))


def test_wilson_interval_known_values():
    from d1.evaluate import wilson
    lo, hi = wilson(5, 10)
    assert abs(lo - 0.2365895936) < 1e-9 and abs(hi - 0.7634104064) < 1e-9
    lo, hi = wilson(0, 37)
    assert lo == 0.0 and abs(hi - 1.96 ** 2 / (37 + 1.96 ** 2)) < 1e-12
    n, k, z = 1000, 123, 1.96
    p = k / n
    c = (p + z * z / (2 * n)) / (1 + z * z / n)
    h = z * math.sqrt(p * (1 - p) / n + z * z / (4 * n * n)) / (1 + z * z / n)
    assert wilson(k, n) == (c - h, c + h)


def test_uniform_legal_oracle_is_uniform_over_set_bits(oracle_lib):
    legal = np.full(60000, 0b1001_0010_0101, np.uint16)  # actions 0, 2, 5, 8, 11
    a = oracle.sample_uniform_legal(legal, 12, seed=4, step=2)
    assert set(np.unique(a)) == {0, 2, 5, 8, 11}
    counts = np.bincount(a, minlength=12)[[0, 2, 5, 8, 11]]
    assert np.all(np.abs(counts / 60000 - 0.2) < 0.01)
    assert (oracle.sample_uniform_legal(np.zeros(4, np.uint16), 12, 1, 1) == -1).all()
