"""Host-side rule of the rollout's stream split: the env ranges that
d1.rollout.Rollout and DecisionGraph step on separate streams cover the batch
exactly once, in order, and small batches stay on one stream."""
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parents[1] / 'dcss-auto_b200'))


@pytest.mark.parametrize('batch,parts,count', [(512, 2, 1), (8191, 2, 1), (8192, 2, 2), (65536, 2, 2),
                                               (65536, 4, 4), (65536, 1, 1), (12288, 4, 3), (131072, 0, 1)])
def test_env_ranges_cover_the_batch(batch, parts, count):
    from d1.rollout import env_ranges
    r = env_ranges(batch, parts)
    assert len(r) == count
    assert r[0][0] == 0 and r[-1][1] == batch
    assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    assert all(hi - lo >= (4096 if count > 1 else 0) for lo, hi in r)
