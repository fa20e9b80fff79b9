"""DESCEND against the reference's stairs build (gpu-d1/branches/d1-stairs-v2).

The reference's own host-side self-test of that build (src/tests.cu,
stairs_semantic_test; built with the flags of that branch's scripts/assets.py by
`make -C oracle ref`) runs on the fixture corpus assembled here and must pass.
Its descend assertions (tests.cu:26-33, 44-46) are then mirrored on the spec
task's one stairs cell, with the spec actions DESCEND = 11 for its 18 and
WAIT = 8 for its 16, on the CPU oracle and on the GPU:
- off the stairs, descend is not legal and costs one wait (negative reward, not
  done);
- on the stairs, descend is legal, waiting there does not descend, and descend
  ends the episode as a descent (not a death or timeout) in one turn with the
  descent reward;
- a wait at the last tick ends the episode by the deadline, not as a descent;
- a descent leaves awake adjacent monsters alive and happens before their next
  action (the monster phase does not run on that turn: stairs learn.cu:732-736).
The stairs build's other rules (three stairs, stair cues, travel) have no
counterpart in the spec task.
"""
import ctypes as C
import subprocess
import sys

import numpy as np
import pytest

import oracle
from spec_cases import build
from test_semantic_reference import BACKENDS, LIMIT, Ours, fixture_floor, cheb, W

WAIT, DESCEND = 8, 11

_RUN = '''
import sys, ctypes as C
sys.path[:0] = [{oracle!r}, {pkg!r}]
import oracle
from d1.spec_env import DEFAULT
lib = C.CDLL({lib!r})
lib.stairs_semantic_test.argtypes = [C.c_void_p, C.c_void_p]
ref = oracle.SemanticReference(DEFAULT)  # the fixture as map 0 of a corpus, native LOS table
values = oracle.config_values(24)        # the build's REQUIRED regular monsters, no ogres
cfg = (C.c_int * len(values))(*values)
print(lib.stairs_semantic_test(C.byref(cfg), C.byref(ref.tables)))
'''


def test_reference_stairs_self_test_passes():
    """The reference's own stairs checks, in a child process: a failed host
    assert aborts the process that runs it."""
    lib = oracle.HERE / '_ref' / 'stairs_tests.so'
    if not lib.exists() or oracle.semantic_library() is None:
        pytest.skip('reference stairs / semantic builds not available (make -C oracle ref)')
    code = _RUN.format(oracle=str(oracle.HERE), pkg=str(oracle.REPO / 'dcss-auto_b200'), lib=str(lib))
    r = subprocess.run([sys.executable, '-c', code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().splitlines()[-1] == '0'


def cases():
    """(case, action, kind) triples on the fixture floor."""
    from d1.spec_env import DEFAULT
    floor = fixture_floor()
    cells = [int(p) for p in np.flatnonzero(floor)]
    rng = np.random.default_rng(8)
    out = []
    for k in range(40):
        p = cells[rng.integers(len(cells))]
        far = next(q for q in cells[::-1] if cheb(q, p) > 8)
        hp = int(rng.integers(1, DEFAULT['hp'] + 1))
        ticks = int(rng.integers(0, 1000))
        mk = lambda **kw: build(player=(p % W, p // W), hp=hp, floor=floor, **kw)
        out.append((mk(stairs=(far % W, far // W), ticks=ticks), DESCEND, 'off'))
        out.append((mk(stairs=(p % W, p // W), ticks=ticks), WAIT, 'stand'))
        out.append((mk(stairs=(p % W, p // W), ticks=ticks), DESCEND, 'descend'))
        out.append((mk(stairs=(far % W, far // W), ticks=LIMIT - 1), WAIT, 'deadline'))
        adj = [q for q in cells if cheb(q, p) == 1]
        if adj:
            q = adj[rng.integers(len(adj))]
            out.append((mk(stairs=(p % W, p // W), ticks=ticks, mons=[(q % W, q // W, 5, 0, 1)], energy=[79]),
                        DESCEND, 'guarded'))
    return out


@pytest.mark.parametrize('backend', BACKENDS)
def test_descend_mirrors_reference_stairs_checks(backend):
    from test_semantic_reference import config
    cfg = config()
    cs = cases()
    ours = Ours(backend, [c for c, _, _ in cs])
    legal = ours.legal
    out = ours.step([a for _, a, _ in cs])
    bonus = 0.001 * (cfg['descend_milli'] - 1)
    for i, (c, a, kind) in enumerate(cs):
        o, can = out[i], (legal[i] >> DESCEND) & 1
        if kind == 'off':  # tests.cu:24: an invalid descent waits
            assert not can and o[9] == 1 and o[1] == 0 and o[0] < 0 and o[8] == 1, i
        elif kind == 'stand':  # tests.cu:28: standing is not descending
            assert can and o[1] == 0 and o[2] == 0, i
        elif kind == 'descend':  # tests.cu:29-30
            assert can and o[1] == 1 and o[2] == 1 and o[6] == 0 and o[7] == 0 and o[8] == 1, i
            assert abs(o[0] - bonus) < 1e-6, i
        elif kind == 'deadline':  # tests.cu:32-33
            assert o[7] == 1 and o[2] == 0 and o[5] == LIMIT, i
        else:  # tests.cu:44-46: descent leaves enemies alive, before their next action
            assert can and o[2] == 1 and o[3] == 0 and o[4] == c['hp'], i
