"""The C-ABI library loads and exports every entry point include/d1.h declares.

No compute runs here (there is no GPU on the CPU runner); only size queries and
the host-path refusal, which returns before any CUDA call."""
import ctypes as C
import pathlib
import re

import pytest

REPO = pathlib.Path(__file__).resolve().parents[1]
HEADER = REPO / 'include' / 'd1.h'


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
    names = re.findall(r'^\s*(?:int|void|float)\s+(\w+)\s*\(', text, flags=re.M)
    assert names
    return names


@pytest.fixture(scope='module')
def lib():
    from d1 import _lib
    return _lib.library()


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_every_declared_symbol_has_python_signature():
    from d1 import _lib
    missing = [n for n in declared_functions() if n not in _lib.SIGNATURES]
    assert not missing, missing


def test_reference_sizes(lib):
    assert lib.learn_config_bytes() == 140
    assert lib.learn_obs_size() == 206
    assert lib.learn_action_size() == 9
    assert lib.learn_out_size() == 8
    assert lib.learn_state_bytes() % 16 == 0


def test_host_path_is_refused_not_emulated(lib):
    from d1 import _lib
    cfg = (C.c_int * 35)(*([1] + [0] * 34))
    assert lib.learn_init(None, 1, C.byref(cfg), None, 0, None, None, None, 0) == _lib.ERR_NO_HOST_PATH
    assert lib.learn_step(None, 1, C.byref(cfg), None, None, 256, None, None, None, None, 0) == _lib.ERR_NO_HOST_PATH
