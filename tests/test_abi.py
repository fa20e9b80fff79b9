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


def test_route_library_exports_the_reference_names():
    """libd1_route.so (the route-cue task) exports every learn_* that
    include/d1_route.h declares, with that build's sizes, and refuses the host
    path like libd1.so."""
    from d1 import _lib
    path = REPO / 'dcss-auto_b200' / 'd1' / 'libd1_route.so'
    route = C.CDLL(str(path))
    text = re.sub(r'/\*.*?\*/', '', (REPO / 'include' / 'd1_route.h').read_text(), flags=re.S)
    names = re.findall(r'^\s*int\s+(\w+)\s*\(', text, flags=re.M)
    assert set(names) == {'learn_state_bytes', 'learn_obs_size', 'learn_action_size', 'learn_out_size',
                          'learn_config_bytes', 'learn_init', 'learn_step', 'learn_step_active', 'learn_heuristic'}
    for name in names:
        assert hasattr(route, name), name
    assert (route.learn_obs_size(), route.learn_action_size(), route.learn_out_size(),
            route.learn_config_bytes(), route.learn_state_bytes()) == (421, 9, 8, 140, 13312)
    p, i = C.c_void_p, C.c_int
    route.learn_init.argtypes = [p, i, p, p, C.c_uint64, p, p, p, i]
    cfg = (C.c_int * 35)(*([40] + [0] * 34))
    assert route.learn_init(None, 1, C.byref(cfg), None, 0, None, None, None, 0) == _lib.ERR_NO_HOST_PATH


def test_route_sizes(lib):
    assert (lib.d1_route_obs_size(), lib.d1_route_action_size(), lib.d1_route_out_size(),
            lib.d1_route_config_bytes(), lib.d1_route_state_bytes(), lib.d1_route_compact_size()) == (
        421, 9, 8, 140, 13312, 171)
