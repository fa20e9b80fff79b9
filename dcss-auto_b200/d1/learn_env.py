"""Reference-compatible D:1 task on the B200 kernels.

Mirrors gpu-d1/scripts/learn_env.py: same constructor, the same `reset(seed)`,
`step(actions, active=None) -> (obs, out)` and `heuristic()` methods and the same
resident tensors (`state`, `obs`, `mask`, `out`, `actions`, `arrays`, `config`,
`tables`). Kernels run on the caller's current torch stream. There is no host
path: `device` must be a CUDA device (the reference's device='cpu' mode is served
by the test oracle in oracle/, not by this package).
"""
import ctypes as C
import pathlib

import numpy as np
import torch

from ._lib import check, library, resolve_device, launch_stream

DATA = pathlib.Path(__file__).resolve().parent / 'data'


class Tables(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ('floor', 'cells', 'index', 'distance')] + [('ncells', C.c_int)]


_MAP = None


def load_map():
    """(header, kinds, (floor, cells, index)) of the reference fixture map.

    Reachable cells are the floor cells with a finite native distance from the
    fixture's player cell, exactly as gpu-d1/scripts/learn_env.py:20-24 selects
    them; the all-pairs distance table is built on the device (see Env)."""
    global _MAP
    if _MAP is None:
        z = np.load(DATA / 'fixture_1057.npz')
        header, kinds, floor, native = z['header'], z['kinds'], z['floor'], z['native_dist']
        cells = np.flatnonzero((floor != 0) & (native < 65535)).astype(np.int16)
        index = np.full(5600, -1, np.int16)
        index[cells] = np.arange(len(cells))
        _MAP = header, kinds.reshape(-1), (floor, cells, index)
    return _MAP


def config_values(enemies):
    """learn_env.py:67-70: [enemies, *header[:7], repair=1, *gdr, *kinds]."""
    header, kinds, _ = load_map()
    ac = int(header[2]) // 100
    gdr = [int((65536 * (ac + j)) ** 0.25) for j in range(2)]
    return [enemies, *map(int, header[:7]), 1, *gdr, *map(int, kinds)]


_DEVICE_TABLES = {}


def device_tables(device):
    """Fixture tables resident on `device`; the distance table is built there by
    learn_distance_table (one warp per source cell)."""
    key = str(device)
    if key not in _DEVICE_TABLES:
        _, _, (floor, cells, index) = load_map()
        lib = library()
        f = torch.from_numpy(floor).to(device)
        c = torch.from_numpy(cells).to(device)
        i = torch.from_numpy(index).to(device)
        d = torch.empty((len(cells), 5600), dtype=torch.int16, device=device)  # u16 bits
        check(lib.learn_distance_table(f.data_ptr(), c.data_ptr(), len(cells), d.data_ptr(),
                                       launch_stream(device)), 'learn_distance_table')
        _DEVICE_TABLES[key] = [f, c, i, d]
    return _DEVICE_TABLES[key]


class Env:
    def __init__(self, batch=512, enemies=6, seed=0, device='cuda', limit=256):
        if not 1 <= enemies <= 8 or limit != 256:
            raise ValueError('Supported: 1..8 enemies, fixed 256-decision deadline')
        self.device = resolve_device(device)
        if self.device.type != 'cuda':
            raise ValueError('libd1 runs on CUDA devices only; use the oracle for CPU reference runs')
        self.batch, self.enemies, self.limit = batch, enemies, limit
        self.lib = library()
        values = config_values(enemies)
        self.config = (C.c_int * len(values))(*values)
        assert C.sizeof(self.config) == self.lib.learn_config_bytes()
        with torch.cuda.device(self.device):
            self.arrays = device_tables(self.device)
        self.tables = Tables(*(a.data_ptr() for a in self.arrays), self.arrays[1].shape[0])
        self.state = torch.zeros((batch, self.lib.learn_state_bytes()), dtype=torch.uint8, device=self.device)
        self.obs = torch.empty((batch, self.lib.learn_obs_size()), device=self.device)
        self.mask = torch.empty((batch, self.lib.learn_action_size()), device=self.device)
        self.out = torch.zeros((batch, self.lib.learn_out_size()), device=self.device)
        self.actions = torch.empty(batch, dtype=torch.int64, device=self.device)
        self.reset(seed)

    @property
    def stream(self):
        return launch_stream(self.device)

    def check(self, code):
        check(code, 'D:1 task call')

    def reset(self, seed):
        self.check(self.lib.learn_init(self.state.data_ptr(), self.batch, C.byref(self.config),
                                       C.byref(self.tables), seed, self.obs.data_ptr(), self.mask.data_ptr(),
                                       self.stream, 1))
        return self.obs

    def step(self, actions, active=None):
        assert actions.device == self.device and actions.dtype == torch.int64 and actions.is_contiguous()
        if active is not None:
            assert active.device == self.device and active.dtype == torch.bool and active.is_contiguous()
            assert active.shape == (self.batch,)
            self.check(self.lib.learn_step_active(self.state.data_ptr(), self.batch, C.byref(self.config),
                                                  C.byref(self.tables), actions.data_ptr(), self.limit,
                                                  self.obs.data_ptr(), self.mask.data_ptr(), self.out.data_ptr(),
                                                  active.data_ptr(), self.stream, 1))
            return self.obs, self.out
        self.check(self.lib.learn_step(self.state.data_ptr(), self.batch, C.byref(self.config), C.byref(self.tables),
                                       actions.data_ptr(), self.limit, self.obs.data_ptr(), self.mask.data_ptr(),
                                       self.out.data_ptr(), self.stream, 1))
        return self.obs, self.out

    def heuristic(self):
        self.check(self.lib.learn_heuristic(self.state.data_ptr(), self.batch, C.byref(self.config),
                                            C.byref(self.tables), self.actions.data_ptr(), self.stream, 1))
        return self.actions

    def compact(self):
        """Canonical (batch, 33) int64 view of the state (see include/d1.h)."""
        rows = torch.empty((self.batch, 33), dtype=torch.int64, device=self.device)
        self.check(self.lib.learn_compact_state(self.state.data_ptr(), self.batch, rows.data_ptr(), self.stream))
        return rows

    def semantic_test(self):
        return self.lib.learn_semantic_test(C.byref(self.config), C.byref(self.tables))
