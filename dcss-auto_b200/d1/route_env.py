"""The route-cue task on the B200 kernels: the reference's selected fast build of
its headline PPO benchmark (gpu-d1/src/learn.cu with LEARN_ENEMIES=40,
MULTI_MAP, SLEEP_ON, EXPLORE_REWARD, MARK_WALLS, FRONTIER_RING_MEMORY_WALLS_OBS,
KNOWN_FRONTIER, FRONTIER_ROUTE_CUE_OBS, FAST_FRONTIER; gpu-d1/scripts/
run_ring_ablations.py:141-157).

RouteEnv mirrors gpu-d1/scripts/learn_env_ring_multi.py:45-117: the same
constructor arguments (batch, enemies 1..40, seed, device, limit 1024, corpus,
map_filter, map_limit), the same reset(seed), step(actions, active=None) ->
(obs, out) and heuristic() methods, and the same resident tensors (state, obs,
mask, out, actions, arrays, config, tables). Kernels run on the caller's
current torch stream; there is no host path.

The corpus is a directory of map-SEED.bin files in the reference's format
(gpu-d1/scripts/learn_env_v2.py:25-64; see d1.maps), or a list of maps given
as CorpusMap objects or (floor, cells, index, distance) tuples.
generated_corpus() builds one from the fixture map plus maps of the BASELINE
task's generator, the reference's 388-map native corpus being unavailable here.
"""
import ctypes as C

import numpy as np
import torch

from ._lib import check, library, launch_stream, resolve_device
from .learn_env import config_values, load_map

OBS, ACTIONS, OUT, ENEMIES, LIMIT = 421, 9, 8, 40, 1024


class Tables(C.Structure):
    """learn.cu:130-139 with MULTI_MAP (learn_env_ring_multi.py:11-17)."""
    _fields_ = [(k, C.c_void_p) for k in ('floor', 'cells', 'index', 'distance')] + [
        ('ncells', C.c_int), ('map_ncells', C.c_void_p), ('distance_offsets', C.c_void_p), ('n_maps', C.c_int),
        ('map_filter', C.c_int)]


def _as_tuple(m):
    if isinstance(m, tuple):
        return m
    return (m.floor, m.cells, m.index, m.distance)


def table_arrays(maps):
    """Concatenated host arrays in the layout of learn_env_ring_multi.py:60-70."""
    maps = [_as_tuple(m) for m in maps]
    floors = np.concatenate([np.asarray(m[0], np.uint8).reshape(-1) for m in maps])
    cells = np.full((len(maps), 5600), -1, np.int16)
    for k, m in enumerate(maps):
        cells[k, :len(m[1])] = m[1]
    index = np.concatenate([np.asarray(m[2], np.int16).reshape(-1) for m in maps])
    distance = np.concatenate([np.asarray(m[3], np.uint16).reshape(-1) for m in maps])
    ncells = np.array([len(m[1]) for m in maps], np.int32)
    offsets = np.concatenate(([0], np.cumsum(ncells[:-1]))).astype(np.int32)
    return [floors, cells.reshape(-1), index, distance, ncells, offsets]


def generated_corpus(n_maps, seed=0, device='cuda'):
    """Map 0: the fixture map (its reachable cells, learn_env.py:20-24); maps
    1..n_maps-1: the floors the BASELINE task's generator draws for env ids
    0..n_maps-2 under `seed`, compiled on the GPU (all-pairs BFS)."""
    from .maps import compile_map
    from .spec_env import SpecEnv
    dev = resolve_device(device)
    _, _, (floor, cells, index) = load_map()
    maps = []
    with torch.cuda.device(dev):
        fm = compile_map(floor, device=dev)
        keep = np.isin(fm.cells, cells)
        rows = np.flatnonzero(keep)
        maps.append((floor, cells, index, fm.distance[rows]))
        if n_maps > 1:
            gen = SpecEnv(n_maps - 1, seed=seed, device=dev, observe=False)
            bits, _ = gen.planes()
            bits = bits.cpu().numpy().view(np.uint32).reshape(n_maps - 1, 70, 3)
            x = np.arange(80)
            for k in range(n_maps - 1):
                fl = ((bits[k][:, x // 32] >> (x % 32).astype(np.uint32)) & 1).astype(np.uint8).reshape(-1)
                m = compile_map(fl, device=dev)
                maps.append((m.floor, m.cells, m.index, m.distance))
    return maps


class RouteEnv:
    def __init__(self, batch=512, enemies=ENEMIES, seed=0, device='cuda', limit=LIMIT, corpus=None, map_filter=-1,
                 map_limit=None, maps=None):
        if not 1 <= enemies <= ENEMIES or limit != LIMIT:
            raise ValueError('This task uses 1..40 enemies and a 1024-decision deadline')
        self.device = resolve_device(device)
        if self.device.type != 'cuda':
            raise ValueError('libd1 runs on CUDA devices only; use the oracle for CPU reference runs')
        self.batch, self.enemies, self.limit = batch, enemies, limit
        self.lib = library()
        if maps is None:
            if corpus is None:
                raise ValueError('give a corpus directory or a list of maps (see generated_corpus)')
            from .maps import read_corpus
            maps = read_corpus(corpus, map_limit=map_limit)
        host = table_arrays(maps)
        self.n_maps = len(host[4])
        if not -2 <= map_filter < self.n_maps:
            raise ValueError(f'map_filter must be -2, -1 or a map index below {self.n_maps}')
        self.arrays = [torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).to(self.device)
                       for a in host]
        self.tables = Tables(self.arrays[0].data_ptr(), self.arrays[1].data_ptr(), self.arrays[2].data_ptr(),
                             self.arrays[3].data_ptr(), int(host[4][0]), self.arrays[4].data_ptr(),
                             self.arrays[5].data_ptr(), self.n_maps, map_filter)
        values = config_values(enemies)
        self.config = (C.c_int * len(values))(*values)
        assert C.sizeof(self.config) == self.lib.d1_route_config_bytes()
        self.state = torch.zeros((batch, self.lib.d1_route_state_bytes()), dtype=torch.uint8, device=self.device)
        self.obs = torch.empty((batch, OBS), device=self.device)
        self.mask = torch.empty((batch, ACTIONS), device=self.device)
        self.out = torch.zeros((batch, OUT), device=self.device)
        self.legal = torch.zeros(batch, dtype=torch.int16, device=self.device)
        self.actions = torch.empty(batch, dtype=torch.int64, device=self.device)
        self.reset(seed)

    @property
    def stream(self):
        return launch_stream(self.device)

    def check(self, code):
        check(code, 'route-cue task call')

    def reset(self, seed):
        self.check(self.lib.d1_route_init(self.state.data_ptr(), self.batch, C.byref(self.config),
                                          C.byref(self.tables), seed, self.obs.data_ptr(), self.mask.data_ptr(),
                                          self.legal.data_ptr(), self.stream))
        return self.obs

    def step(self, actions, active=None):
        assert actions.device == self.device and actions.dtype == torch.int64 and actions.is_contiguous()
        act = None
        if active is not None:
            assert active.device == self.device and active.dtype == torch.bool and active.is_contiguous()
            assert active.shape == (self.batch,)
            act = active.data_ptr()
        self.check(self.lib.d1_route_step(self.state.data_ptr(), self.batch, C.byref(self.config),
                                          C.byref(self.tables), actions.data_ptr(), self.limit, self.obs.data_ptr(),
                                          self.mask.data_ptr(), self.out.data_ptr(), act, self.legal.data_ptr(),
                                          self.stream))
        return self.obs, self.out

    def heuristic(self):
        self.check(self.lib.d1_route_heuristic(self.state.data_ptr(), self.batch, C.byref(self.config),
                                               C.byref(self.tables), self.actions.data_ptr(), self.stream))
        return self.actions

    def observe(self):
        """Re-observe the rows as they are (e.g. rows edited by hand)."""
        self.check(self.lib.d1_route_observe(self.state.data_ptr(), self.batch, C.byref(self.config),
                                             C.byref(self.tables), self.obs.data_ptr(), self.mask.data_ptr(),
                                             self.legal.data_ptr(), self.stream))
        return self.obs

    def compact(self):
        """(batch, 171) int64 view: rng.state, rng.inc, episode, hp, regen, blocks,
        player, ticks, killed, map_id, frontier_count, pos/energy/hp/awake x 40."""
        rows = torch.empty((self.batch, self.lib.d1_route_compact_size()), dtype=torch.int64, device=self.device)
        self.check(self.lib.d1_route_compact(self.state.data_ptr(), self.batch, rows.data_ptr(), self.stream))
        return rows

    def memory(self):
        """(viewed u32 bit planes [batch, 210] as int32, frontier list i16 [batch, 5600], -1 past the count)."""
        v = torch.empty((self.batch, 210), dtype=torch.int32, device=self.device)
        f = torch.empty((self.batch, 5600), dtype=torch.int16, device=self.device)
        self.check(self.lib.d1_route_memory(self.state.data_ptr(), self.batch, v.data_ptr(), f.data_ptr(),
                                            self.stream))
        return v, f
