"""TEST INFRASTRUCTURE ONLY -- Python handles on the CPU oracle and on the reference build.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference leg
import this module, and only as the checker. It wraps:

* liboracle.so      -- the plain-C restatement in oracle/d1_oracle.c;
* _ref/learn_v1.so  -- the reference's own gpu-d1/src/learn.cu default build,
                       compiled for the host from the reference sources by
                       `make -C oracle ref` (present only where the reference
                       tree was available when it was built).

The fixture tables are assembled the way gpu-d1/scripts/learn_env.py:15-40 and
:66-75 assemble them.
"""
import ctypes as C
import os
import pathlib
import subprocess

import numpy as np

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent
DATA = REPO / 'dcss-auto_b200' / 'd1' / 'data'


def reference_dir():
    """The reference's gpu-d1 folder: $DCSS_REFERENCE/gpu-d1, where DCSS_REFERENCE
    names the reference checkout (default: a folder `reference` beside this
    repository). Only the build recipes and host-side tests read it; it may be
    absent, and nothing on a GPU box needs it."""
    root = os.environ.get('DCSS_REFERENCE')
    return (pathlib.Path(root) if root else REPO.parent / 'reference') / 'gpu-d1'

V1_OBS, V1_ACTIONS, V1_OUT, V1_COMPACT = 206, 9, 8, 33


class Tables(C.Structure):
    _fields_ = [(k, C.c_void_p) for k in ('floor', 'cells', 'index', 'distance')] + [('ncells', C.c_int)]


def build(ref=False):
    """Compile the oracle (and, when asked and possible, the reference build)."""
    subprocess.run(['make', '-s', '-C', str(HERE), 'liboracle.so'], check=True)
    if ref:
        subprocess.run(['make', '-s', '-C', str(HERE), 'ref'], check=True)


_LIB = None


def library():
    global _LIB
    if _LIB is None:
        path = HERE / 'liboracle.so'
        if not path.exists():
            build()
        lib = C.CDLL(str(path))
        p, i = C.c_void_p, C.c_int
        lib.oracle_v1_init.argtypes = [p, i, p, p, C.c_uint64, p, p]
        lib.oracle_v1_step.argtypes = [p, i, p, p, p, i, p, p, p, p]
        lib.oracle_v1_heuristic.argtypes = [p, i, p, p, p]
        lib.oracle_v1_compact.argtypes = [p, i, p]
        lib.oracle_v1_compact_from_reference.argtypes = [p, i, i, p]
        lib.oracle_v1_semantic_test.argtypes = [p, p]
        lib.oracle_distance_table.argtypes = [p, p, i, p]
        _LIB = lib
    return _LIB


def reference_library():
    """The reference's own host build, or None when it was not built here."""
    path = HERE / '_ref' / 'learn_v1.so'
    if not path.exists():
        return None
    lib = C.CDLL(str(path))
    p, i = C.c_void_p, C.c_int
    lib.learn_init.argtypes = [p, i, p, p, C.c_uint64, p, p, p, i]
    lib.learn_step.argtypes = [p, i, p, p, p, i, p, p, p, p, i]
    lib.learn_step_active.argtypes = [p, i, p, p, p, i, p, p, p, p, p, i]
    lib.learn_heuristic.argtypes = [p, i, p, p, p, p, i]
    lib.learn_semantic_test.argtypes = [p, p]
    return lib


_FIXTURE = None


def fixture():
    """(header, kinds, floor, cells, index, distance) for the reference map."""
    global _FIXTURE
    if _FIXTURE is None:
        z = np.load(DATA / 'fixture_1057.npz')
        header, kinds, floor, native = z['header'], z['kinds'], z['floor'], z['native_dist']
        cells = np.flatnonzero((floor != 0) & (native < 65535)).astype(np.int16)
        index = np.full(5600, -1, np.int16)
        index[cells] = np.arange(len(cells))
        distance = np.empty((len(cells), 5600), np.uint16)
        code = library().oracle_distance_table(floor.ctypes.data, cells.ctypes.data, len(cells),
                                               distance.ctypes.data)
        assert code == 0
        _FIXTURE = (header, kinds, floor, cells, index, distance)
    return _FIXTURE


def config_values(enemies):
    """learn_env.py:67-70: [enemies, *header[:7], repair=1, *gdr, *kinds]."""
    header, kinds = fixture()[:2]
    ac = int(header[2]) // 100
    gdr = [int((65536 * (ac + j)) ** 0.25) for j in range(2)]
    return [enemies, *map(int, header[:7]), 1, *gdr, *map(int, kinds.reshape(-1))]


class _Host:
    """Host-memory env driven through a learn_*-shaped C entry table."""

    def __init__(self, batch, enemies, seed, limit):
        if not 1 <= enemies <= 8 or limit != 256:
            raise ValueError('Supported: 1..8 enemies, fixed 256-decision deadline')
        _, _, floor, cells, index, distance = fixture()
        self.batch, self.enemies, self.limit = batch, enemies, limit
        values = config_values(enemies)
        self.config = (C.c_int * len(values))(*values)
        self.arrays = [floor, cells, index, distance]
        self.tables = Tables(floor.ctypes.data, cells.ctypes.data, index.ctypes.data, distance.ctypes.data,
                             len(cells))
        self.obs = np.zeros((batch, V1_OBS), np.float32)
        self.mask = np.zeros((batch, V1_ACTIONS), np.float32)
        self.out = np.zeros((batch, V1_OUT), np.float32)
        self.actions = np.zeros(batch, np.int64)


class OracleV1(_Host):
    """The plain-C restatement of the reference default build."""

    def __init__(self, batch=512, enemies=6, seed=0, limit=256):
        super().__init__(batch, enemies, seed, limit)
        self.lib = library()
        self.state = np.zeros((batch, self.lib.oracle_v1_state_bytes()), np.uint8)
        self.reset(seed)

    def reset(self, seed):
        code = self.lib.oracle_v1_init(self.state.ctypes.data, self.batch, C.byref(self.config),
                                       C.byref(self.tables), seed, self.obs.ctypes.data, self.mask.ctypes.data)
        assert code == 0
        return self.obs

    def step(self, actions, active=None):
        actions = np.ascontiguousarray(actions, np.int64)
        act = None if active is None else np.ascontiguousarray(active, np.uint8)
        self.lib.oracle_v1_step(self.state.ctypes.data, self.batch, C.byref(self.config), C.byref(self.tables),
                                actions.ctypes.data, self.limit, self.obs.ctypes.data, self.mask.ctypes.data,
                                self.out.ctypes.data, None if act is None else act.ctypes.data)
        return self.obs, self.out

    def heuristic(self):
        self.lib.oracle_v1_heuristic(self.state.ctypes.data, self.batch, C.byref(self.config),
                                     C.byref(self.tables), self.actions.ctypes.data)
        return self.actions

    def compact(self):
        rows = np.zeros((self.batch, V1_COMPACT), np.int64)
        self.lib.oracle_v1_compact(self.state.ctypes.data, self.batch, rows.ctypes.data)
        return rows

    def semantic_test(self):
        return self.lib.oracle_v1_semantic_test(C.byref(self.config), C.byref(self.tables))


class ReferenceV1(_Host):
    """The reference's own learn.cu host path (gpu=0), when built."""

    def __init__(self, batch=512, enemies=6, seed=0, limit=256):
        super().__init__(batch, enemies, seed, limit)
        self.lib = reference_library()
        if self.lib is None:
            raise FileNotFoundError('oracle/_ref/learn_v1.so was not built')
        self.state = np.zeros((batch, self.lib.learn_state_bytes()), np.uint8)
        self.reset(seed)

    def reset(self, seed):
        code = self.lib.learn_init(self.state.ctypes.data, self.batch, C.byref(self.config), C.byref(self.tables),
                                   seed, self.obs.ctypes.data, self.mask.ctypes.data, None, 0)
        assert code == 0
        return self.obs

    def step(self, actions, active=None, lo=0, hi=None):
        """Steps envs [lo, hi) (all by default; slices let a thread pool split the batch)."""
        actions = np.ascontiguousarray(actions, np.int64)
        if active is None:
            hi = self.batch if hi is None else hi
            self.lib.learn_step(self.state[lo:hi].ctypes.data, hi - lo, C.byref(self.config), C.byref(self.tables),
                                actions[lo:hi].ctypes.data, self.limit, self.obs[lo:hi].ctypes.data,
                                self.mask[lo:hi].ctypes.data, self.out[lo:hi].ctypes.data, None, 0)
        else:
            act = np.ascontiguousarray(active, np.bool_)
            self.lib.learn_step_active(self.state.ctypes.data, self.batch, C.byref(self.config),
                                       C.byref(self.tables), actions.ctypes.data, self.limit, self.obs.ctypes.data,
                                       self.mask.ctypes.data, self.out.ctypes.data, act.ctypes.data, None, 0)
        return self.obs, self.out

    def heuristic(self):
        self.lib.learn_heuristic(self.state.ctypes.data, self.batch, C.byref(self.config), C.byref(self.tables),
                                 self.actions.ctypes.data, None, 0)
        return self.actions

    def compact(self):
        rows = np.zeros((self.batch, V1_COMPACT), np.int64)
        code = library().oracle_v1_compact_from_reference(self.state.ctypes.data, self.batch,
                                                          self.state.shape[1], rows.ctypes.data)
        assert code == 0
        return rows

    def semantic_test(self):
        return self.lib.learn_semantic_test(C.byref(self.config), C.byref(self.tables))


# ---------------------------------------------------------------------------
# spec task: generated maps, Philox, 12 semantic actions
# ---------------------------------------------------------------------------
SPEC_OBS, SPEC_ACTIONS, SPEC_OUT, SPEC_COMPACT, SPEC_MAXM = 1832, 12, 10, 56, 11


class Kind(C.Structure):
    _fields_ = [(k, C.c_int) for k in ('speed', 'damage', 'tohit', 'bypass')]


class SpecConfig(C.Structure):
    _fields_ = ([(k, C.c_int) for k in ('hp', 'ac100', 'ev100', 'sh100', 'shield_limit', 'regen')]
                + [('gdr', C.c_int * 2)]
                + [(k, C.c_int) for k in ('min_monsters', 'max_monsters', 'min_mhp', 'max_mhp', 'ogre', 'ogre_hp',
                                          'ogre_min_damage', 'limit', 'explore_milli', 'kill_milli',
                                          'descend_milli', 'death_milli')]
                + [('kinds', Kind * 5)])


def spec_config(values):
    """Build the C struct from a dict with the SpecConfig field names."""
    c = SpecConfig()
    for k, v in values.items():
        if k == 'gdr':
            c.gdr[0], c.gdr[1] = v
        elif k == 'kinds':
            for i, kind in enumerate(v):
                c.kinds[i] = Kind(*kind)
        else:
            setattr(c, k, int(v))
    return c


_RAYS_SET = False


def rays():
    z = np.load(DATA / 'los_rays.npz')
    return z['end_x'].astype(np.int32), z['end_y'].astype(np.int32), z['blockers'].astype(np.uint64)


def spec_library():
    global _RAYS_SET
    lib = library()
    if not _RAYS_SET:
        p, i = C.c_void_p, C.c_int
        lib.oracle_set_rays.argtypes = [p, p, p, i]
        lib.oracle_los_mask.argtypes = [p, i, p]
        lib.oracle_philox.argtypes = [p, p, p]
        lib.oracle_philox.restype = None
        lib.oracle_spec_init.argtypes = [p, i, p, C.c_uint64, i, p, p]
        lib.oracle_spec_step.argtypes = [p, i, p, p, p, p, p]
        lib.oracle_spec_compact.argtypes = [p, i, p]
        lib.oracle_spec_planes.argtypes = [p, i, p, p]
        lib.oracle_spec_crop.argtypes = [p, i, i, p]
        lib.oracle_sample_ar.argtypes = [p, p, p, i, C.c_uint64, C.c_uint64, i, p, p, p, p]
        lib.oracle_sample_uniform_legal.argtypes = [p, i, i, C.c_uint64, C.c_uint64, i, p]
        ex, ey, blk = rays()
        lib._rays_keep = (ex, ey, blk)
        assert lib.oracle_set_rays(ex.ctypes.data, ey.ctypes.data, blk.ctypes.data, len(ex)) == 0
        _RAYS_SET = True
    return lib


def los_mask(floor_u8, origin):
    out = np.zeros(10, np.uint32)
    assert spec_library().oracle_los_mask(np.ascontiguousarray(floor_u8, np.uint8).ctypes.data, origin,
                                          out.ctypes.data) == 0
    return out


def philox(ctr, key):
    ctr = np.ascontiguousarray(ctr, np.uint32)
    key = np.ascontiguousarray(key, np.uint32)
    out = np.zeros(4, np.uint32)
    spec_library().oracle_philox(ctr.ctypes.data, key.ctypes.data, out.ctypes.data)
    return out


class OracleSpec:
    """CPU restatement of the spec task; float obs [n, 1832], u16 legal bits [n]."""

    def __init__(self, batch, config, seed=0, first_env=0):
        self.lib = spec_library()
        self.batch = batch
        self.config = spec_config(config)
        self.state = np.zeros((batch, self.lib.oracle_spec_state_bytes()), np.uint8)
        self.obs = np.zeros((batch, SPEC_OBS), np.float32)
        self.legal = np.zeros(batch, np.uint16)
        self.out = np.zeros((batch, SPEC_OUT), np.float32)
        assert self.lib.oracle_spec_init(self.state.ctypes.data, batch, C.byref(self.config), seed, first_env,
                                         self.obs.ctypes.data, self.legal.ctypes.data) == 0

    def step(self, actions):
        actions = np.ascontiguousarray(actions, np.int64)
        self.lib.oracle_spec_step(self.state.ctypes.data, self.batch, C.byref(self.config), actions.ctypes.data,
                                  self.obs.ctypes.data, self.legal.ctypes.data, self.out.ctypes.data)
        return self.obs, self.out

    def compact(self):
        rows = np.zeros((self.batch, SPEC_COMPACT), np.int64)
        self.lib.oracle_spec_compact(self.state.ctypes.data, self.batch, rows.ctypes.data)
        return rows

    def crop(self, g=0):
        """u16 [n, 63, 64] egocentric crops under D4 element g (conv policy input)."""
        out = np.zeros((self.batch, 63, 64), np.uint16)
        assert self.lib.oracle_spec_crop(self.state.ctypes.data, self.batch, g, out.ctypes.data) == 0
        return out

    def planes(self):
        f = np.zeros((self.batch, 210), np.uint32)
        v = np.zeros((self.batch, 210), np.uint32)
        self.lib.oracle_spec_planes(self.state.ctypes.data, self.batch, f.ctypes.data, v.ctypes.data)
        return f, v


def exp_nonpos(x):
    lib = library()
    lib.oracle_exp_nonpos.argtypes = [C.c_void_p, C.c_int, C.c_void_p]
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib.oracle_exp_nonpos(x.ctypes.data, x.size, y.ctypes.data)
    return y


def sample_actions(logits, legal, seed, step, first_env=0):
    """Oracle of the policy sampler: (actions int64, logp float32)."""
    lib = spec_library()
    lib.oracle_sample_actions.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_uint64, C.c_uint64, C.c_int,
                                          C.c_void_p, C.c_void_p]
    logits = np.ascontiguousarray(logits, np.float32)
    legal = np.ascontiguousarray(legal, np.uint16)
    n = logits.shape[0]
    a = np.empty(n, np.int64)
    lp = np.empty(n, np.float32)
    lib.oracle_sample_actions(logits.ctypes.data, legal.ctypes.data, n, seed, step, first_env, a.ctypes.data,
                              lp.ctypes.data)
    return a, lp


AR_ENV_ACTION = np.array([0, 1, 2, 3, 4, 5, 6, 7, -1, 0, 1, 2, 3, 4, 5, 6, 7, 10, 8, 9, 11, -1, -1, -1, -1, -1, -1, -1],
                         np.int64)


def sample_ar(verb_logits, target_logits, legal, seed, step, first_env=0):
    """Oracle of the autoregressive verb x target sampler:
    (joint int64, env action int64, logp float32, entropy float32)."""
    lib = spec_library()
    vl = np.ascontiguousarray(verb_logits, np.float32)
    tl = np.ascontiguousarray(target_logits, np.float32)
    legal = np.ascontiguousarray(legal, np.uint16)
    n = vl.shape[0]
    assert vl.shape == (n, 12) and tl.shape == (n, 2, 9)
    j, a = np.empty(n, np.int64), np.empty(n, np.int64)
    lp, ent = np.empty(n, np.float32), np.empty(n, np.float32)
    lib.oracle_sample_ar(vl.ctypes.data, tl.ctypes.data, legal.ctypes.data, n, seed, step, first_env, j.ctypes.data,
                         a.ctypes.data, lp.ctypes.data, ent.ctypes.data)
    return j, a, lp, ent


def sample_uniform_legal(legal, nact, seed, step, first_env=0):
    """Oracle of the random baseline: int64 actions (-1 where nothing is legal)."""
    lib = spec_library()
    legal = np.ascontiguousarray(legal, np.uint16)
    a = np.empty(legal.shape[0], np.int64)
    lib.oracle_sample_uniform_legal(legal.ctypes.data, nact, legal.shape[0], seed, step, first_env, a.ctypes.data)
    return a


# ---------------------------------------------------------------------------
# route-cue task: the reference's selected fast build of its headline PPO task
# (gpu-d1/src/learn.cu with the flags of oracle/Makefile ROUTEFLAGS), driven
# through its own host path (learn_step(..., gpu=0))
# ---------------------------------------------------------------------------
ROUTE_OBS, ROUTE_ACTIONS, ROUTE_OUT, ROUTE_ENEMIES, ROUTE_LIMIT = 421, 9, 8, 40, 1024
# Compact view (int64 per env): rng.state, rng.inc, episode, hp, regen, blocks,
# player, ticks, killed, map_id, frontier_count, then pos[40], energy[40],
# hp[40], awake[40].
ROUTE_COMPACT = 11 + 4 * ROUTE_ENEMIES


class RouteTables(C.Structure):
    """learn.cu:130-139 with MULTI_MAP (the layout learn_env_ring_multi.py:11-17 fills)."""
    _fields_ = [(k, C.c_void_p) for k in ('floor', 'cells', 'index', 'distance')] + [
        ('ncells', C.c_int), ('map_ncells', C.c_void_p), ('distance_offsets', C.c_void_p), ('n_maps', C.c_int),
        ('map_filter', C.c_int)]


def route_library():
    path = HERE / '_ref' / 'learn_route.so'
    if not path.exists():
        return None
    lib = C.CDLL(str(path))
    p, i = C.c_void_p, C.c_int
    lib.learn_init.argtypes = [p, i, p, p, C.c_uint64, p, p, p, i]
    lib.learn_step.argtypes = [p, i, p, p, p, i, p, p, p, p, i]
    lib.learn_step_active.argtypes = [p, i, p, p, p, i, p, p, p, p, p, i]
    lib.learn_heuristic.argtypes = [p, i, p, p, p, p, i]
    return lib


def floor_from_bits(bits):
    """u8 [5600] floor from a row-padded bit plane u32 [210] (3 words per row)."""
    words = np.asarray(bits, np.uint32).reshape(70, 3)
    x = np.arange(80)
    return ((words[:, x // 32] >> (x % 32).astype(np.uint32)) & 1).astype(np.uint8).reshape(-1)


def route_map(floor, cells=None):
    """(floor u8[5600], cells i16[ncells], index i16[5600], distance u16[ncells, 5600])
    for one map; cells default to every floor cell in index order."""
    floor = np.ascontiguousarray(floor, np.uint8)
    if cells is None:
        cells = np.flatnonzero(floor).astype(np.int16)
    cells = np.ascontiguousarray(cells, np.int16)
    index = np.full(5600, -1, np.int16)
    index[cells] = np.arange(len(cells))
    distance = np.empty((len(cells), 5600), np.uint16)
    assert library().oracle_distance_table(floor.ctypes.data, cells.ctypes.data, len(cells),
                                           distance.ctypes.data) == 0
    return floor, cells, index, distance


def route_corpus(n_maps, spec_config_values, seed=0):
    """A small corpus in the reference's multi-map layout: map 0 is the fixture
    (its reachable cells, as learn_env.py:15-40 selects them), maps 1.. are the
    floors of the spec generator's maps for env ids 0..n_maps-2 under `seed`
    (the reference's 388-map native corpus is not available)."""
    _, _, floor, cells, index, distance = fixture()
    maps = [(floor, cells, index, distance)]
    if n_maps > 1:
        gen = OracleSpec(n_maps - 1, spec_config_values, seed=seed)
        fl, _ = gen.planes()
        maps += [route_map(floor_from_bits(fl[k])) for k in range(n_maps - 1)]
    return maps


def route_arrays(maps):
    """Concatenated table arrays as learn_env_ring_multi.py:60-70 builds them:
    floor u8[n*5600], cells i16[n*5600] (-1 padded per map), index i16[n*5600],
    distance u16[sum(ncells)*5600], map_ncells i32[n], distance_offsets i32[n]."""
    floors = np.concatenate([m[0] for m in maps]).astype(np.uint8)
    cells = np.full((len(maps), 5600), -1, np.int16)
    for k, m in enumerate(maps):
        cells[k, :len(m[1])] = m[1]
    index = np.concatenate([m[2] for m in maps]).astype(np.int16)
    distance = np.concatenate([m[3].reshape(-1) for m in maps]).astype(np.uint16)
    ncells = np.array([len(m[1]) for m in maps], np.int32)
    offsets = np.concatenate(([0], np.cumsum(ncells[:-1]))).astype(np.int32)
    return dict(floor=floors, cells=cells.reshape(-1), index=index, distance=distance, map_ncells=ncells,
                distance_offsets=offsets)


# Byte offsets in the reference's State for this build (learn.cu:106-129; World is
# RNG 16 B, hp/regen/blocks/fixture, u64 episode and 13 u64 stats = 144 B).
_RS = dict(rng=0, hp=16, regen=20, blocks=24, episode=32, player=144, ticks=148, killed=152, map_id=156, pos=160,
           energy=240, occ=320, mhp=11520, awake=11600, seen=11680, viewed=17280, fcells=22880, fslot=34080,
           fcount=45280)


class ReferenceRoute:
    """The reference's own route-cue build on the host (gpu=0) over a corpus."""

    def __init__(self, batch, maps, enemies=ROUTE_ENEMIES, seed=0, map_filter=-1):
        self.lib = route_library()
        if self.lib is None:
            raise FileNotFoundError('oracle/_ref/learn_route.so was not built')
        self.batch, self.enemies, self.limit = batch, enemies, ROUTE_LIMIT
        values = config_values(enemies)
        self.config = (C.c_int * len(values))(*values)
        self.arrays = route_arrays(maps)
        a = self.arrays
        self.tables = RouteTables(a['floor'].ctypes.data, a['cells'].ctypes.data, a['index'].ctypes.data,
                                  a['distance'].ctypes.data, int(a['map_ncells'][0]), a['map_ncells'].ctypes.data,
                                  a['distance_offsets'].ctypes.data, len(maps), map_filter)
        assert self.lib.learn_state_bytes() == 45288
        self.state = np.zeros((batch, self.lib.learn_state_bytes()), np.uint8)
        self.obs = np.zeros((batch, ROUTE_OBS), np.float32)
        self.mask = np.zeros((batch, ROUTE_ACTIONS), np.float32)
        self.out = np.zeros((batch, ROUTE_OUT), np.float32)
        self.actions = np.zeros(batch, np.int64)
        self.reset(seed)

    def reset(self, seed):
        assert self.lib.learn_init(self.state.ctypes.data, self.batch, C.byref(self.config), C.byref(self.tables),
                                   seed, self.obs.ctypes.data, self.mask.ctypes.data, None, 0) == 0
        return self.obs

    def step(self, actions, active=None, lo=0, hi=None):
        """Steps envs [lo, hi) (all by default; slices let a thread pool split the batch)."""
        hi = self.batch if hi is None else hi
        actions = np.ascontiguousarray(actions, np.int64)
        st, ob, mk, ou = (self.state[lo:hi], self.obs[lo:hi], self.mask[lo:hi], self.out[lo:hi])
        if active is None:
            self.lib.learn_step(st.ctypes.data, hi - lo, C.byref(self.config), C.byref(self.tables),
                                actions[lo:hi].ctypes.data, self.limit, ob.ctypes.data, mk.ctypes.data,
                                ou.ctypes.data, None, 0)
        else:
            act = np.ascontiguousarray(active, np.bool_)
            self.lib.learn_step_active(st.ctypes.data, hi - lo, C.byref(self.config), C.byref(self.tables),
                                       actions[lo:hi].ctypes.data, self.limit, ob.ctypes.data, mk.ctypes.data,
                                       ou.ctypes.data, act[lo:hi].ctypes.data, None, 0)
        return self.obs, self.out

    def heuristic(self):
        self.lib.learn_heuristic(self.state.ctypes.data, self.batch, C.byref(self.config), C.byref(self.tables),
                                 self.actions.ctypes.data, None, 0)
        return self.actions

    def _field(self, name, dtype, count=1):
        off = _RS[name]
        size = np.dtype(dtype).itemsize * count
        return self.state[:, off:off + size].copy().view(dtype).reshape(self.batch, count)

    def compact(self):
        """The compact view (ROUTE_COMPACT int64 per env) read from the reference's State bytes."""
        rng = self._field('rng', np.uint64, 2).view(np.int64)
        i32 = lambda k: self._field(k, np.int32).astype(np.int64)
        head = [rng[:, :1], rng[:, 1:], self._field('episode', np.uint64).view(np.int64), i32('hp'), i32('regen'),
                i32('blocks'), i32('player'), i32('ticks'), i32('killed'), i32('map_id'), i32('fcount')]
        mon = [self._field(k, np.int16, ROUTE_ENEMIES).astype(np.int64) for k in ('pos', 'energy', 'mhp', 'awake')]
        return np.concatenate(head + mon, axis=1)

    def viewed_bits(self):
        """The remembered-cell (viewed) plane as u32 [n, 210] row-padded bits."""
        v = self._field('viewed', np.uint8, 5600).reshape(self.batch, 70, 80).astype(np.uint32)
        out = np.zeros((self.batch, 70, 3), np.uint32)
        for x in range(80):
            out[:, :, x // 32] |= v[:, :, x] << np.uint32(x % 32)
        return out.reshape(self.batch, 210)

    def frontier(self):
        """The frontier list, i16 [n, 5600] with entries past the count set to -1."""
        cells = self._field('fcells', np.int16, 5600).copy()
        count = self._field('fcount', np.int32)[:, 0]
        cells[np.arange(5600)[None, :] >= count[:, None]] = -1
        return cells


# ------------------------------------------------------------------ semantic-actions build
class SemanticTables(C.Structure):
    """semantic-actions-v1 learn.cu:141-151 (MULTI_MAP, with the LOS table)."""
    _fields_ = [(k, C.c_void_p) for k in ('floor', 'cells', 'index', 'distance')] + [
        ('ncells', C.c_int), ('map_ncells', C.c_void_p), ('distance_offsets', C.c_void_p), ('n_maps', C.c_int),
        ('map_filter', C.c_int), ('los', C.c_void_p)]


# semantic_harness.cu's field numbers for sem_offset
SEM_FIELDS = ('hp', 'regen', 'player', 'ticks', 'killed', 'pos', 'energy', 'mhp', 'awake', 'occ', 'viewed', 'seen',
              'floor_seen', 'enemy_slot')
# The build's five actions (semantic-actions-v1 learn.cu:800)
SEM_ATTACK, SEM_EXPLORE, SEM_ENGAGE, SEM_WAIT, SEM_REST = range(5)


def semantic_library():
    """The reference's semantic-actions build driven by oracle/semantic_harness.cu
    (host code), or None when it was not built here."""
    path = HERE / '_ref' / 'semantic_rules.so'
    if not path.exists():
        return None
    lib = C.CDLL(str(path))
    p, i = C.c_void_p, C.c_int
    lib.sem_empty.argtypes = [p, p, p, i, i, i, C.c_uint64]
    lib.sem_put.argtypes = [p, p, p, i, i, i, i]
    lib.sem_transition.argtypes = [p, p, p, i, i, p]
    lib.sem_primitive.argtypes = [p, p, p, i, i, p]
    lib.sem_observe.argtypes = [p, p, p, p, p]
    lib.sem_adjacent_attack.argtypes = [p, p, p]
    lib.sem_visible_awake.argtypes = [p, p, p]
    lib.sem_in_view.argtypes = [p, p, i]
    lib.sem_detects.argtypes = [p, p, i]
    return lib


class SemanticReference:
    """One hand-built env of the reference's semantic-actions build on the fixture
    map (map 0 of a one-map corpus, its native LOS table), on the host.

    `spec` is a spec-task config dict (d1.spec_env.DEFAULT's keys): the player's
    HP, defence and regeneration and kinds 0-3 are copied into the build's Config
    (sim.h:64-67; count = the build's REQUIRED regular monsters, as its reset
    asserts without ogres), so both tasks play the same numbers. Monster slot `id` has kind c.kinds[id % 6]; slots from
    sem_required() on are the build's ogres, which these cases never use."""

    def __init__(self, spec):
        lib = semantic_library()
        if lib is None:
            raise RuntimeError('oracle/_ref/semantic_rules.so is not built (make -C oracle ref)')
        self.lib = lib
        z = np.load(DATA / 'fixture_1057.npz')
        floor, native_los = z['floor'], z['native_los']
        _, _, _, cells, index, distance = fixture()
        arrays = route_arrays([(floor, cells, index, distance)])
        arrays['los'] = np.ascontiguousarray(native_los, np.uint32).reshape(-1)
        self.arrays = arrays
        self.tables = SemanticTables(*(arrays[k].ctypes.data for k in ('floor', 'cells', 'index', 'distance')),
                                     len(cells), arrays['map_ncells'].ctypes.data,
                                     arrays['distance_offsets'].ctypes.data, 1, 0, arrays['los'].ctypes.data)
        kinds = list(spec['kinds'][:4]) + list(spec['kinds'][:2])
        values = [lib.sem_required(), 0, spec['hp'], spec['ac100'], spec['ev100'], spec['sh100'],
                  spec['shield_limit'], spec['regen'], 1, *spec['gdr'], *[v for k in kinds for v in k]]
        self.config = (C.c_int * len(values))(*values)
        self.state = np.zeros(lib.sem_state_bytes(), np.uint8)
        self.obs = np.zeros(lib.sem_obs_size(), np.float32)
        self.mask = np.zeros(lib.sem_action_size(), np.float32)
        self.out = np.zeros(lib.sem_out_size(), np.float32)
        self.off = {k: lib.sem_offset(i) for i, k in enumerate(SEM_FIELDS)}
        self.floor = floor

    def _args(self):
        return self.state.ctypes.data, C.byref(self.config), C.byref(self.tables)

    def empty(self, player, hp, ticks=0, seed=0):
        self.lib.sem_empty(*self._args(), player, hp, ticks, seed)

    def put(self, slot, pos, hp, awake):
        self.lib.sem_put(*self._args(), slot, pos, hp, int(awake))

    def step(self, action, limit=2048):
        self.lib.sem_transition(*self._args(), action, limit, self.out.ctypes.data)
        return self.out.copy()

    def primitive(self, d, limit=2048):
        self.lib.sem_primitive(*self._args(), d, limit, self.out.ctypes.data)
        return self.out.copy()

    def viewed(self):
        o = self.off['viewed']
        return self.state[o:o + 5600].copy()

    def observe(self):
        self.lib.sem_observe(*self._args(), self.obs.ctypes.data, self.mask.ctypes.data)
        return self.mask.copy()

    def attack_dir(self):
        return self.lib.sem_adjacent_attack(*self._args())

    def visible_awake(self):
        return bool(self.lib.sem_visible_awake(*self._args()))

    def detects(self, origin):
        return bool(self.lib.sem_detects(self.state.ctypes.data, C.byref(self.tables), origin))

    def field(self, name, index=None, dtype=np.int32):
        o = self.off[name]
        if name in ('pos', 'energy', 'mhp', 'awake', 'occ', 'enemy_slot'):
            dtype, o = np.int16, o + 2 * (index or 0)
        elif name in ('viewed', 'seen'):
            dtype, o = np.uint8, o + (index or 0)
        return int(self.state[o:o + np.dtype(dtype).itemsize].view(dtype)[0])
