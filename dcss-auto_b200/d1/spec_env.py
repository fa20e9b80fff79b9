"""The BASELINE D:1 task on the B200 kernels (configs 0, 1 and 4).

`SpecEnv` keeps the reference Env's shape -- `reset(seed)`, `step(actions,
active=None) -> (obs, out)` and resident tensors -- with the spec task's
buffers: obs bf16 [n, 1832] (one-hot 15x15 window x 8 channels + 32 scalars),
legal u16 [n] (bit a set when action a is legal), out f32 [n, 10]. The
observation can be written straight into a caller-provided buffer via
`step(actions, obs_out=...)`, and the compact observation (320 B per env: a
channel byte per window cell and the 32 scalars as bf16; `expand_cobs` turns it
back into the one-hot form) into a rollout slot via `cobs_out=...`.

Env ids are global (`first_env + i`), so a shard of a multi-GPU run produces
exactly the trajectories the same ids would produce on one GPU.
"""
import ctypes as C
import pathlib

import numpy as np
import torch

from ._lib import check, library, resolve_device, launch_stream

DATA = pathlib.Path(__file__).resolve().parent / 'data'

OBS, ACTIONS, OUT, COMPACT = 1832, 12, 10, 56
ACTION_NAMES = ['N', 'E', 'S', 'W', 'NE', 'SE', 'SW', 'NW', 'wait', 'rest', 'attack', 'descend']


class Kind(C.Structure):
    _fields_ = [(k, C.c_int) for k in ('speed', 'damage', 'tohit', 'bypass')]


class SpecConfig(C.Structure):
    _fields_ = ([(k, C.c_int) for k in ('hp', 'ac100', 'ev100', 'sh100', 'shield_limit', 'regen')]
                + [('gdr', C.c_int * 2)]
                + [(k, C.c_int) for k in ('min_monsters', 'max_monsters', 'min_mhp', 'max_mhp', 'ogre', 'ogre_hp',
                                          'ogre_min_damage', 'limit', 'explore_milli', 'kill_milli',
                                          'descend_milli', 'death_milli')]
                + [('kinds', Kind * 5)])


def gdr_for(ac100):
    """Cached GDR pair for AC = ac100 // 100 and +1 (gpu-d1/scripts/learn_env.py:67-68)."""
    ac = ac100 // 100
    return tuple(int((65536 * (ac + j)) ** 0.25) for j in range(2))


# BASELINE config 0/1: player HP 15 AC 2 (EV, SH, shield limit and regeneration
# from the reference fixture header), 3-10 monsters with HP 2-8 drawn from rat,
# jackal, goblin and kobold; config 4 adds one sleeping ogre (HP 30, damage 2-17).
# Kind rows are (speed, max damage, to-hit, bypass); rat, jackal and goblin are
# the reference fixture's roster entries, kobold and ogre are added here.
DEFAULT = dict(hp=15, ac100=200, ev100=794, sh100=906, shield_limit=2, regen=23, gdr=gdr_for(200),
               min_monsters=3, max_monsters=10, min_mhp=2, max_mhp=8, ogre=0, ogre_hp=30, ogre_min_damage=2,
               limit=512, explore_milli=2, kill_milli=1000, descend_milli=3000, death_milli=1000,
               kinds=[(10, 3, 19, 15), (14, 3, 19, 15), (10, 1, 19, 15), (10, 4, 19, 15), (5, 17, 30, 25)])
OGRE = dict(DEFAULT, ogre=1)


def make_config(values=None):
    values = dict(DEFAULT if values is None else values)
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


_RAYS = {}


def device_rays(device):
    """Register the native LOS ray fan with the library (packed once per device:
    4 x u32 per ray = blocker mask lo, hi, end bit index, 0)."""
    key = str(device)
    if key not in _RAYS:
        z = np.load(DATA / 'los_rays.npz')
        blk = z['blockers'].astype(np.uint64)
        packed = np.zeros((len(blk), 4), np.uint32)
        packed[:, 0] = (blk & np.uint64(0xffffffff)).astype(np.uint32)
        packed[:, 1] = (blk >> np.uint64(32)).astype(np.uint32)
        packed[:, 2] = (z['end_y'] * 8 + z['end_x']).astype(np.uint32)
        _RAYS[key] = torch.from_numpy(packed.view(np.int32)).to(device)
    rays = _RAYS[key]
    check(library().d1_spec_set_rays(rays.data_ptr(), rays.shape[0]), 'd1_spec_set_rays')
    return rays


COBS, COBS_SCALARS, CELLS = 320, 256, 225


def expand_cobs(cobs):
    """One-hot bf16 observations [n, 1832] of compact rows u8 [n, 320] (torch
    ops; the kernels expand the same way inside d1_ppo_gather_cobs)."""
    codes = cobs[:, :CELLS].long()
    onehot = torch.nn.functional.one_hot(codes, 8).to(torch.bfloat16).reshape(cobs.shape[0], CELLS * 8)
    scalars = cobs[:, COBS_SCALARS:COBS].contiguous().view(torch.bfloat16)
    return torch.cat([onehot, scalars], 1)


class SpecEnv:
    def __init__(self, batch, config=None, seed=0, first_env=0, device='cuda', observe=True):
        """observe=False skips the 1832-feature observation writes (the conv
        policy reads the env state through d1_spec_crop instead); legal bits and
        outcomes are still written."""
        self.device = resolve_device(device)
        if self.device.type != 'cuda':
            raise ValueError('libd1 runs on CUDA devices only; use the oracle for CPU reference runs')
        self.lib = library()
        self.batch, self.first_env = batch, first_env
        self.values = dict(DEFAULT if config is None else config)
        self.config = make_config(self.values)
        assert C.sizeof(self.config) == self.lib.d1_spec_config_bytes()
        with torch.cuda.device(self.device):
            self.rays = device_rays(self.device)
        self.state = torch.zeros((batch, self.lib.d1_spec_state_bytes()), dtype=torch.uint8, device=self.device)  # row tail is padding
        self.obs = torch.empty((batch, OBS), dtype=torch.bfloat16, device=self.device) if observe else None
        self.legal = torch.empty(batch, dtype=torch.int16, device=self.device)  # u16 bits
        self.out = torch.zeros((batch, OUT), device=self.device)
        self.reset(seed)

    @property
    def stream(self):
        return launch_stream(self.device)

    def reset(self, seed, obs_out=None, legal_out=None, cobs_out=None):
        obs = self.obs if obs_out is None else obs_out
        legal = self.legal if legal_out is None else legal_out
        check(self.lib.d1_spec_init_ex(self.state.data_ptr(), self.batch, C.byref(self.config), seed, self.first_env,
                                       None if obs is None else obs.data_ptr(),
                                       None if cobs_out is None else cobs_out.data_ptr(), legal.data_ptr(),
                                       self.stream), 'd1_spec_init_ex')
        return obs

    def step(self, actions, active=None, obs_out=None, legal_out=None, out_out=None, cobs_out=None, rows=None):
        """One semantic decision per env. `obs_out`/`legal_out`/`out_out`/`cobs_out`
        let the caller point the writes at rollout-buffer slots (no extra copies).
        rows=(lo, hi) steps only envs lo..hi-1 of the batch (every tensor is still
        the whole batch's; the launch reads and writes its rows only), so that
        parts of one batch can run on different streams."""
        assert actions.device == self.device and actions.dtype == torch.int64 and actions.is_contiguous()
        lo, hi = (0, self.batch) if rows is None else rows
        assert 0 <= lo <= hi <= self.batch and actions.shape[0] == self.batch
        act = 0
        if active is not None:
            assert active.device == self.device and active.dtype == torch.bool and active.shape == (self.batch,)
            act = active[lo:hi].data_ptr()
        obs = self.obs if obs_out is None else obs_out
        legal = self.legal if legal_out is None else legal_out
        out = self.out if out_out is None else out_out
        assert out.dim() == 2 and out.shape == (self.batch, OUT) and out.dtype == torch.float32
        # any [B, 10] view: row-major, or a transposed view of a [10, B] plane stack
        check(self.lib.d1_spec_step_strided(self.state[lo:hi].data_ptr(), hi - lo, C.byref(self.config),
                                            actions[lo:hi].data_ptr(), None if obs is None else obs[lo:hi].data_ptr(),
                                            None if cobs_out is None else cobs_out[lo:hi].data_ptr(),
                                            legal[lo:hi].data_ptr(), out[lo:hi].data_ptr(), out.stride(0),
                                            out.stride(1), act or None, self.stream),
              'd1_spec_step_strided')
        return obs, out

    def observe(self, obs_out=None, legal_out=None, cobs_out=None):
        """Observation and legal bits of the rows as they are (no step)."""
        obs = self.obs if obs_out is None else obs_out
        legal = self.legal if legal_out is None else legal_out
        check(self.lib.d1_spec_observe(self.state.data_ptr(), self.batch, C.byref(self.config),
                                       None if obs is None else obs.data_ptr(),
                                       None if cobs_out is None else cobs_out.data_ptr(), legal.data_ptr(),
                                       self.stream), 'd1_spec_observe')
        return obs

    def legal_mask(self):
        """Legal actions as a float [n, 12] mask (the reference's mask layout)."""
        bits = self.legal.to(torch.int32) & 0xffff
        return ((bits[:, None] >> torch.arange(ACTIONS, device=self.device)) & 1).float()

    def compact(self):
        rows = torch.empty((self.batch, COMPACT), dtype=torch.int64, device=self.device)
        check(self.lib.d1_spec_compact(self.state.data_ptr(), self.batch, rows.data_ptr(), self.stream))
        return rows

    def planes(self):
        f = torch.empty((self.batch, 210), dtype=torch.int32, device=self.device)
        v = torch.empty((self.batch, 210), dtype=torch.int32, device=self.device)
        check(self.lib.d1_spec_planes(self.state.data_ptr(), self.batch, f.data_ptr(), v.data_ptr(), self.stream))
        return f, v
