"""Hand-built states of the BASELINE (spec) task for rule tests, in both layouts:
the GPU state row of libd1 (include/d1.h, d1_spec_observe) and the CPU
oracle's struct (oracle/d1_oracle.c, Spec).

A case is an open rectangular room (walls around it), the player with a given HP
and turn count, and up to 11 monsters placed by hand. As in the reference's
isolated()/put() (gpu-d1/branches/semantic-actions-v1/src/semantic_tests.cu:
2-8), everything in the player's view is already remembered and every monster
holds energy -30000 (an awake one therefore only acts after waking afresh).
"""
import numpy as np

import oracle

W, H, N = 80, 70, 5600
GPU_ROW, ORACLE_ROW = 7680, 1888


def plane(bits_u8):
    """u8[5600] -> row-padded bit plane u32[210]."""
    v = np.asarray(bits_u8, np.uint32).reshape(H, W)
    out = np.zeros((H, 3), np.uint32)
    for x in range(W):
        out[:, x // 32] |= v[:, x] << np.uint32(x % 32)
    return out.reshape(-1)


def build(player=(40, 35), hp=3, ticks=0, mons=(), room=(25, 25, 60, 45), stairs=(30, 30), env=0, seed=5,
          floor=None, energy=None):
    """mons: (x, y, hp, kind, awake) tuples. `floor` (u8[5600]) replaces the
    rectangular room when given; `energy` (one value per monster) replaces the
    default -30000."""
    if floor is None:
        floor = np.zeros((H, W), np.uint8)
        x0, y0, x1, y1 = room
        floor[y0:y1 + 1, x0:x1 + 1] = 1
    floor = np.ascontiguousarray(floor, np.uint8).reshape(-1)
    p = player[1] * W + player[0]
    los = oracle.los_mask(floor, p)  # 17x17, bit (dy+8)*17 + dx+8
    vis = np.zeros(15, np.uint32)
    viewed = np.zeros(N, np.uint8)
    for dy in range(-7, 8):
        for dx in range(-7, 8):
            bit = (dy + 8) * 17 + dx + 8
            if (int(los[bit // 32]) >> (bit % 32)) & 1:
                vis[dy + 7] |= np.uint32(1 << (dx + 7))
                viewed[(player[1] + dy) * W + player[0] + dx] = 1
    return dict(env=env, seed=seed, hp=hp, ticks=ticks, player=p, stairs=stairs[1] * W + stairs[0],
                nmon=len(mons), floor_seen=int((viewed & floor).sum()), mons=list(mons),
                energy=list(energy) if energy is not None else [-30000] * len(mons),
                floor=plane(floor), viewed=plane(viewed), vis=vis)


def gpu_row(c):
    r = np.zeros(GPU_ROW, np.uint8)
    u = r[:64].view(np.uint32)
    u[2], u[3], u[4], u[5] = c['env'], c['seed'] & 0xffffffff, c['seed'] >> 32, 0
    r[24:60].view(np.int32)[:] = [c['hp'], 0, 0, c['player'], c['ticks'], 0, c['stairs'], c['nmon'],
                                 c['floor_seen']]
    r[64:64 + 30].view(np.uint16)[:] = c['vis'].astype(np.uint16)
    m = r[128:224].view(np.int16)
    for i, (x, y, mh, kind, awake) in enumerate(c['mons']):
        m[i], m[16 + i], m[32 + i] = y * W + x, c['energy'][i], mh
        r[224 + i], r[240 + i] = kind, awake
    r[256:256 + 840] = c['floor'].view(np.uint8)
    r[1096:1096 + 840] = c['viewed'].view(np.uint8)
    return r


def oracle_row(c):
    r = np.zeros(ORACLE_ROW, np.uint8)
    u = r[:24].view(np.uint32)
    u[2], u[3], u[4], u[5] = c['env'], c['seed'] & 0xffffffff, c['seed'] >> 32, 0
    r[24:60].view(np.int32)[:] = [c['hp'], 0, 0, c['player'], c['ticks'], 0, c['stairs'], c['nmon'],
                                 c['floor_seen']]
    pos, en, mh = r[60:82].view(np.int16), r[82:104].view(np.int16), r[104:126].view(np.int16)
    for i, (x, y, hp, kind, awake) in enumerate(c['mons']):
        pos[i], en[i], mh[i] = y * W + x, c['energy'][i], hp
        r[126 + i], r[137 + i] = kind, awake
    r[148:148 + 840] = c['floor'].view(np.uint8)
    r[988:988 + 840] = c['viewed'].view(np.uint8)
    r[1828:1888] = c['vis'].view(np.uint8)
    return r


class OracleCase:
    """One hand-built env on the CPU oracle."""

    def __init__(self, case, config):
        self.env = oracle.OracleSpec(1, config)
        assert self.env.state.shape[1] == ORACLE_ROW
        self.env.state[0] = oracle_row(case)
        lib = self.env.lib
        import ctypes as C
        lib.oracle_spec_observe.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        lib.oracle_spec_observe(self.env.state.ctypes.data, 1, C.byref(self.env.config), self.env.obs.ctypes.data,
                                self.env.legal.ctypes.data)

    def step(self, a):
        self.env.step(np.array([a], np.int64))
        return self.env.out[0].copy()

    @property
    def legal(self):
        return int(self.env.legal[0])

    @property
    def row(self):
        return self.env.state[0].copy()

    def compact(self):
        return self.env.compact()[0]

    def obs(self):
        return self.env.obs[0].copy()


class GpuCase:
    """One hand-built env on libd1 (d1_spec_observe / d1_spec_step)."""

    def __init__(self, case, config):
        import torch
        from d1.spec_env import SpecEnv
        self.torch = torch
        self.env = SpecEnv(1, config=config)
        self.env.state[0] = torch.from_numpy(gpu_row(case)).cuda()
        self.env.observe()

    def step(self, a):
        self.env.step(self.torch.tensor([a], dtype=self.torch.int64, device='cuda'))
        return self.env.out[0].cpu().numpy()

    @property
    def legal(self):
        return int(self.env.legal[0].item()) & 0xffff

    @property
    def row(self):
        return self.env.state[0].cpu().numpy()

    def compact(self):
        return self.env.compact()[0].cpu().numpy()

    def obs(self):
        return self.env.obs[0].float().cpu().numpy()
