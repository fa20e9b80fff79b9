// The BASELINE D:1 task ("spec") on sm_100a: generated rooms+corridors maps, a
// per-env Philox4x32-10 stream, 12 semantic actions, and a one-hot 15x15x8 + 32
// bf16 observation written straight into the policy input buffer.
//
// One warp per environment (see d1_common.cuh). Everything spatial is lane-
// parallel over 80x70 bit planes held in shared memory: map generation is a
// rasterisation of the room/corridor rectangles, LOS is the native Crawl ray fan
// evaluated as 64-bit quadrant masks, the monster pursuit field is a layered
// bitset BFS that stops one layer past the farthest awake monster, and each
// observation cell is one 16-byte store of eight bf16 channels.
//
// State row (7680 B per env):
//   0    u64 ctr (Philox draws consumed)   8 u32 env, seed_lo, seed_hi, episode
//   24   i32 hp, regen, blocks, player     40 i32 ticks, killed, stairs, nmon
//   56   i32 floor_seen                    64 u16 vis[16] (LOS window rows, dy+7 -> bit dx+7)
//   96..127 unused
//   128  i16 pos[16]  160 i16 energy[16]  192 i16 hp[16]  224 u8 kind[16]  240 u8 awake[16]
//   256  u32 floor[210]  (row y = words 3y..3y+2, bit x%32 of word x/32)
//   1096 u32 viewed[210] (cells ever in view: remembered terrain)
//   2048 u8 dist[5600]   (pursuit BFS distance mod 256, valid where reached;
//                         scratch of the step, kept in the row so that the
//                         shared memory per env -- the occupancy limit -- is
//                         4.6 KB instead of 10.2 KB)
#include <cuda_bf16.h>

#include "d1_common.cuh"
#include "d1_pdl.cuh"

namespace d1 {
namespace spec {

constexpr int MAXM = 11, OBS = 1832, CELLS = 225, ACTIONS = 12, OUT = 10, COMPACT = 56;
// Compact observation row: the channel (0-7) of each window cell as a byte
// (0-224, then zeros to 255), the 32 scalars as bf16 at byte 256.
constexpr int COBS = 320, COBS_SCALARS = 256;
// Divisors of the 32 observation scalars (entries 0 and 2 are the config's HP
// and turn limit, filled in by the caller).
__device__ const float SCALAR_DEN[32] = {1.f, 100.f, 1.f,  10.f, 80.f, 70.f, 10.f, 10.f, 1.f, 7.f,  7.f,
                                         16.f, 1.f,  4.f,  1.f,  80.f, 70.f, 1.f,  8.f,  16.f, 1.f, 1.f,
                                         1024.f, 2.f, 1.f, 1.f, 7.f,  7.f,  1.f,  30.f, 1.f, 1.f};
constexpr int ROW = 7680, OFF_DIST = 2048, PL = 210, OFF_VIS = 64, OFF_MON = 128, OFF_FLOOR = 256, OFF_VIEWED = 256 + 4 * PL;
#ifndef D1_SPEC_WARPS
#define D1_SPEC_WARPS 1
#endif
#ifndef D1_SPEC_MIN_WARPS
#define D1_SPEC_MIN_WARPS 32
#endif
// Warps (envs) per block, and the resident warps per SM the register budget is
// sized for (a launch-bounds hint). The step is latency bound (an SM with 15 %
// fewer resident envs took 7 % longer), so the budget is 32 warps: 62
// registers without spills, 4.6 KB of shared memory per env, and 32 one-warp
// blocks -- the SM's block limit -- resident per SM.
constexpr int WARPS = D1_SPEC_WARPS, MIN_BLOCKS = (D1_SPEC_MIN_WARPS + D1_SPEC_WARPS - 1) / D1_SPEC_WARPS;
constexpr int MAX_RAYS = 320;
constexpr int PRIM_WAIT = 8, PRIM_DESCEND = 9;

// ------------------------------------------------------------------ RNG
// Philox4x32-10 (Salmon et al., SC'11). Draw n of env e under seed s is word
// n & 3 of philox(ctr = {lo(n>>2), hi(n>>2), hi(s), 0}, key = {e, lo(s)}).
__device__ __forceinline__ uint4 philox(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    }
    return c;
}
// One out-of-line copy of the ten rounds: every draw site of the rules shares it,
// which keeps the hot loop small enough for the instruction cache.
__device__ __noinline__ uint4 philox_block(uint64_t b, uint32_t c2, uint32_t k0, uint32_t k1) {
    return philox(make_uint4((uint32_t)b, (uint32_t)(b >> 32), c2, 0u), k0, k1);
}
// Warp-cooperative stream: lane j holds block (base + j), so one refill (one
// Philox evaluation per lane) serves the next 128 draws of the env; a draw is a
// select plus one shuffle. Only ever called from warp-uniform code.
struct WarpPhilox {
    uint64_t n, base;
    uint32_t k0, k1, c2;
    uint4 blk;
    int lane;
    __device__ __forceinline__ void refill() {
        base = n >> 2;
        blk = philox_block(base + (uint64_t)lane, c2, k0, k1);
    }
    __device__ __forceinline__ uint32_t next() {
        const uint64_t b = n >> 2;
        if (b - base >= 32) refill();
        const uint32_t sel = (uint32_t)n & 3u;
        const uint32_t mine = sel == 0 ? blk.x : sel == 1 ? blk.y : sel == 2 ? blk.z : blk.w;
        const uint32_t v = __shfl_sync(FULL, mine, (int)(b - base));
        n++;
        return v;
    }
};

// ------------------------------------------------------------------ state
struct Smem {
    uint32_t floor[PL], viewed[PL], seen[PL], cur[PL];
    uint32_t occ[PL];  // live monster positions during the monster phase
    uint32_t vis[16];  // LOS window rows: vis[dy+7] bit dx+7
    uint16_t vmask[16], fmask[16];  // remembered / floor bits of the window rows
    uint4 onehot[8];  // observation cell of channel c: bf16 1.0 in half-word c
    uint4 crow[COBS / 16];  // the compact observation row, staged for 16-byte stores
    uint8_t opqb[32];
    uint8_t occ_ch[CELLS + 7];
};
// The LOS ray fan in global memory (2.2 KB, L1-resident): per ray a 64-bit
// blocker mask over the 8x8 quadrant and its end cell.
struct RayArgs {
    const uint4 *ray;  // {blocker mask lo, hi, end bit index ey*8+ex, 0}
    int n;
};

struct Env {
    WarpPhilox rng;
    uint32_t env, episode;
    int hp, regen, blocks, player, ticks, killed, stairs, nmon, floor_seen;
    // lane-distributed monster slot (lane < MAXM), hp 0 when empty
    int m_pos, m_energy, m_hp, m_kind, m_awake, m_dist;
    int lane, dirty_lo, dirty_hi;
    bool floor_dirty;
    Smem *sm;
    uint8_t *dist;  // this env's BFS distance field (global, in the state row)
};

__device__ __forceinline__ int bitp(const uint32_t *plane, int p) {
    const int x = p % W, y = p / W;
    return (plane[y * 3 + (x >> 5)] >> (x & 31)) & 1;
}
__device__ __forceinline__ bool floor_at(const Env &e, int p) { return p >= 0 && p < N && bitp(e.sm->floor, p); }

__device__ __forceinline__ D1Kind kind_of(const D1SpecConfig &c, int k) {
    D1Kind r = c.kinds[0];
#pragma unroll
    for (int j = 1; j < 5; j++)
        if (k == j) r = c.kinds[j];
    return r;
}

// Bits [s, s+15) of a 3-word row, zero outside the row; s in [-7, 72].
__device__ __forceinline__ uint32_t row15(const uint32_t *r, int s) {
    uint64_t a;
    int t;
    if (s >= 32) {
        a = (uint64_t)r[1] | ((uint64_t)r[2] << 32);
        t = s - 32;
    } else {
        a = (uint64_t)r[0] | ((uint64_t)r[1] << 32);
        t = s;
    }
    const uint64_t v = t >= 0 ? (a >> t) : (a << (-t));
    return (uint32_t)v & 0x7fffu;
}
// OR a 15-bit mask into a 3-word row at bit offset s (s may be negative).
__device__ __forceinline__ void or_row15(uint32_t *r, int s, uint32_t m) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
        const int sh = s - 32 * i;
        uint32_t part = 0;
        if (sh >= 0 && sh < 32) part = (uint32_t)((uint64_t)m << sh);
        else if (sh < 0 && sh > -15) part = m >> (-sh);
        r[i] |= part;
    }
}

// ------------------------------------------------------------------ LOS
// Native ray fan (gpu-d1/scripts/compile_corpus.py:67-81) for the 15x15 view:
// in each quadrant a ray dies on any in-map wall it crosses; live rays light
// their end cell if it is on the map; the origin is always lit.
__device__ void compute_los(Env &e, const RayArgs &ra) {
    Smem &s = *e.sm;
    const int lane = e.lane, px = e.player % W, py = e.player / W;
    {
        // lane = quadrant q * 8 + row y: the 8 cells x = 0..7 outward from the
        // player in that quadrant row; opaque = on the map and not floor.
        const int q = lane >> 3, y = lane & 7;
        const bool east = (q == 0 || q == 3);
        const int sy = (q < 2) ? 1 : -1;
        const int cy = py + sy * y;
        uint32_t b = 0;
        if (cy >= 0 && cy < H) {
            const uint32_t *row = s.floor + cy * 3;
            // 15 columns px-7 .. px+7 and which of them are on the map
            const uint32_t fl = row15(row, px - 7);
            uint32_t on = 0x7fffu;
            if (px - 7 < 0) on &= 0x7fffu << (7 - px);
            if (px + 7 > W - 1) on &= 0x7fffu >> (px + 7 - (W - 1));
            const uint32_t opq15 = on & ~fl;
            b = east ? (opq15 >> 7) & 0xffu : (__brev(opq15) >> 24) & 0xffu;  // west: bit x = column px - x
        }
        s.opqb[lane] = (uint8_t)b;
    }
    __syncwarp();
    const unsigned long long o0 = *reinterpret_cast<const unsigned long long *>(s.opqb + 0);
    const unsigned long long o1 = *reinterpret_cast<const unsigned long long *>(s.opqb + 8);
    const unsigned long long o2 = *reinterpret_cast<const unsigned long long *>(s.opqb + 16);
    const unsigned long long o3 = *reinterpret_cast<const unsigned long long *>(s.opqb + 24);
    unsigned long long v0 = 0, v1 = 0, v2 = 0, v3 = 0;
    // Rolled for the same reason as observe's cell loop (instruction fetch).
#pragma unroll 1
    for (int i = 0; i < (ra.n + 31) / 32; i++) {
        const int r = lane + 32 * i;
        const uint4 rv = r < ra.n ? __ldg(ra.ray + r) : make_uint4(0xffffffffu, 0xffffffffu, 0u, 0u);
        const unsigned long long blk = (unsigned long long)rv.x | ((unsigned long long)rv.y << 32);
        const unsigned long long endb = 1ull << rv.z;
        if (!(blk & o0)) v0 |= endb;
        if (!(blk & o1)) v1 |= endb;
        if (!(blk & o2)) v2 |= endb;
        if (!(blk & o3)) v3 |= endb;
    }
    // OR across lanes.
    uint32_t w[8] = {(uint32_t)v0, (uint32_t)(v0 >> 32), (uint32_t)v1, (uint32_t)(v1 >> 32),
                     (uint32_t)v2, (uint32_t)(v2 >> 32), (uint32_t)v3, (uint32_t)(v3 >> 32)};
#pragma unroll
    for (int i = 0; i < 8; i++) w[i] = __reduce_or_sync(FULL, w[i]);
    // Compose row dy = lane - 7 of the window. Quadrant q uses (sx, sy) =
    // (+,+), (-,+), (-,-), (+,-); its byte |dy| holds dx = 0..7 outward.
    if (lane < 15) {
        const int dy = lane - 7, ay = dy < 0 ? -dy : dy;
        const int sh = (ay & 3) * 8;
        const int hiw = ay >> 2;
        uint32_t pos = 0, neg = 0;  // x >= 0 side, x <= 0 side (before reversal)
        const uint32_t q0 = hiw ? w[1] : w[0], q1 = hiw ? w[3] : w[2];
        const uint32_t q2 = hiw ? w[5] : w[4], q3 = hiw ? w[7] : w[6];
        if (dy >= 0) {
            pos |= (q0 >> sh) & 0xffu;  // q0 (+,+)
            neg |= (q1 >> sh) & 0xffu;  // q1 (-,+)
        }
        if (dy <= 0) {
            pos |= (q3 >> sh) & 0xffu;  // q3 (+,-)
            neg |= (q2 >> sh) & 0xffu;  // q2 (-,-)
        }
        uint32_t row = (pos << 7) | (__brev(neg) >> 24);
        if (dy == 0) row |= 1u << 7;
        const int cy = py + dy;
        if (cy < 0 || cy >= H) row = 0;
        // Columns off the map are never lit.
        const int lo = 7 - px;       // window column of x = 0
        const int hi = 7 + (W - 1 - px);
        if (lo > 0) row &= ~((1u << lo) - 1u);
        if (hi < 14) row &= (1u << (hi + 1)) - 1u;
        s.vis[lane] = row;
    }
    if (lane == 15) s.vis[15] = 0;
    __syncwarp();
}

__device__ __forceinline__ bool visible(const Env &e, int p) {
    const int dx = p % W - e.player % W, dy = p / W - e.player / W;
    if (dx < -7 || dx > 7 || dy < -7 || dy > 7) return false;
    return (e.sm->vis[dy + 7] >> (dx + 7)) & 1u;
}

// Mark everything in view as remembered; return the number of newly seen floor
// cells (semantic-actions-v1 learn.cu:296-331 with MARK_WALLS).
__device__ int reveal(Env &e) {
    Smem &s = *e.sm;
    const int px = e.player % W, py = e.player / W;
    int newly = 0;
    if (e.lane < 15) {
        const int cy = py + e.lane - 7;
        if (cy >= 0 && cy < H) {
            uint32_t *vr = s.viewed + cy * 3;
            const uint32_t *fr = s.floor + cy * 3;
            const uint32_t fresh = s.vis[e.lane] & ~row15(vr, px - 7);
            newly = __popc(fresh & row15(fr, px - 7));
            or_row15(vr, px - 7, fresh);
        }
    }
    newly = __reduce_add_sync(FULL, newly);
    __syncwarp();
    e.floor_seen += newly;
    e.dirty_lo = imin(e.dirty_lo, imax(0, py - 7));
    e.dirty_hi = imax(e.dirty_hi, imin(H - 1, py + 7));
    return newly;
}

// ------------------------------------------------------------------ map generation
// 4-9 rooms (sides 4-12) inside the wall border; room k joins room k-1 by an L
// corridor between centres (horizontal- or vertical-first by a coin flip). The
// rectangles are drawn in order on one lane-distributed list, then rasterised
// with each lane owning rows lane, lane+32, lane+64.
__device__ void gen_map(Env &e) {
    Smem &s = *e.sm;
    int rx0 = 0, ry0 = 0, rx1 = -1, ry1 = -1;  // rectangle `lane`
    int nrect = 0;
    const int rooms = 4 + rng_r(e.rng, 6);
    int pcx = 0, pcy = 0;
    for (int k = 0; k < rooms; k++) {
        const int w = 4 + rng_r(e.rng, 9), h = 4 + rng_r(e.rng, 9);
        const int x0 = 1 + rng_r(e.rng, W - w - 1), y0 = 1 + rng_r(e.rng, H - h - 1);
        if (e.lane == nrect) {
            rx0 = x0; ry0 = y0; rx1 = x0 + w - 1; ry1 = y0 + h - 1;
        }
        nrect++;
        const int cx = x0 + w / 2, cy = y0 + h / 2;
        if (k > 0) {
            int ax0, ay0, ax1, ay1, bx0, by0, bx1, by1;
            if (rng_r(e.rng, 2) == 0) {
                ax0 = pcx; ay0 = pcy; ax1 = cx; ay1 = pcy;
                bx0 = cx; by0 = pcy; bx1 = cx; by1 = cy;
            } else {
                ax0 = pcx; ay0 = pcy; ax1 = pcx; ay1 = cy;
                bx0 = pcx; by0 = cy; bx1 = cx; by1 = cy;
            }
            if (e.lane == nrect) {
                rx0 = imin(ax0, ax1); rx1 = imax(ax0, ax1); ry0 = imin(ay0, ay1); ry1 = imax(ay0, ay1);
            }
            if (e.lane == nrect + 1) {
                rx0 = imin(bx0, bx1); rx1 = imax(bx0, bx1); ry0 = imin(by0, by1); ry1 = imax(by0, by1);
            }
            nrect += 2;
        }
        pcx = cx;
        pcy = cy;
    }
    for (int it = 0; it < 3; it++) {  // uniform trip count: every lane joins every shuffle
        const int y = e.lane + 32 * it;
        uint32_t w0 = 0, w1 = 0, w2 = 0;
        for (int j = 0; j < nrect; j++) {
            const int a0 = __shfl_sync(FULL, rx0, j), a1 = __shfl_sync(FULL, rx1, j);
            const int b0 = __shfl_sync(FULL, ry0, j), b1 = __shfl_sync(FULL, ry1, j);
            if (y < b0 || y > b1) continue;
            // bits a0..a1 inclusive across the three words (a1 <= 78)
            const uint64_t lo_mask = (a1 >= 63 ? ~0ull : ((1ull << (a1 + 1)) - 1ull)) & ~((1ull << imin(a0, 63)) - 1ull);
            if (a0 < 64) {
                w0 |= (uint32_t)lo_mask;
                w1 |= (uint32_t)(lo_mask >> 32);
            }
            if (a1 >= 64) {
                const int l0 = imax(a0, 64) - 64, l1 = a1 - 64;
                w2 |= (uint32_t)(((1ull << (l1 + 1)) - 1ull) & ~((1ull << l0) - 1ull));
            }
        }
        if (y < H) {
            s.floor[y * 3] = w0;
            s.floor[y * 3 + 1] = w1;
            s.floor[y * 3 + 2] = w2;
        }
    }
    __syncwarp();
}

// Floor count and the k-th floor cell in row-major order. Lane l owns words
// [7l, 7l+7) of the plane, so word order is cell order.
__device__ __forceinline__ int floor_count(const Env &e) {
    int c = 0;
#pragma unroll
    for (int i = 0; i < 7; i++) {
        const int w = e.lane * 7 + i;
        if (w < PL) c += __popc(e.sm->floor[w]);
    }
    return __reduce_add_sync(FULL, c);
}
__device__ int kth_floor(const Env &e, int k) {
    uint32_t words[7];
    int c = 0;
#pragma unroll
    for (int i = 0; i < 7; i++) {
        const int w = e.lane * 7 + i;
        words[i] = w < PL ? e.sm->floor[w] : 0u;
        c += __popc(words[i]);
    }
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(FULL, incl, o);
        if (e.lane >= o) incl += t;
    }
    const int excl = incl - c;
    const bool mine = k >= excl && k < incl;
    int cell = -1;
    if (mine) {
        int r = k - excl;
#pragma unroll
        for (int i = 0; i < 7; i++) {
            const int pc = __popc(words[i]);
            if (cell < 0 && r < pc) {
                uint32_t v = words[i];
                for (int t = 0; t < r; t++) v &= v - 1u;
                const int bit = __ffs(v) - 1;
                const int w = e.lane * 7 + i;
                cell = (w / 3) * W + (w % 3) * 32 + bit;
            }
            if (cell < 0) r -= pc;
        }
    }
    const unsigned who = __ballot_sync(FULL, mine);
    return who ? __shfl_sync(FULL, cell, __ffs(who) - 1) : -1;
}

__device__ __forceinline__ int occupant(const Env &e, int p) { return d1::occupant(e.m_pos, e.m_hp, p); }

__device__ void reset(Env &e, const D1SpecConfig &c, const RayArgs &ra) {
    gen_map(e);
    const int nf = floor_count(e);
    e.stairs = kth_floor(e, rng_r(e.rng, nf));
    int tries = 0;
    do {
        e.player = kth_floor(e, rng_r(e.rng, nf));
    } while (e.player == e.stairs && ++tries < 4096);
    e.m_pos = 0;
    e.m_energy = 0;
    e.m_hp = 0;
    e.m_kind = 0;
    e.m_awake = 0;
    e.nmon = 0;
    const int target = c.min_monsters + rng_r(e.rng, c.max_monsters - c.min_monsters + 1);
    for (int i = 0; i < target; i++) {
        const int kind = rng_r(e.rng, 4), hp = c.min_mhp + rng_r(e.rng, c.max_mhp - c.min_mhp + 1);
        int p;
        bool bad;
        tries = 0;
        do {
            p = kth_floor(e, rng_r(e.rng, nf));
            bad = p == e.player || p == e.stairs || occupant(e, p) >= 0;
        } while (bad && ++tries < 4096);
        if (bad) break;
        const int energy = 70 + rng_r(e.rng, 10);
        if (e.lane == i) {
            e.m_pos = p;
            e.m_hp = hp;
            e.m_kind = kind;
            e.m_energy = energy;
            e.m_awake = 0;
        }
        e.nmon = i + 1;
    }
    if (c.ogre) {
        for (int t = 0; t < 64; t++) {
            const int p = kth_floor(e, rng_r(e.rng, nf));
            if (cheb(p, e.player) >= 12 && p != e.stairs && occupant(e, p) < 0) {
                const int i = e.nmon++;
                const int energy = 70 + rng_r(e.rng, 10);
                if (e.lane == i) {
                    e.m_pos = p;
                    e.m_hp = c.ogre_hp;
                    e.m_kind = 4;
                    e.m_energy = energy;
                    e.m_awake = 0;
                }
                break;
            }
        }
    }
    e.hp = c.hp;
    e.regen = 0;
    e.blocks = 0;
    e.ticks = 0;
    e.killed = 0;
    e.floor_seen = 0;
    for (int r = e.lane; r < PL; r += 32) e.sm->viewed[r] = 0;
    __syncwarp();
    e.floor_dirty = true;
    e.dirty_lo = 0;
    e.dirty_hi = H - 1;
    compute_los(e, ra);
    reveal(e);
}

// ------------------------------------------------------------------ pursuit field
// Layered BFS from the player over floor. Only monsters that will move this
// turn (awake, energy >= 80, not adjacent) read the field, and they act at most
// `1 + extra_layers` times, each move raising their distance by at most one; the
// search therefore stops `extra_layers` layers past the farthest of them, where
// every cell a move compares against has its exact distance and every farther
// cell reads as unreached -- which all comparisons of sim.h:207-253 treat like
// any value larger than the mover's own. Layer k only touches rows within k of
// the player. Distances are stored mod 256 and recovered relative to the
// mover's exact distance (every compared cell lies within 24 steps of it).
// Sets m_dist (65535 = unreached) on each mover lane.
__device__ void pursuit_bfs(Env &e, int extra_layers) {
    Smem &s = *e.sm;
    const bool need = e.lane < e.nmon && e.m_hp > 0 && e.m_awake && e.m_energy >= 80 && cheb(e.m_pos, e.player) > 1;
    e.m_dist = 65535;
    if (!__any_sync(FULL, need)) return;
    for (int r = e.lane; r < PL; r += 32) {
        s.seen[r] = 0;
        s.cur[r] = 0;
    }
    __syncwarp();
    if (e.lane == 0) {
        const int r = (e.player / W) * 3 + (e.player % W) / 32;
        const uint32_t bit = 1u << ((e.player % W) % 32);
        s.seen[r] = bit;
        s.cur[r] = bit;
        e.dist[e.player] = 0;
    }
    __syncwarp();
    const int py = e.player / W;
    int stop_after = 0x7fffffff;
    for (int k = 1;; k++) {
        const int ylo = imax(0, py - k), yhi = imin(H - 1, py + k);
        uint32_t nw[3][3];
        bool any = false;
#pragma unroll
        for (int i = 0; i < 3; i++) {
            const int y = ylo + e.lane + 32 * i;
            nw[i][0] = nw[i][1] = nw[i][2] = 0;
            if (y <= yhi) {
                const uint32_t *c0 = s.cur + y * 3;
                uint32_t a0 = c0[0], a1 = c0[1], a2 = c0[2];
                if (y > 0) { a0 |= c0[-3]; a1 |= c0[-2]; a2 |= c0[-1]; }
                if (y < H - 1) { a0 |= c0[3]; a1 |= c0[4]; a2 |= c0[5]; }
                const uint32_t d0 = a0 | (a0 << 1) | (a0 >> 1) | (a1 << 31);
                const uint32_t d1 = a1 | (a1 << 1) | (a0 >> 31) | (a1 >> 1) | (a2 << 31);
                const uint32_t d2 = a2 | (a2 << 1) | (a1 >> 31) | (a2 >> 1);
                const int r = y * 3;
                nw[i][0] = d0 & s.floor[r] & ~s.seen[r];
                nw[i][1] = d1 & s.floor[r + 1] & ~s.seen[r + 1];
                nw[i][2] = d2 & s.floor[r + 2] & ~s.seen[r + 2];
                any |= (nw[i][0] | nw[i][1] | nw[i][2]) != 0;
            }
        }
        __syncwarp();
        // Rolled (instruction fetch bound): the word is picked by predication so
        // nw stays in registers.
#pragma unroll 1
        for (int ij = 0; ij < 9; ij++) {
            const int i = ij / 3, j = ij - 3 * i;
            const int y = ylo + e.lane + 32 * i;
            if (y <= yhi) {
                {
                    const int r = y * 3 + j;
                    uint32_t w = 0;
#pragma unroll
                    for (int ii = 0; ii < 3; ii++)
#pragma unroll
                        for (int jj = 0; jj < 3; jj++) w = (ii == i && jj == j) ? nw[ii][jj] : w;
                    s.seen[r] |= w;
                    s.cur[r] = w;
                    while (w) {
                        const int b = __ffs(w) - 1;
                        e.dist[y * W + j * 32 + b] = (uint8_t)k;
                        w &= w - 1;
                    }
                }
            }
        }
        __syncwarp();
        if (need && e.m_dist == 65535 && bitp(s.seen, e.m_pos)) e.m_dist = k;
        if (!__any_sync(FULL, any)) break;
        if (k >= stop_after) break;
        if (stop_after == 0x7fffffff && !__any_sync(FULL, need && e.m_dist == 65535)) {
            const int dmax = __reduce_max_sync(FULL, need ? e.m_dist : 0);
            stop_after = dmax + extra_layers;
            if (k >= stop_after) break;
        }
    }
}
// Distance of a reached cell q, given the exact distance D of a cell within
// 127 steps of it; 65535 when q was not reached.
__device__ __forceinline__ int dist_rel(const Env &e, int q, int D) {
    if (!bitp(e.sm->seen, q)) return 65535;
    return D + (int)(int8_t)(uint8_t)(e.dist[q] - (uint8_t)D);
}

// ------------------------------------------------------------------ monster turn
// sim.h:207-253 on the generated map: rotated compass walk with reservoir ties,
// then the bounded 24-node repair search. Returns the target cell and its exact
// distance.
__device__ int choose_move(Env &e, int p, int D, int &dq_out) {
    const int lane = e.lane;
    const int rotation = rng_r(e.rng, 4);
    if (D == 65535) return -1;  // unreachable component: every comparison fails
    const int d = lane & 7;
    const int q = neighbor(p, d);
    const bool okq = q >= 0 && floor_at(e, q) && q != e.player && !bitp(e.sm->occ, q);
    const int dq = okq ? dist_rel(e, q, D) : 0;
    // the rotated tie walk of sim.h:213-222 (walk_pick): a free neighbour's
    // distance is D - 1, D or D + 1, so the candidates are those at D - 1
    const unsigned cand = __ballot_sync(FULL, lane < 8 && okq && dq < D);
    if (cand) {
        const int dir = walk_pick(e.rng, cand, rotation);
        dq_out = __shfl_sync(FULL, dq, dir);
        return __shfl_sync(FULL, q, dir);
    }
    // Repair search (sim.h:225-252): FIFO over free floor from p, at most 24
    // nodes on the list, returning the first step of the first cell met (list
    // order, then compass order) that is closer to the player than p. A head's
    // 8 neighbours are tested at once: the first closer one in compass order is
    // the one the serial walk would meet first, and the others join the list in
    // compass order while there is room. The list membership plane reuses the
    // search frontier plane and the list the compact-row staging (both idle
    // during the monster phase).
    uint32_t *inl = e.sm->cur;
    int16_t *lc = reinterpret_cast<int16_t *>(e.sm->crow), *lf = lc + 24;
    for (int r = lane; r < PL; r += 32) inl[r] = 0u;
    __syncwarp();
    if (lane == 0) {
        lc[0] = (int16_t)p;
        lf[0] = -1;
        inl[(p / W) * 3 + (p % W) / 32] |= 1u << ((p % W) & 31);
    }
    __syncwarp();
    int len = 1;
    for (int head = 0; head < len; head++) {
        const int ch = lc[head], fh = lf[head];
        const int qn = neighbor(ch, d);
        const bool okn = lane < 8 && qn >= 0 && floor_at(e, qn) && qn != e.player && !bitp(e.sm->occ, qn) &&
                         !bitp(inl, qn);
        const int dqn = okn ? dist_rel(e, qn, D) : 65535;
        const unsigned closer = __ballot_sync(FULL, okn && dqn < D);
        if (closer) {
            const int qz = __shfl_sync(FULL, qn, __ffs(closer) - 1);
            const int step = head == 0 ? qz : fh;
            dq_out = dist_rel(e, step, D);
            return step;
        }
        const unsigned cand = __ballot_sync(FULL, okn);
        const int rank = __popc(cand & ((1u << lane) - 1u));
        __syncwarp();
        if (okn && len + rank < 24) {
            lc[len + rank] = (int16_t)qn;
            lf[len + rank] = (int16_t)(head == 0 ? qn : fh);
            atomicOr(&inl[(qn / W) * 3 + (qn % W) / 32], 1u << ((qn % W) & 31));
        }
        len = imin(24, len + __popc(cand));
        __syncwarp();
    }
    return -1;
}

__device__ void act(Env &e, const D1SpecConfig &c, int id) {
    if (e.lane == id) e.m_energy -= 10;
    const int mp = __shfl_sync(FULL, e.m_pos, id);
    if (cheb(mp, e.player) == 1) {
        const int kind = __shfl_sync(FULL, e.m_kind, id);
        const D1Kind k = kind_of(c, kind);
        D1Config pc;
        pc.ev100 = c.ev100;
        pc.sh100 = c.sh100;
        pc.ac100 = c.ac100;
        pc.shield_limit = c.shield_limit;
        pc.gdr[0] = c.gdr[0];
        pc.gdr[1] = c.gdr[1];
        incoming_attack(e.rng, pc, k.damage, k.tohit, k.bypass, kind == 4 ? c.ogre_min_damage : 1, e.hp, e.blocks);
        return;
    }
    const int D = __shfl_sync(FULL, e.m_dist, id);
    int dq = 65535;
    const int q = choose_move(e, mp, D, dq);
    if (q >= 0 && e.lane == id) {
        uint32_t *occ = e.sm->occ;
        occ[(mp / W) * 3 + (mp % W) / 32] &= ~(1u << ((mp % W) & 31));
        occ[(q / W) * 3 + (q % W) / 32] |= 1u << ((q % W) & 31);
        e.m_pos = q;
        e.m_dist = dq;
    }
    __syncwarp();
}

__device__ __forceinline__ bool visible_awake(const Env &e) {
    return __ballot_sync(FULL, e.lane < e.nmon && e.m_hp > 0 && e.m_awake && visible(e, e.m_pos)) != 0;
}
// semantic-actions-v1 learn.cu:423-428: weakest visible adjacent monster, first
// compass direction on ties; -1 if none.
__device__ int adjacent_attack(const Env &e) {
    unsigned key = 0xffffffffu;
    if (e.lane < e.nmon && e.m_hp > 0 && cheb(e.m_pos, e.player) == 1 && visible(e, e.m_pos)) {
        const int dx = e.m_pos % W - e.player % W, dy = e.m_pos / W - e.player / W;
        // direction index of (dx, dy) in compass order N,E,S,W,NE,SE,SW,NW
        const int dir = dy == -1 ? (dx == 0 ? 0 : dx == 1 ? 4 : 7) : dy == 0 ? (dx == 1 ? 1 : 3)
                                                                              : (dx == 0 ? 2 : dx == 1 ? 5 : 6);
        key = ((unsigned)e.m_hp << 3) | (unsigned)dir;
    }
    key = __reduce_min_sync(FULL, key);
    return key == 0xffffffffu ? -1 : (int)(key & 7u);
}

// saw_awake (tracked only when `watch`, i.e. inside a rest macro): an awake
// monster was in view at some point of the turn -- after the player's move, after
// any monster's action, or at its end; the rest macro's interrupt signal
// (semantic-actions-v1 learn.cu:680-681,708,729,819).
struct Prim {
    float reward;
    bool done, descended, death, timeout, saw_awake;
};

// One physical turn (learn.cu:505-598 with the sleep/explore/stairs variants).
__device__ Prim primitive(Env &e, const D1SpecConfig &c, const RayArgs &ra, int extra_layers, int d, bool watch) {
    Prim r;
    r.saw_awake = false;
    int reward_milli = -1;
    e.blocks = 0;
    e.regen += c.regen;
    while (e.regen >= 100) {
        e.hp = imin(c.hp, e.hp + 1);
        e.regen -= 100;
    }
    if (d >= 0 && d < 8) {
        const int p = neighbor(e.player, d);
        if (floor_at(e, p)) {
            const int id = occupant(e, p);
            if (id >= 0) {
                if (rng_r(e.rng, 5) != 0) {
                    const int dmg = 1 + rng_r(e.rng, 4);
                    if (e.lane == id) e.m_hp = (int16_t)(e.m_hp - dmg);
                    if (__shfl_sync(FULL, e.m_hp, id) <= 0) {
                        if (e.lane == id) {
                            e.m_hp = 0;
                            e.m_energy = -30000;
                        }
                        e.killed++;
                        reward_milli += c.kill_milli;
                    }
                }
            } else {
                e.player = p;
                compute_los(e, ra);
            }
        }
    }
    const bool descended = d == PRIM_DESCEND && e.player == e.stairs && e.hp > 0;
    reward_milli += c.explore_milli * reveal(e);
    // (The interrupt rule's first check, an awake monster in view right after
    // the player's move, is always false inside a rest: the player does not
    // move, and the previous turn ended -- or the rest began -- with none.)
    if (!descended) {
        const bool alive = e.lane < e.nmon && e.m_hp > 0;
        if (alive && !e.m_awake && cheb(e.m_pos, e.player) <= 6 && visible(e, e.m_pos)) {
            e.m_awake = 1;
            e.m_energy = 70;
        }
        if (alive && !e.m_awake) e.m_energy = -30000;
        if (alive) e.m_energy = (int16_t)(e.m_energy + kind_of(c, e.m_kind).speed);
        if (__any_sync(FULL, alive && e.m_energy >= 80)) {
            for (int r = e.lane; r < PL; r += 32) e.sm->occ[r] = 0;
            __syncwarp();
            if (alive) atomicOr(&e.sm->occ[(e.m_pos / W) * 3 + (e.m_pos % W) / 32], 1u << ((e.m_pos % W) & 31));
            __syncwarp();
        }
        pursuit_bfs(e, extra_layers);
        while (e.hp > 0) {
            const int id = scan_ready(e.m_energy, e.lane, e.nmon);
            if (id < 0) break;
            act(e, c, id);
            if (watch && __any_sync(FULL, e.lane == id && e.m_awake && visible(e, e.m_pos))) r.saw_awake = true;
        }
    }
    e.ticks++;
    const bool death = e.hp <= 0, timeout = !descended && !death && e.ticks >= c.limit;
    if (descended) reward_milli += c.descend_milli;
    if (death) reward_milli -= c.death_milli;
    r.reward = 0.001f * (float)reward_milli;
    r.done = descended || death || timeout;
    r.descended = descended;
    r.death = death;
    r.timeout = timeout;
    if (watch && !r.saw_awake) r.saw_awake = visible_awake(e);
    return r;
}

// Semantic decision: 0-7 move/attack, 8 wait, 9 rest (repeat waits until full
// HP, an awake monster in view during a turn, or the end; semantic-actions-v1
// learn.cu:803-826), 10 attack the weakest visible
// adjacent monster, 11 descend. Illegal actions cost one wait turn.
// Returns out[lane] for lane < OUT.
__device__ float decision(Env &e, const D1SpecConfig &c, const RayArgs &ra, int extra_layers, int a) {
    float total = 0.f;
    int elapsed = 0;
    bool invalid = false;
    Prim r;
    for (;;) {
        int d = PRIM_WAIT;
        if (a >= 0 && a < 8) d = a;
        else if (a == 8) d = PRIM_WAIT;
        else if (a == 9) invalid = e.hp >= c.hp || visible_awake(e) || c.regen <= 0;
        else if (a == 10) {
            d = adjacent_attack(e);
            if (d < 0) {
                d = PRIM_WAIT;
                invalid = true;
            }
        } else if (a == 11) {
            if (e.player == e.stairs) d = PRIM_DESCEND;
            else invalid = true;
        } else
            invalid = true;
        r = primitive(e, c, ra, extra_layers, d, a == 9);
        elapsed++;
        total += r.reward;
        if (r.done || invalid || a != 9) break;
        if (r.saw_awake || e.hp >= c.hp) break;
        // A rest turn with no living monster awake leaves a fixed point behind:
        // the player stands still (nothing new in view), every sleeping monster
        // keeps failing the same wake test, and none holds the energy to act.
        // Each further turn therefore changes only regeneration, HP and the
        // clock, and pays one wait (-1 milli); those turns run here as scalar
        // arithmetic, bit-identical to running them as primitives.
        if (!__any_sync(FULL, e.lane < e.nmon && e.m_hp > 0 && e.m_awake)) {
            for (;;) {
                e.blocks = 0;
                e.regen += c.regen;
                while (e.regen >= 100) {
                    e.hp = imin(c.hp, e.hp + 1);
                    e.regen -= 100;
                }
                e.ticks++;
                r.timeout = e.ticks >= c.limit;
                r.done = r.timeout;
                r.reward = 0.001f * (float)(-1);
                elapsed++;
                total += r.reward;
                if (r.done || e.hp >= c.hp) break;
            }
            break;
        }
    }
    float o = 0.f;
    switch (e.lane) {
        case 0: o = total; break;
        case 1: o = r.done; break;
        case 2: o = r.descended; break;
        case 3: o = (float)e.killed; break;
        case 4: o = (float)imax(0, e.hp); break;
        case 5: o = (float)e.ticks; break;
        case 6: o = r.death; break;
        case 7: o = r.timeout; break;
        case 8: o = (float)elapsed; break;
        case 9: o = invalid; break;
    }
    if (r.done) {
        e.episode++;
        reset(e, c, ra);
    }
    return o;
}

// ------------------------------------------------------------------ observation
// Channels per window cell: 0 unknown/off-map, 1 remembered wall, 2 remembered
// floor out of view, 3 visible floor, 4 stairs, 5 visible sleeping monster,
// 6 visible awake monster, 7 visible ogre. Each cell is one 16-byte store of
// eight bf16 values; the 32 scalars follow at element 1800.
__device__ void observe(Env &e, const D1SpecConfig &c, __nv_bfloat16 *obs, uint8_t *cobs, uint16_t *legal) {
    Smem &s = *e.sm;
    const int lane = e.lane, px = e.player % W, py = e.player / W;
    for (int j = lane; j < (CELLS + 7) / 4; j += 32) reinterpret_cast<uint32_t *>(s.occ_ch)[j] = 0xffffffffu;
    if (lane < 8) {
        const uint32_t one = 0x3f80u << (16 * (lane & 1));
        const int w = lane >> 1;
        s.onehot[lane] = make_uint4(w == 0 ? one : 0u, w == 1 ? one : 0u, w == 2 ? one : 0u, w == 3 ? one : 0u);
    }
    __syncwarp();
    const bool alive = lane < e.nmon && e.m_hp > 0;
    const bool mvis = alive && visible(e, e.m_pos);
    if (mvis) {
        const int dx = e.m_pos % W - px, dy = e.m_pos / W - py;
        s.occ_ch[(dy + 7) * 15 + dx + 7] = (uint8_t)(e.m_kind == 4 ? 7 : e.m_awake ? 6 : 5);
    }
    __syncwarp();
    if (lane < 15) {
        const int cy = py + lane - 7;
        uint32_t vm = 0, fm = 0;
        if (cy >= 0 && cy < H) {
            vm = row15(s.viewed + cy * 3, px - 7);
            fm = row15(s.floor + cy * 3, px - 7);
        }
        s.vmask[lane] = (uint16_t)vm;
        s.fmask[lane] = (uint16_t)fm;
    }
    __syncwarp();
    const int sdx = e.stairs % W - px, sdy = e.stairs / W - py;
    const int sj = (sdx >= -7 && sdx <= 7 && sdy >= -7 && sdy <= 7) ? (sdy + 7) * 15 + sdx + 7 : -1;
    uint4 *dst = reinterpret_cast<uint4 *>(obs);
    // Half-warps take window rows 2k and 2k + 1, a lane per column (lanes 15
    // and 31 idle), so each store of the warp covers 30 consecutive cells.
    // Rolled: this kernel is bound by instruction fetch (ncu: "no instruction"
    // is the top stall), so compact code beats unrolled code here.
    const int wx = lane & 15;
#pragma unroll 1
    for (int k = 0; k < 8; k++) {
        const int wy = 2 * k + (lane >> 4);
        if ((obs || cobs) && wx < 15 && wy < 15) {
            const int jc = wy * 15 + wx;
            const uint32_t vm = s.vmask[wy], fm = s.fmask[wy], vr = s.vis[wy];
            const int m = s.occ_ch[jc];
            const int floor_ch = m != 0xff ? m : (jc == sj ? 4 : (((vr >> wx) & 1u) ? 3 : 2));
            const int ch = ((vm >> wx) & 1u) ? (((fm >> wx) & 1u) ? floor_ch : 1) : 0;
            if (obs) dst[jc] = s.onehot[ch];
            if (cobs) reinterpret_cast<uint8_t *>(s.crow)[jc] = (uint8_t)ch;
        }
    }
    if (cobs && lane < COBS_SCALARS - CELLS) reinterpret_cast<uint8_t *>(s.crow)[CELLS + lane] = 0;
    // scalars
    const int nvis = __popc(__ballot_sync(FULL, mvis));
    const int nvis_awake = __popc(__ballot_sync(FULL, mvis && e.m_awake));
    const unsigned nkey = __reduce_min_sync(FULL, mvis ? ((unsigned)cheb(e.m_pos, e.player) << 5) | lane : 0xffffffffu);
    const int near = nkey == 0xffffffffu ? -1 : (int)(nkey & 31u);
    const bool adj = mvis && cheb(e.m_pos, e.player) == 1;
    const int nadj = __popc(__ballot_sync(FULL, adj));
    const unsigned wk = __reduce_min_sync(FULL, adj ? (unsigned)e.m_hp : 0xffffffffu);
    const int weakest = wk == 0xffffffffu ? 0 : (int)wk;
    const unsigned og = __ballot_sync(FULL, mvis && e.m_kind == 4);
    const int ogre = og ? __ffs(og) - 1 : -1;
    // visible_awake(e) is any(mvis && awake) and adjacent_attack(e) >= 0 is any(adj):
    // both reuse the ballots above
    const bool rest_ok = e.hp < c.hp && c.regen > 0 && nvis_awake == 0;
    const bool attack_ok = nadj > 0;
    const bool known = bitp(s.viewed, e.stairs);
    const int np = __shfl_sync(FULL, e.m_pos, near < 0 ? 0 : near), nh = __shfl_sync(FULL, e.m_hp, near < 0 ? 0 : near);
    const int na = __shfl_sync(FULL, e.m_awake, near < 0 ? 0 : near), nk = __shfl_sync(FULL, e.m_kind, near < 0 ? 0 : near);
    const int op = __shfl_sync(FULL, e.m_pos, ogre < 0 ? 0 : ogre), oh = __shfl_sync(FULL, e.m_hp, ogre < 0 ? 0 : ogre);
    const int oa = __shfl_sync(FULL, e.m_awake, ogre < 0 ? 0 : ogre);
    // Feature `lane` = num / den with the same operands as the oracle's
    // expressions (every value is an int or a 0/1 flag over a float constant),
    // so one correctly rounded division per lane reproduces it. Every lane holds
    // the same 32 numerators: lane 0 stages them in shared memory (the monster
    // occupancy plane, which the next monster phase re-initialises) and each
    // lane reads its own, instead of a per-lane array in local memory.
    const int npx = near >= 0 ? np % W - px : 0, npy = near >= 0 ? np / W - py : 0;
    const int opx = ogre >= 0 ? op % W - px : 0, opy = ogre >= 0 ? op / W - py : 0;
    float4 *stage = reinterpret_cast<float4 *>(s.occ);
    if (lane == 0) {
        stage[0] = make_float4((float)e.hp, (float)e.regen, (float)e.ticks, (float)e.killed);
        stage[1] = make_float4((float)px, (float)py, (float)nvis, (float)nvis_awake);
        stage[2] = make_float4(near >= 0 ? 1.f : 0.f, (float)npx, (float)npy, near >= 0 ? (float)nh : 0.f);
        stage[3] = make_float4(near >= 0 ? (float)na : 0.f, near >= 0 ? (float)nk : 0.f, known ? 1.f : 0.f,
                               known ? (float)(e.stairs % W - px) : 0.f);
        stage[4] = make_float4(known ? (float)(e.stairs / W - py) : 0.f, e.player == e.stairs ? 1.f : 0.f,
                               (float)nadj, (float)weakest);
        stage[5] = make_float4(rest_ok ? 1.f : 0.f, attack_ok ? 1.f : 0.f, (float)e.floor_seen, (float)e.blocks);
        stage[6] = make_float4(1.f, ogre >= 0 ? 1.f : 0.f, (float)opx, (float)opy);
        stage[7] = make_float4(ogre >= 0 ? (float)oa : 0.f, ogre >= 0 ? (float)oh : 0.f, 0.f, 0.f);
    }
    __syncwarp();
    const float num = reinterpret_cast<const float *>(s.occ)[lane];
    const float den = lane == 0 ? (float)c.hp : lane == 2 ? (float)c.limit : __ldg(SCALAR_DEN + lane);
    const float f = num / den;
    if (obs) obs[1800 + lane] = __float2bfloat16_rn(f);
    if (cobs) {
        reinterpret_cast<__nv_bfloat16 *>(reinterpret_cast<uint8_t *>(s.crow) + COBS_SCALARS)[lane] =
            __float2bfloat16_rn(f);
        __syncwarp();
        if (lane < COBS / 16) reinterpret_cast<uint4 *>(cobs)[lane] = s.crow[lane];
    }
    if (lane < 8) {
        const bool ok = floor_at(e, neighbor(e.player, lane));
        const unsigned b = __ballot_sync(0xffu, ok);
        if (lane == 0) {
            uint32_t bits = (b & 0xffu) | (1u << 8);
            if (rest_ok) bits |= 1u << 9;
            if (attack_ok) bits |= 1u << 10;
            if (e.player == e.stairs) bits |= 1u << 11;
            *legal = (uint16_t)bits;
        }
    }
}

// ------------------------------------------------------------------ row I/O
__device__ void load(Env &e, const uint8_t *row) {
    const uint64_t *q = reinterpret_cast<const uint64_t *>(row);
    const uint32_t *u = reinterpret_cast<const uint32_t *>(row);
    const int *i32 = reinterpret_cast<const int *>(row);
    e.rng.n = q[0];
    e.env = u[2];
    e.rng.k0 = u[2];
    e.rng.k1 = u[3];
    e.rng.c2 = u[4];
    e.episode = u[5];
    e.hp = i32[6]; e.regen = i32[7]; e.blocks = i32[8]; e.player = i32[9];
    e.ticks = i32[10]; e.killed = i32[11]; e.stairs = i32[12]; e.nmon = i32[13];
    e.floor_seen = i32[14];
    const int l = e.lane & 15;
    const int16_t *m = reinterpret_cast<const int16_t *>(row + OFF_MON);
    e.m_pos = m[l];
    e.m_energy = m[16 + l];
    e.m_hp = e.lane < MAXM ? m[32 + l] : 0;
    e.m_kind = row[OFF_MON + 96 + l];
    e.m_awake = row[OFF_MON + 112 + l];
    // All plane words are loaded into registers before any shared-memory store:
    // the compiler cannot prove the generic shared pointer does not alias the
    // row, so interleaving would serialise the DRAM round trips.
    const uint32_t *fp = reinterpret_cast<const uint32_t *>(row + OFF_FLOOR);
    const uint32_t *vp = reinterpret_cast<const uint32_t *>(row + OFF_VIEWED);
    uint32_t fw[7], vw[7];
#pragma unroll
    for (int i = 0; i < 7; i++) {
        const int r = e.lane + 32 * i;
        fw[i] = r < PL ? __ldg(fp + r) : 0u;
        vw[i] = r < PL ? __ldg(vp + r) : 0u;
    }
    const uint32_t vis16 = e.lane < 16 ? reinterpret_cast<const uint16_t *>(row + OFF_VIS)[e.lane] : 0u;
#pragma unroll
    for (int i = 0; i < 7; i++) {
        const int r = e.lane + 32 * i;
        if (r < PL) {
            e.sm->floor[r] = fw[i];
            e.sm->viewed[r] = vw[i];
        }
    }
    if (e.lane < 16) e.sm->vis[e.lane] = vis16;
    __syncwarp();
    e.rng.refill();
    e.dirty_lo = H;
    e.dirty_hi = -1;
    e.floor_dirty = false;
}
__device__ void store(const Env &e, uint8_t *row) {
    if (e.lane == 0) {
        uint64_t *q = reinterpret_cast<uint64_t *>(row);
        uint32_t *u = reinterpret_cast<uint32_t *>(row);
        int *i32 = reinterpret_cast<int *>(row);
        q[0] = e.rng.n;
        u[2] = e.env; u[3] = e.rng.k1; u[4] = e.rng.c2; u[5] = e.episode;
        i32[6] = e.hp; i32[7] = e.regen; i32[8] = e.blocks; i32[9] = e.player;
        i32[10] = e.ticks; i32[11] = e.killed; i32[12] = e.stairs; i32[13] = e.nmon;
        i32[14] = e.floor_seen;
    }
    if (e.lane < 16) {
        reinterpret_cast<uint16_t *>(row + OFF_VIS)[e.lane] = (uint16_t)e.sm->vis[e.lane];
        int16_t *m = reinterpret_cast<int16_t *>(row + OFF_MON);
        m[e.lane] = (int16_t)e.m_pos;
        m[16 + e.lane] = (int16_t)e.m_energy;
        m[32 + e.lane] = (int16_t)e.m_hp;
        row[OFF_MON + 96 + e.lane] = (uint8_t)e.m_kind;
        row[OFF_MON + 112 + e.lane] = (uint8_t)e.m_awake;
    }
    uint32_t *fp = reinterpret_cast<uint32_t *>(row + OFF_FLOOR);
    uint32_t *vp = reinterpret_cast<uint32_t *>(row + OFF_VIEWED);
    if (e.floor_dirty)
        for (int r = e.lane; r < PL; r += 32) fp[r] = e.sm->floor[r];
    if (e.dirty_lo <= e.dirty_hi)
        for (int r = e.dirty_lo * 3 + e.lane; r < (e.dirty_hi + 1) * 3; r += 32) vp[r] = e.sm->viewed[r];
}

__global__ void __launch_bounds__(WARPS * 32, MIN_BLOCKS)
    init_kernel(uint8_t *state, int n, D1SpecConfig c, RayArgs ra, uint64_t seed, int first_env,
                __nv_bfloat16 *obs, uint8_t *cobs, uint16_t *legal) {
    __shared__ Smem sms[WARPS];
    const int w = threadIdx.x >> 5, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    Env e;
    e.lane = threadIdx.x & 31;
    e.sm = &sms[w];
    e.dist = state + (size_t)env * ROW + OFF_DIST;
    e.env = (uint32_t)(first_env + env);
    e.episode = 0;
    e.rng.n = 0;
    e.rng.k0 = e.env;
    e.rng.k1 = (uint32_t)seed;
    e.rng.c2 = (uint32_t)(seed >> 32);
    e.rng.lane = e.lane;
    e.rng.refill();
    e.dirty_lo = H;
    e.dirty_hi = -1;
    reset(e, c, ra);
    observe(e, c, obs ? obs + (size_t)env * OBS : nullptr, cobs ? cobs + (size_t)env * COBS : nullptr, legal + env);
    uint8_t *row = state + (size_t)env * ROW;
    for (int i = e.lane; i < OFF_FLOOR / 4; i += 32) reinterpret_cast<uint32_t *>(row)[i] = 0;
    __syncwarp();
    store(e, row);
}

__global__ void __launch_bounds__(WARPS * 32, MIN_BLOCKS)
    step_kernel(uint8_t *state, int n, D1SpecConfig c, RayArgs ra, int extra_layers, const int64_t *actions,
                __nv_bfloat16 *obs, uint8_t *cobs, uint16_t *legal, float *out, int64_t out_env, int64_t out_col,
                const bool *active) {
    pdl_wait();  // before any global access: the actions come from the previous kernel
    __shared__ Smem sms[WARPS];
    const int w = threadIdx.x >> 5, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    if (active && !active[env]) return;
    Env e;
    e.lane = threadIdx.x & 31;
    e.rng.lane = e.lane;
    e.sm = &sms[w];
    uint8_t *row = state + (size_t)env * ROW;
    e.dist = row + OFF_DIST;
    load(e, row);
    const float o = decision(e, c, ra, extra_layers, (int)actions[env]);
    if (e.lane < OUT) out[env * out_env + e.lane * out_col] = o;
    observe(e, c, obs ? obs + (size_t)env * OBS : nullptr, cobs ? cobs + (size_t)env * COBS : nullptr, legal + env);
    store(e, row);
}

// Observation of rows as they are (rows built or edited by hand): no step.
__global__ void __launch_bounds__(WARPS * 32, MIN_BLOCKS)
    observe_kernel(uint8_t *state, int n, D1SpecConfig c, __nv_bfloat16 *obs, uint8_t *cobs, uint16_t *legal) {
    __shared__ Smem sms[WARPS];
    const int w = threadIdx.x >> 5, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    Env e;
    e.lane = threadIdx.x & 31;
    e.rng.lane = e.lane;
    e.sm = &sms[w];
    uint8_t *row = state + (size_t)env * ROW;
    e.dist = row + OFF_DIST;
    load(e, row);
    observe(e, c, obs ? obs + (size_t)env * OBS : nullptr, cobs ? cobs + (size_t)env * COBS : nullptr, legal + env);
}

// ------------------------------------------------------------------ conv-policy crop
// Egocentric 63 x 63 crop under D4 element g, one u16 code per pixel (rows of
// pitch 64, column 63 zero): bits 0-2 the observation's one-hot class, bit 3
// "on the map", bits 4-8 the hp of a visible monster there. Pixel (x, y) shows
// the map cell at offset d4(g, x - 31, y - 31) from the player, with
// d4 = rotation by g % 4 quarter turns ((dx, dy), (dy, -dx), (-dx, -dy), (-dy, dx))
// followed by an x mirror when g >= 4, the sampling rule of the reference's
// centered-map encoder (vision15-centered-map-v1/src/fast_maps.cu:7-9). One warp
// per env: the planes and the 15 x 15 monster window are staged in shared
// memory, then each lane codes two pixels of every crop row.
constexpr int CROP = 63, CROP_PITCH = 64, CROP_WARPS = 8;
struct CropSmem {
    uint32_t floor[PL], viewed[PL], vis[16];
    uint16_t occ[CELLS];  // code of the visible monster in the 15 x 15 window, 0 = none
};
__global__ void __launch_bounds__(CROP_WARPS * 32) crop_kernel(const uint8_t *state, int n, int g, uint16_t *out) {
    __shared__ CropSmem sms[CROP_WARPS];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, env = blockIdx.x * CROP_WARPS + w;
    if (env >= n) return;
    CropSmem &s = sms[w];
    const uint8_t *row = state + (size_t)env * ROW;
    const int *i32 = reinterpret_cast<const int *>(row);
    const int player = i32[9], stairs = i32[12], nmon = i32[13];
    const int px = player % W, py = player / W;
    const uint32_t *fp = reinterpret_cast<const uint32_t *>(row + OFF_FLOOR);
    const uint32_t *vp = reinterpret_cast<const uint32_t *>(row + OFF_VIEWED);
    for (int r = lane; r < PL; r += 32) {
        s.floor[r] = fp[r];
        s.viewed[r] = vp[r];
    }
    if (lane < 16) s.vis[lane] = reinterpret_cast<const uint16_t *>(row + OFF_VIS)[lane];
    for (int j = lane; j < CELLS; j += 32) s.occ[j] = 0;
    __syncwarp();
    if (lane < MAXM && lane < nmon) {
        const int16_t *m = reinterpret_cast<const int16_t *>(row + OFF_MON);
        const int pos = m[lane], hp = m[32 + lane];
        const int kind = row[OFF_MON + 96 + lane], awake = row[OFF_MON + 112 + lane];
        const int dx = pos % W - px, dy = pos / W - py;
        if (hp > 0 && dx >= -7 && dx <= 7 && dy >= -7 && dy <= 7 && ((s.vis[dy + 7] >> (dx + 7)) & 1u)) {
            const int cls = kind == 4 ? 7 : awake ? 6 : 5;
            s.occ[(dy + 7) * 15 + dx + 7] = (uint16_t)(cls | 8 | ((hp > 31 ? 31 : hp) << 4));
        }
    }
    __syncwarp();
    const int r = g & 3;
    const bool mirror = g >= 4;
    uint16_t *o = out + (size_t)env * (CROP * CROP_PITCH);
    for (int y = 0; y < CROP; y++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int x = lane + 32 * h;
            uint32_t code = 0;
            if (x < CROP) {
                const int dx = x - 31, dy = y - 31;
                int sx = r == 0 ? dx : r == 1 ? dy : r == 2 ? -dx : -dy;
                const int sy = r == 0 ? dy : r == 1 ? -dx : r == 2 ? -dy : dx;
                if (mirror) sx = -sx;
                const int cx = px + sx, cy = py + sy;
                if (cx >= 0 && cx < W && cy >= 0 && cy < H) {
                    const int word = cy * 3 + (cx >> 5), bit = cx & 31;
                    uint32_t cls = 0;
                    if ((s.viewed[word] >> bit) & 1u) {
                        if (!((s.floor[word] >> bit) & 1u)) {
                            cls = 1;
                        } else {
                            const bool win = sx >= -7 && sx <= 7 && sy >= -7 && sy <= 7;
                            const bool vis = win && ((s.vis[sy + 7] >> (sx + 7)) & 1u);
                            const uint32_t occ = vis ? s.occ[(sy + 7) * 15 + sx + 7] : 0u;
                            cls = occ ? occ : (cy * W + cx == stairs ? 4u : vis ? 3u : 2u);
                        }
                    }
                    code = cls | 8u;
                }
            }
            o[y * CROP_PITCH + x] = (uint16_t)code;
        }
    }
}

// ------------------------------------------------------------------ map compiler: LOS table
// The per-origin LOS masks of a map in the reference's corpus format
// (gpu-d1/scripts/compile_corpus.py:67-85: 17x17 window, bit (dy+8)*17 + dx+8,
// 10 x u32 per origin, rays from the native fan) for every one of the 5600
// cells, one warp per origin with the env step's own ray evaluation. Replaces
// the reference's per-map Python loop over origins x quadrants x rays.
constexpr int LOS_WARPS = 4;
__global__ void __launch_bounds__(LOS_WARPS * 32) los_table_kernel(const uint8_t *floor_u8, RayArgs ra, uint32_t *out) {
    __shared__ Smem sms[LOS_WARPS];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int origin = blockIdx.x * LOS_WARPS + w;
    if (blockIdx.x * LOS_WARPS + w >= N) return;  // warp-uniform
    Smem &s = sms[w];
    for (int r = lane; r < PL; r += 32) {
        const int y = r / 3, x0 = (r % 3) * 32;
        uint32_t bits = 0;
        for (int b = 0; b < 32 && x0 + b < W; b++) bits |= (floor_u8[y * W + x0 + b] ? 1u : 0u) << b;
        s.floor[r] = bits;
    }
    __syncwarp();
    Env e;
    e.lane = lane;
    e.sm = &s;
    e.dist = nullptr;  // no pursuit search here
    e.player = origin;
    compute_los(e, ra);
    // row dy = lane - 7 (15 bits, dx = -7..7) lands at bit (lane + 1) * 17 + 1
    const uint32_t row = lane < 15 ? s.vis[lane] : 0u;
    const int base = (lane + 1) * 17 + 1, w0 = base >> 5, sh = base & 31;
    const uint32_t c0 = row << sh, c1 = sh ? row >> (32 - sh) : 0u;
    uint32_t mine = 0;
#pragma unroll
    for (int i = 0; i < 10; i++) {
        const uint32_t v = __reduce_or_sync(FULL, (w0 == i ? c0 : 0u) | (w0 + 1 == i ? c1 : 0u));
        if (lane == i) mine = v;
    }
    if (lane < 10) out[(size_t)origin * 10 + lane] = mine;
}

__global__ void compact_kernel(const uint8_t *state, int n, int64_t *rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * COMPACT) return;
    const int env = i / COMPACT, f = i % COMPACT;
    const uint8_t *row = state + (size_t)env * ROW;
    int64_t v;
    if (f == 0) v = (int64_t) reinterpret_cast<const uint64_t *>(row)[0];
    else if (f == 1) v = reinterpret_cast<const uint32_t *>(row)[2];
    else if (f == 2) v = reinterpret_cast<const uint32_t *>(row)[5];
    else if (f < 12) v = reinterpret_cast<const int *>(row)[6 + (f - 3)];
    else {
        const int k = (f - 12) % MAXM, g = (f - 12) / MAXM;
        const int16_t *m = reinterpret_cast<const int16_t *>(row + OFF_MON);
        if (g == 0) v = m[k];
        else if (g == 1) v = m[16 + k];
        else if (g == 2) v = m[32 + k];
        else v = row[OFF_MON + 96 + k] * 2 + row[OFF_MON + 112 + k];
    }
    rows[i] = v;
}

__global__ void planes_kernel(const uint8_t *state, int n, uint32_t *floor, uint32_t *viewed) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * PL) return;
    const int env = i / PL, r = i % PL;
    const uint8_t *row = state + (size_t)env * ROW;
    floor[i] = reinterpret_cast<const uint32_t *>(row + OFF_FLOOR)[r];
    viewed[i] = reinterpret_cast<const uint32_t *>(row + OFF_VIEWED)[r];
}

}  // namespace spec
}  // namespace d1

using namespace d1;

static spec::RayArgs g_rays = {nullptr, 0};

extern "C" {

int d1_spec_state_bytes(void) { return spec::ROW; }
int d1_spec_obs_size(void) { return spec::OBS; }
int d1_spec_action_size(void) { return spec::ACTIONS; }
int d1_spec_out_size(void) { return spec::OUT; }
int d1_spec_config_bytes(void) { return (int)sizeof(D1SpecConfig); }

int d1_spec_set_rays(const void *rays, int n) {
    if (n <= 0 || n > spec::MAX_RAYS || !rays || (reinterpret_cast<uintptr_t>(rays) & 15)) return D1_ERR_BAD_ARGUMENT;
    g_rays.ray = static_cast<const uint4 *>(rays);
    g_rays.n = n;
    return 0;
}

// A monster with speed S acts at most floor((S - 1) / 10) + 1 times per turn and
// each move can raise its distance by one, so the pursuit field must be exact one
// layer past the farthest awake monster for every action after its first.
static int spec_extra_layers(const D1SpecConfig &c) {
    int smax = 1;
    for (int k = 0; k < 5; k++) smax = c.kinds[k].speed > smax ? c.kinds[k].speed : smax;
    const int acts = (smax - 1) / 10 + 1;
    return acts > 1 ? acts - 1 : 1;
}

static int spec_check(int n, const D1SpecConfig *c) {
    if (n < 0 || !c || g_rays.n == 0) return D1_ERR_BAD_ARGUMENT;
    if (c->min_monsters < 0 || c->max_monsters > 10 || c->min_monsters > c->max_monsters || c->min_mhp < 1 ||
        c->max_mhp < c->min_mhp || c->limit <= 0 || c->hp <= 0 || c->ogre_min_damage < 1 ||
        c->kinds[4].damage < c->ogre_min_damage || c->ac100 < 0 || c->regen < 0)
        return D1_ERR_BAD_ARGUMENT;
    for (int k = 0; k < 5; k++)
        if (c->kinds[k].speed < 0 || c->kinds[k].speed > 60 || c->kinds[k].damage < 1 || c->kinds[k].tohit < 0 ||
            c->kinds[k].bypass < 0)
        return D1_ERR_BAD_ARGUMENT;
    return 0;
}

int d1_spec_init_ex(void *state, int n, const D1SpecConfig *c, uint64_t seed, int first_env, void *obs_bf16,
                    void *cobs, uint16_t *legal, void *stream) {
    if (int err = spec_check(n, c)) return err;
    if (n == 0) return 0;
    spec::init_kernel<<<(n + spec::WARPS - 1) / spec::WARPS, spec::WARPS * 32, 0, (cudaStream_t)stream>>>(
        (uint8_t *)state, n, *c, g_rays, seed, first_env, (__nv_bfloat16 *)obs_bf16, (uint8_t *)cobs, legal);
    return (int)cudaGetLastError();
}

int d1_spec_init(void *state, int n, const D1SpecConfig *c, uint64_t seed, int first_env, void *obs_bf16,
                 uint16_t *legal, void *stream) {
    return d1_spec_init_ex(state, n, c, seed, first_env, obs_bf16, nullptr, legal, stream);
}

int d1_los_table(const uint8_t *floor, uint32_t *masks, void *stream) {
    if (!floor || !masks) return D1_ERR_BAD_ARGUMENT;
    if (!g_rays.ray) return D1_ERR_BAD_ARGUMENT;
    spec::los_table_kernel<<<(d1::N + spec::LOS_WARPS - 1) / spec::LOS_WARPS, spec::LOS_WARPS * 32, 0,
                             (cudaStream_t)stream>>>(floor, g_rays, masks);
    return (int)cudaGetLastError();
}

int d1_spec_crop(const void *state, int n, int g, uint16_t *crop, void *stream) {
    if (n < 0 || g < 0 || g > 7 || !state || !crop) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    spec::crop_kernel<<<(n + spec::CROP_WARPS - 1) / spec::CROP_WARPS, spec::CROP_WARPS * 32, 0,
                        (cudaStream_t)stream>>>((const uint8_t *)state, n, g, crop);
    return (int)cudaGetLastError();
}

int d1_spec_step_strided(void *state, int n, const D1SpecConfig *c, const int64_t *actions, void *obs_bf16,
                         void *cobs, uint16_t *legal, float *out, int64_t out_env, int64_t out_col, const bool *active,
                         void *stream) {
    if (int err = spec_check(n, c)) return err;
    if (n == 0) return 0;
    if (out_env < 1 || out_col < 1) return D1_ERR_BAD_ARGUMENT;
    cudaLaunchAttribute attr;
    const cudaLaunchConfig_t cfg = pdl_config(dim3((n + spec::WARPS - 1) / spec::WARPS), dim3(spec::WARPS * 32), 0,
                                              (cudaStream_t)stream, &attr);
    return (int)cudaLaunchKernelEx(&cfg, spec::step_kernel, (uint8_t *)state, n, *c, g_rays, spec_extra_layers(*c),
                                   actions, (__nv_bfloat16 *)obs_bf16, (uint8_t *)cobs, legal, out, out_env, out_col,
                                   active);
}

int d1_spec_step_ex(void *state, int n, const D1SpecConfig *c, const int64_t *actions, void *obs_bf16, void *cobs,
                    uint16_t *legal, float *out, const bool *active, void *stream) {
    return d1_spec_step_strided(state, n, c, actions, obs_bf16, cobs, legal, out, spec::OUT, 1, active, stream);
}

int d1_spec_step(void *state, int n, const D1SpecConfig *c, const int64_t *actions, void *obs_bf16, uint16_t *legal,
                 float *out, const bool *active, void *stream) {
    return d1_spec_step_ex(state, n, c, actions, obs_bf16, nullptr, legal, out, active, stream);
}

int d1_spec_observe(void *state, int n, const D1SpecConfig *c, void *obs_bf16, void *cobs, uint16_t *legal,
                    void *stream) {
    if (int err = spec_check(n, c)) return err;
    if (n == 0) return 0;
    if (!state || !legal) return D1_ERR_BAD_ARGUMENT;
    spec::observe_kernel<<<(n + spec::WARPS - 1) / spec::WARPS, spec::WARPS * 32, 0, (cudaStream_t)stream>>>(
        (uint8_t *)state, n, *c, (__nv_bfloat16 *)obs_bf16, (uint8_t *)cobs, legal);
    return (int)cudaGetLastError();
}

int d1_spec_compact(const void *state, int n, int64_t *rows, void *stream) {
    if (n < 0) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    const int total = n * spec::COMPACT;
    spec::compact_kernel<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>((const uint8_t *)state, n, rows);
    return (int)cudaGetLastError();
}

int d1_spec_planes(const void *state, int n, uint32_t *floor, uint32_t *viewed, void *stream) {
    if (n < 0) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    const int total = n * spec::PL;
    spec::planes_kernel<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>((const uint8_t *)state, n, floor,
                                                                                 viewed);
    return (int)cudaGetLastError();
}

}  // extern "C"
