// Shared device machinery for the D:1 env-step kernels (sm_100a).
//
// Execution model: one warp owns one environment. The game rules are a serial
// integer program with a single RNG stream (gpu-d1/src/sim.h), so every lane of
// the warp runs the same scalar rule code in lockstep on warp-uniform registers
// (no divergence, no broadcasts), while the spatial work -- neighbour scans,
// occupancy, LOS, BFS layers, observation rows -- is spread across the 32 lanes.
// Per-monster state is lane-distributed: lane i holds monster i's position,
// energy and HP, and uniform code reads it with __shfl_sync.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/d1.h"

namespace d1 {

constexpr int W = 80, H = 70, N = W * H;
constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ int imin(int a, int b) { return a < b ? a : b; }
__device__ __forceinline__ int imax(int a, int b) { return a > b ? a : b; }
__device__ __forceinline__ int iabs(int a) { return a < 0 ? -a : a; }
// Chebyshev distance between two cells (gpu-d1/src/sim.h:14).
__device__ __forceinline__ int cheb(int a, int b) { return imax(iabs(a % W - b % W), iabs(a / W - b / W)); }

// Compass order N, E, S, W, NE, SE, SW, NW (gpu-d1/src/sim.h:201-206).
__device__ __forceinline__ int neighbor(int p, int d) {
    // dx/dy packed as 2-bit signed fields to avoid a local-memory table.
    const int dx = (int)((0xA19u >> (2 * d)) & 3u) - 1;   // {0,1,0,-1,1,1,-1,-1} + 1
    const int dy = (int)((0x2864u >> (2 * d)) & 3u) - 1;  // {-1,0,1,0,-1,1,1,-1} + 1
    int x = p % W + dx, y = p / W + dy;
    return (x >= 0 && x < W && y >= 0 && y < H) ? y * W + x : -1;
}

// splitmix64 finalizer (gpu-d1/src/sim.h:15-20): the reference's per-env seed mix.
__device__ __forceinline__ uint64_t mix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ULL;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}

// PCG32 XSH-RR, the reference-compatible stream (gpu-d1/src/sim.h:21-35). Held in
// warp-uniform registers; every lane advances its identical copy.
struct Pcg {
    uint64_t state, inc;
    __device__ __forceinline__ uint32_t next() {
        uint64_t old = state;
        state = old * 6364136223846793005ULL + (inc | 1);
        uint32_t x = (uint32_t)(((old >> 18) ^ old) >> 27), r = (uint32_t)(old >> 59);
        return (x >> r) | (x << ((0u - r) & 31));
    }
    __device__ __forceinline__ void seed(uint64_t s, uint64_t seq) {
        state = 0;
        inc = (seq << 1) | 1;
        next();
        state += s;
        next();
    }
};

// Bounded draw / average / random rounding over any 32-bit stream with next():
// the unbiased multiply-high + rejection of gpu-d1/src/sim.h:36-59.
template <class G> __device__ __forceinline__ int rng_r(G &g, int bound) {
    if (bound <= 1) return 0;
    uint32_t x = g.next();
    uint64_t m = (uint64_t)x * (uint32_t)bound;
    uint32_t low = (uint32_t)m;
    if (low < (uint32_t)bound) {
        uint32_t t = (0u - (uint32_t)bound) % (uint32_t)bound;
        while (low < t) {
            x = g.next();
            m = (uint64_t)x * (uint32_t)bound;
            low = (uint32_t)m;
        }
    }
    return (int)(m >> 32);
}
// The pursuit step's tie walk (gpu-d1/src/sim.h:213-222) without the walk. The
// reference visits the directions in the order (z + rotation) % 4 for z < 4,
// then 4 + (z + rotation) % 4, keeping a free neighbour that is closer to the
// player than the mover. Distances of neighbouring cells differ by at most one,
// so the cells it can keep are exactly those one step closer (bit d of `cand`
// for direction d): the first of them in walk order, each later one replacing
// it when its draw r(2), r(3), ... comes up 0. The same draws in the same order;
// returns the kept direction (cand != 0).
template <class G> __device__ __forceinline__ int walk_pick(G &g, unsigned cand, int rotation) {
    const unsigned lo = cand & 0xfu, hi = (cand >> 4) & 0xfu;
    const unsigned walk = (((lo >> rotation) | (lo << (4 - rotation))) & 0xfu) |
                          ((((hi >> rotation) | (hi << (4 - rotation))) & 0xfu) << 4);
    int pick = __ffs(walk) - 1;
    unsigned later = walk & (walk - 1);
    for (int t = 2; later; t++) {
        const int z = __ffs(later) - 1;
        later &= later - 1;
        if (rng_r(g, t) == 0) pick = z;
    }
    return pick < 4 ? (pick + rotation) % 4 : 4 + (pick - 4 + rotation) % 4;
}
// Directions d (bit d, compass order) in which p's neighbour holds a live
// monster, for lane-distributed monsters: each monster lane marks its own
// direction from p, and one OR-reduction collects them.
__device__ __forceinline__ unsigned occupied_dirs(int p, int pos, bool live) {
    unsigned bit = 0;
    if (live) {
        const int dx = pos % W - p % W, dy = pos / W - p / W;
        if (dx >= -1 && dx <= 1 && dy >= -1 && dy <= 1 && (dx | dy)) {
            const int dir = dy == -1 ? (dx == 0 ? 0 : dx == 1 ? 4 : 7)
                                     : dy == 0 ? (dx == 1 ? 1 : 3) : (dx == 0 ? 2 : dx == 1 ? 5 : 6);
            bit = 1u << dir;
        }
    }
    return __reduce_or_sync(FULL, bit);
}
template <class G> __device__ __forceinline__ int rng_avg(G &g, int n) {
    int a = rng_r(g, n);
    return (a + rng_r(g, n + 1)) / 2;
}
template <class G> __device__ __forceinline__ int rng_round(G &g, int n, int d) {
    int rem = n % d;
    return n / d + ((rem && rng_r(g, d) < rem) ? 1 : 0);
}

// Incoming monster melee against the player (gpu-d1/src/sim.h:130-163): to-hit
// against random-rounded EV, 5% automatic hit/miss, shield block up to the
// per-turn limit, AC save with the cached GDR table. Warp-uniform.
// `damage_min` is 1 for every reference monster (1 + r(damage)); the spec ogre
// rolls damage_min + r(damage_max - damage_min + 1).
template <class G>
__device__ __forceinline__ void incoming_attack(G &g, const D1Config &c, int damage_max, int tohit, int bypass_max,
                                                int damage_min, int &hp, int &blocks) {
    int hit = rng_r(g, tohit + 1);
    int ev = rng_round(g, c.ev100, 100);
    ev = rng_avg(g, 2 * ev);
    int margin = hit - ev;
    if (rng_r(g, 100) < 5) margin = (rng_r(g, 2) ? 1 : -1) * 1000;
    int bypass = rng_r(g, bypass_max);
    int sh = rng_round(g, c.sh100, 100);
    int block = rng_avg(g, sh * 2) / 3 - 1;
    if (block >= bypass && blocks < c.shield_limit) {
        blocks++;
        return;
    }
    if (margin < 0) return;
    int damage = damage_min + rng_r(g, damage_max - damage_min + 1);
    int ac = rng_round(g, c.ac100, 100);
    int gac = rng_round(g, c.ac100, 100);
    int gdr = (gac - c.ac100 / 100) ? c.gdr[1] : c.gdr[0];
    int saved = rng_r(g, ac + 1);
    int half = rng_round(g, ac, 2);
    saved = imax(saved, imin(gdr * damage_max / 100, half));
    damage = imax(0, damage - saved);
    hp -= damage;
}

// Lane-distributed monster table helpers. Lanes >= count must hold hp <= 0.
// Which live monster stands on cell q (-1 if none): the occupancy-grid lookup of
// the reference (learn.cu State::occ), answered by one ballot.
__device__ __forceinline__ int occupant(int m_pos, int m_hp, int q) {
    unsigned b = __ballot_sync(FULL, m_hp > 0 && m_pos == q);
    return b ? __ffs(b) - 1 : -1;
}
// Stable max-energy pick over ids < count with energy >= 80, smaller id first on
// ties (gpu-d1/src/sim.h:165-174), as one warp max-reduction.
__device__ __forceinline__ int scan_ready(int m_energy, int lane, int count) {
    unsigned key = (lane < count && m_energy >= 80) ? ((unsigned)(m_energy + 32768) << 5) | (31u - lane) : 0u;
    key = __reduce_max_sync(FULL, key);
    return key ? 31 - (int)(key & 31u) : -1;
}

}  // namespace d1
