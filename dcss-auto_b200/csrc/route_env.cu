// The reference's route-cue task on sm_100a: gpu-d1/src/learn.cu built with
// -DLEARN_ENEMIES=40 -DMULTI_MAP -DSLEEP_ON -DEXPLORE_REWARD -DMARK_WALLS
// -DFRONTIER_RING_MEMORY_WALLS_OBS -DKNOWN_FRONTIER -DFRONTIER_ROUTE_CUE_OBS
// -DFAST_FRONTIER (EXPLORE_MILLI 2, DEATH_MILLI 1000, CLEAR_PER_ENEMY_MILLI 0),
// the selected fast build of the reference's headline PPO benchmark
// (gpu-d1/scripts/run_ring_ablations.py:141-157, gpu-d1/PERFORMANCE.md:16).
//
// One warp per environment (see d1_common.cuh); the rules run warp-uniform on a
// single PCG stream in the reference's draw order, everything spatial runs over
// 80x70 bit planes in shared memory:
//   * occupancy is a bit plane of live monster cells (the reference's int16
//     occupancy grid of 11.2 KB per env);
//   * the remembered (viewed) plane is 840 B; seen = viewed & floor;
//   * the frontier set is a bit plane built from the frontier list, and the
//     list itself is kept in global memory in exactly the reference's
//     swap-remove order (its nearest-frontier tie break depends on that order);
//   * the known-floor BFS of learn.cu:177-203 is a layered 3x3 dilation over
//     (viewed & floor) that stops at the first layer holding a frontier cell
//     (FAST_FRONTIER), keeping each cell's distance mod 3 in two bit planes --
//     enough for the route walk-back, whose neighbours differ by at most one.
//
// State row (13,312 B per env):
//   0    u64 rng.state   8 u64 rng.inc   16 u64 episode
//   24   i32 hp, regen, blocks, player, ticks, killed, map_id, frontier_count
//   56   unused
//   64   i16 pos[40]   144 i16 energy[40]   224 i16 hp[40]   304 u8 awake[40]
//   352  u32 viewed[210]  (row y = words 3y..3y+2, bit x%32 of word x/32)
//   1216 u32 floor[210]   (the episode map's floor, written at reset)
//   2112 i16 frontier[5600] (entries [0, frontier_count) in list order)
#include "d1_common.cuh"

namespace d1 {
namespace route {

constexpr int ENEMIES = 40, OBS = 421, ACTIONS = 9, OUT = 8, COMPACT = 11 + 4 * ENEMIES;
constexpr int BASE_OBS = 81 * 2 + ENEMIES * 5 + 4;  // 366 (learn.cu:48-49)
constexpr int EXPLORE_MILLI = 2, DEATH_MILLI = 1000, CLEAR_MILLI = 3000;
constexpr int PL = 210;
constexpr int OFF_POS = 64, OFF_ENERGY = 144, OFF_HP = 224, OFF_AWAKE = 304, OFF_VIEWED = 352, OFF_FLOOR = 1216,
              OFF_LIST = 2112;
constexpr int ROW = OFF_LIST + 2 * N;  // 13,312
constexpr int WARPS = 4;

struct Smem {
    uint32_t floor[PL], viewed[PL], occ[PL], front[PL], reach[PL];
    union {
        struct {
            uint32_t a[PL], b[PL], m0[PL], m1[PL];
        } bfs;
        float obs[4 * PL];        // the observation row, staged after the search
        uint32_t keys[11 * 12];   // reveal: sorted refresh keys per region row
        struct {                  // monster phase, repair search
            uint32_t inlist[PL];     // cells on its list
            int16_t cell[24], first[24];  // the list and each entry's first step
        } nb;
    } u;
    uint32_t nw[11 * 3];  // reveal: newly viewed bits of the region rows
};

struct Env {
    Pcg rng;
    uint64_t episode;
    int hp, regen, blocks, player, ticks, killed, map_id, fcount;
    // monster `lane` (a) and monster `lane + 32` (b, lanes < 8); hp 0 = dead/unused
    int pa, ea, ha, wa, pb, eb, hb, wb;
    bool dirty_all;  // the viewed plane was cleared this step (store every row)
    int dirty_y0;    // otherwise the rows [dirty_y0, dirty_y0 + 8] changed (-100: none)
};

__device__ __forceinline__ bool bit(const uint32_t *pl, int p) {
    const int y = p / W, x = p - y * W;
    return (pl[y * 3 + (x >> 5)] >> (x & 31)) & 1u;
}
__device__ __forceinline__ void bit_or(uint32_t *pl, int p) {
    const int y = p / W, x = p - y * W;
    atomicOr(pl + y * 3 + (x >> 5), 1u << (x & 31));
}
__device__ __forceinline__ void bit_clear(uint32_t *pl, int p) {
    const int y = p / W, x = p - y * W;
    atomicAnd(pl + y * 3 + (x >> 5), ~(1u << (x & 31)));
}
__device__ __forceinline__ D1Kind kind_of(const D1Config &c, int k) {
    D1Kind r = c.kinds[0];
#pragma unroll
    for (int j = 1; j < 6; j++)
        if (k == j) r = c.kinds[j];
    return r;
}
__device__ __forceinline__ int monster_hp0(int k) {  // learn.cu:305 {8,10,12,16,12,10}
    return k == 0 ? 8 : k == 1 ? 10 : k == 2 ? 12 : k == 3 ? 16 : k == 4 ? 12 : 10;
}
// Warp-uniform read of monster `id`'s register (a for ids < 32, b above).
__device__ __forceinline__ int mget(int ra, int rb, int id) {
    return id < 32 ? __shfl_sync(FULL, ra, id) : __shfl_sync(FULL, rb, id - 32);
}
__device__ __forceinline__ void mset(int &ra, int &rb, int id, int v, int lane) {
    if (id < 32) {
        if (lane == id) ra = v;
    } else if (lane == id - 32) {
        rb = v;
    }
}
// The monster standing on q (-1 if none): the reference's occupancy lookup
// s.occ[q] (learn.cu:519), as two ballots over the lane-distributed table.
__device__ __forceinline__ int occupant(const Env &e, int q, int lane) {
    unsigned b = __ballot_sync(FULL, e.ha > 0 && e.pa == q);
    if (b) return __ffs(b) - 1;
    b = __ballot_sync(FULL, lane < 8 && e.hb > 0 && e.pb == q);
    return b ? 31 + __ffs(b) : -1;
}
// Stable max-energy pick (sim.h:164-175): energy >= 80, larger first, smaller
// id on ties; one warp max-reduction over both halves of the table.
__device__ __forceinline__ int scan_ready(const Env &e, int count, int lane) {
    const unsigned ka = (lane < count && e.ea >= 80) ? ((unsigned)(e.ea + 32768) << 6) | (63u - lane) : 0u;
    const unsigned kb = (lane < 8 && lane + 32 < count && e.eb >= 80) ? ((unsigned)(e.eb + 32768) << 6) | (31u - lane)
                                                                          : 0u;
    const unsigned key = __reduce_max_sync(FULL, ka > kb ? ka : kb);
    return key ? 63 - (int)(key & 63u) : -1;
}
__device__ __forceinline__ const uint16_t *field(const D1RouteTables &t, int map, int p) {
    const int row = t.index[(size_t)map * N + p];
    return t.distance + ((size_t)t.distance_offsets[map] + (size_t)row) * N;
}

// Floor bit plane of map `map` from its u8[5600] table: 350 16-byte units, each
// packed into 16 bits (a 16-bit half-word of the padded row).
__device__ __forceinline__ uint32_t pack4(uint32_t w) {
    const uint32_t m = __vcmpne4(w, 0u) & 0x01010101u;
    return (m * 0x00204081u) >> 21 & 0xFu;
}
__device__ void load_floor(Smem &s, const D1RouteTables &t, int map, int lane) {
    const uint4 *src = reinterpret_cast<const uint4 *>(t.floor + (size_t)map * N);
    uint16_t *h = reinterpret_cast<uint16_t *>(s.floor);
    for (int q = lane; q < 350; q += 32) {
        const uint4 v = __ldg(src + q);
        const uint32_t b = pack4(v.x) | pack4(v.y) << 4 | pack4(v.z) << 8 | pack4(v.w) << 12;
        const int y = q / 5;
        h[y * 6 + (q - y * 5)] = (uint16_t)b;
    }
    for (int y = lane; y < H; y += 32) h[y * 6 + 5] = 0;
    __syncwarp();
}

// ------------------------------------------------------------------ frontier
// Row y of a plane as three words, with rows outside the map and the bits
// past x = 79 read as `pad`.
__device__ __forceinline__ void row3(const uint32_t *pl, int y, bool pad, uint32_t &a0, uint32_t &a1, uint32_t &a2) {
    if (y < 0 || y >= H) {
        a0 = a1 = a2 = pad ? ~0u : 0u;
        return;
    }
    a0 = pl[y * 3];
    a1 = pl[y * 3 + 1];
    a2 = pl[y * 3 + 2] | (pad ? 0xFFFF0000u : 0u);
}
// want(c) of learn.cu:227-237 (MARK_WALLS): seen floor with an in-bounds
// neighbour that was never in view. Out-of-map neighbours count as viewed.
__device__ __forceinline__ void want_row(const Smem &s, int y, uint32_t w[3]) {
    uint32_t u0, u1, u2, m0, m1, m2, d0, d1, d2;
    row3(s.viewed, y - 1, true, u0, u1, u2);
    row3(s.viewed, y, true, m0, m1, m2);
    row3(s.viewed, y + 1, true, d0, d1, d2);
    // all viewed among the row's 3x3 neighbourhood (x-1 / x+1 padded with 1)
    const uint32_t c0 = u0 & d0, c1 = u1 & d1, c2 = u2 & d2;        // column x of rows y-1, y+1
    const uint32_t v0 = c0 & m0, v1 = c1 & m1, v2 = c2 & m2;        // and row y (the cell itself)
    const uint32_t l0 = (v0 << 1) | 1u, l1 = (v1 << 1) | (v0 >> 31), l2 = (v2 << 1) | (v1 >> 31);   // x-1
    const uint32_t r0 = (v0 >> 1) | (v1 << 31), r1 = (v1 >> 1) | (v2 << 31), r2 = (v2 >> 1) | 0x80000000u;  // x+1
    const uint32_t all0 = c0 & l0 & r0, all1 = c1 & l1 & r1, all2 = c2 & l2 & r2;
    // the cell itself need not be in `all` (it is viewed: seen requires it)
    w[0] = s.floor[y * 3] & s.viewed[y * 3] & ~all0;
    w[1] = s.floor[y * 3 + 1] & s.viewed[y * 3 + 1] & ~all1;
    w[2] = s.floor[y * 3 + 2] & s.viewed[y * 3 + 2] & ~all2 & 0xFFFFu;
}
// 3 bits of a padded row at x-1, x, x+1 (cells outside 0..79 read 0).
__device__ __forceinline__ uint32_t bits3(const uint32_t *r, int x) {
    uint32_t v = 0;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const int xx = x - 1 + k;
        if (xx >= 0 && xx < W) v |= ((r[xx >> 5] >> (xx & 31)) & 1u) << k;
    }
    return v;
}
// Compass index of the step from a to b (adjacent cells): N E S W NE SE SW NW.
__device__ __forceinline__ int dir_of(int dx, int dy) {
    return (int)((0x526103407ull >> (4 * ((dy + 1) * 3 + (dx + 1)))) & 15u);
}
// Position of cell c in the list [0, count) (-1 if absent).
__device__ __forceinline__ int find_slot(const int16_t *list, int count, int c, int lane) {
    for (int base = 0; base < count; base += 32) {
        const int j = base + lane;
        const int v = j < count ? (int)list[j] : -1;
        const unsigned b = __ballot_sync(FULL, v == c);
        if (b) return base + __ffs(b) - 1;
    }
    return -1;
}

// learn.cu:239-289 reveal + refresh_frontier (MARK_WALLS, RING_MEMORY_WALLS):
// marks the 9x9 view around the player, returns the newly seen floor cells,
// and brings the frontier plane and list up to date. The reference refreshes,
// in scan order, each newly viewed cell and then its 8 neighbours; a refresh
// appends a cell that became a frontier anchor and swap-removes one that
// stopped being one. All refreshes see the final memory, so a cell's first
// refresh decides it and later ones are no-ops: the list operations are the
// changed cells ordered by (first newly viewed cell of their 3x3, in scan
// order; 0 for itself, else 1 + its compass direction from that cell).
__device__ int reveal(Env &e, Smem &s, int16_t *list, int lane) {
    const int px = e.player % W, py = e.player / W;
    const int wx0 = imax(0, px - 4), wx1 = imin(W - 1, px + 4);
    // region row i = lane (< 11) is map row py - 5 + i; window rows are i = 1..9
    const int y = py - 5 + lane;
    const bool in_region = lane < 11 && y >= 0 && y < H;
    const bool in_win = lane >= 1 && lane <= 9 && y >= 0 && y < H;
    int newly = 0;
    if (lane < 11) {
        uint32_t nv[3] = {0u, 0u, 0u};
        if (in_win) {
#pragma unroll
            for (int w = 0; w < 3; w++) {
                const int lo = imax(wx0, 32 * w), hi = imin(wx1, 32 * w + 31);
                uint32_t cm = 0u;
                if (lo <= hi) cm = (hi - lo == 31 ? ~0u : ((1u << (hi - lo + 1)) - 1u)) << (lo - 32 * w);
                nv[w] = cm & ~s.viewed[y * 3 + w];
                s.viewed[y * 3 + w] |= cm;
                newly += __popc(nv[w] & s.floor[y * 3 + w]);
            }
        }
#pragma unroll
        for (int w = 0; w < 3; w++) s.nw[lane * 3 + w] = nv[w];
    }
    newly = __reduce_add_sync(FULL, newly);
    e.dirty_y0 = py - 4;
    __syncwarp();
    // touched cells T (3x3 dilation of the newly viewed cells) whose membership
    // differs from want(); their refresh keys, sorted, per region row
    int nkeys = 0;
    if (in_region) {
        uint32_t t0 = 0, t1 = 0, t2 = 0;
#pragma unroll
        for (int dy = -1; dy <= 1; dy++) {
            const int r = lane + dy;
            if (r >= 0 && r < 11) {
                t0 |= s.nw[r * 3];
                t1 |= s.nw[r * 3 + 1];
                t2 |= s.nw[r * 3 + 2];
            }
        }
        const uint32_t T0 = t0 | (t0 << 1) | (t0 >> 1) | (t1 << 31);
        const uint32_t T1 = t1 | (t1 << 1) | (t0 >> 31) | (t1 >> 1) | (t2 << 31);
        const uint32_t T2 = (t2 | (t2 << 1) | (t1 >> 31) | (t2 >> 1)) & 0xFFFFu;
        uint32_t wv[3];
        want_row(s, y, wv);
        const uint32_t T[3] = {T0, T1, T2};
        uint32_t *keys = s.u.keys + lane * 12;
#pragma unroll
        for (int w = 0; w < 3; w++) {
            const uint32_t old = s.front[y * 3 + w];
            uint32_t d = T[w] & (old ^ wv[w]);
            s.front[y * 3 + w] = (old & ~T[w]) | (wv[w] & T[w]);
            while (d) {
                const int x = 32 * w + __ffs(d) - 1;
                d &= d - 1;
                // first newly viewed cell of the 3x3 around (x, y), in scan order
                int ps = -1;
                for (int dy = -1; dy <= 1 && ps < 0; dy++) {
                    const int r = lane + dy;
                    if (r < 0 || r >= 11) continue;
                    const uint32_t b = bits3(s.nw + r * 3, x);
                    if (b) ps = (y + dy) * W + x - 1 + __ffs(b) - 1;
                }
                const int c = y * W + x;
                const uint32_t k = ps == c ? 0u : 1u + (uint32_t)dir_of(x - ps % W, y - ps / W);
                uint32_t key = (uint32_t)ps * 16u + k;
                // insertion into the row's sorted key list (at most 11 entries)
                int j = nkeys++;
                while (j > 0 && keys[j - 1] > key) {
                    keys[j] = keys[j - 1];
                    j--;
                }
                keys[j] = key;
            }
        }
    }
    __syncwarp();
    // the list operations in key order
    int head = 0;
    for (;;) {
        const uint32_t mine = head < nkeys ? s.u.keys[lane * 12 + head] : 0xFFFFFFFFu;
        const uint32_t g = __reduce_min_sync(FULL, mine);
        if (g == 0xFFFFFFFFu) break;
        if (mine == g) head++;
        const int ps = (int)(g >> 4), k = (int)(g & 15u);
        const int c = k == 0 ? ps : neighbor(ps, k - 1);
        if (bit(s.front, c)) {
            if (lane == 0) list[e.fcount] = (int16_t)c;
            e.fcount++;
        } else {
            const int slot = find_slot(list, e.fcount, c, lane);
            if (slot >= 0) {
                const int last = list[e.fcount - 1];
                __syncwarp();
                if (lane == 0) list[slot] = (int16_t)last;
                e.fcount--;
            }
        }
        __syncwarp();
    }
    return newly;
}

// ------------------------------------------------------------------ rules
__device__ void reset(Env &e, const D1Config &c, const D1RouteTables &t, int map_filter, Smem &s, int16_t *list,
                      int lane) {
    e.map_id = map_filter >= 0 ? map_filter : rng_r(e.rng, t.n_maps);
    load_floor(s, t, e.map_id, lane);
    for (int i = lane; i < PL; i += 32) {
        s.occ[i] = 0u;
        s.viewed[i] = 0u;
        s.front[i] = 0u;
    }
    __syncwarp();
    const int16_t *cells = t.cells + (size_t)e.map_id * N;
    const int ncell = t.map_ncells[e.map_id];
    e.player = cells[rng_r(e.rng, ncell)];
    e.hp = c.hp;
    e.regen = 0;
    e.blocks = 0;
    e.ticks = 0;
    e.killed = 0;
    for (int i = 0; i < c.count; i++) {
        int p;
        do {
            p = cells[rng_r(e.rng, ncell)];
        } while (p == e.player || bit(s.occ, p));
        const int en = 70 + rng_r(e.rng, 10);
        if (lane == 0) bit_or(s.occ, p);
        __syncwarp();
        mset(e.pa, e.pb, i, p, lane);
        mset(e.ha, e.hb, i, monster_hp0(i % 6), lane);
        mset(e.ea, e.eb, i, en, lane);
        mset(e.wa, e.wb, i, 0, lane);
    }
    e.fcount = 0;
    e.dirty_all = true;
    reveal(e, s, list, lane);  // the initial view earns no exploration reward
}

// sim.h:207-253 over the occupancy plane: distance-field step with random
// rotation and reservoir ties (walk_pick), then the bounded 24-node repair
// search; the eight neighbour tests run one per lane.
__device__ int choose_move(Env &e, const D1Config &c, const Smem &s, const uint16_t *dist, int p, int lane) {
    const int rotation = rng_r(e.rng, 4);
    const int d = lane & 7;
    const int q = neighbor(p, d);
    const bool ok = q >= 0 && bit(s.floor, q) && q != e.player && !bit(s.occ, q);
    const int bd = dist[p];
    const unsigned cand = __ballot_sync(FULL, lane < 8 && ok && (int)dist[q] < bd);
    if (cand) return __shfl_sync(FULL, q, walk_pick(e.rng, cand, rotation));
    if (!c.repair) return -1;
    // Repair search (sim.h:225-252): FIFO over free floor from p, at most 24
    // nodes on the list, returning the first step of the first cell met (list
    // order, then compass order) that is closer to the player than p. A head's
    // 8 neighbours are tested at once: the first closer one in compass order is
    // the one the serial walk would meet first, and the others join the list in
    // compass order while there is room. The list and its membership plane live
    // in shared memory.
    Smem &sw = const_cast<Smem &>(s);
    uint32_t *inl = sw.u.nb.inlist;
    int16_t *lc = sw.u.nb.cell, *lf = sw.u.nb.first;
    for (int i = lane; i < PL; i += 32) inl[i] = 0u;
    __syncwarp();
    if (lane == 0) {
        lc[0] = (int16_t)p;
        lf[0] = -1;
        bit_or(inl, p);
    }
    __syncwarp();
    const int dp = dist[p];
    int len = 1;
    for (int head = 0; head < len; head++) {
        const int ch = lc[head], fh = lf[head];
        const int qn = neighbor(ch, d);
        const bool okn = lane < 8 && qn >= 0 && bit(s.floor, qn) && qn != e.player && !bit(s.occ, qn) && !bit(inl, qn);
        const int dqn = okn ? (int)dist[qn] : 65535;
        const unsigned closer = __ballot_sync(FULL, okn && dqn < dp);
        if (closer) {
            const int qz = __shfl_sync(FULL, qn, __ffs(closer) - 1);
            return head == 0 ? qz : fh;
        }
        const unsigned cand = __ballot_sync(FULL, okn);
        const int rank = __popc(cand & ((1u << lane) - 1u));
        __syncwarp();
        if (okn && len + rank < 24) {
            lc[len + rank] = (int16_t)qn;
            lf[len + rank] = (int16_t)(head == 0 ? qn : fh);
            bit_or(inl, qn);
        }
        len = imin(24, len + __popc(cand));
        __syncwarp();
    }
    return -1;
}

// sim.h:254-269
__device__ void act(Env &e, const D1Config &c, Smem &s, const uint16_t *dist, int id, int lane) {
    mset(e.ea, e.eb, id, (int16_t)(mget(e.ea, e.eb, id) - 10), lane);
    const int mp = mget(e.pa, e.pb, id);
    if (cheb(mp, e.player) == 1) {
        const D1Kind k = kind_of(c, id % 6);
        incoming_attack(e.rng, c, k.damage, k.tohit, k.bypass, 1, e.hp, e.blocks);
        return;
    }
    const int q = choose_move(e, c, s, dist, mp, lane);
    if (q >= 0) {
        if (lane == 0) {
            bit_clear(s.occ, mp);
            bit_or(s.occ, q);
        }
        __syncwarp();
        mset(e.pa, e.pb, id, q, lane);
    }
}

// learn.cu:505-598 for this build. Returns lane j's outcome value (j < 8).
__device__ float transition(Env &e, const D1Config &c, const D1RouteTables &t, Smem &s, int16_t *list, int action,
                            int limit, int lane) {
    int reward_milli = -1;
    e.blocks = 0;
    e.regen += c.regen;
    while (e.regen >= 100) {
        e.hp = imin(c.hp, e.hp + 1);
        e.regen -= 100;
    }
    if (action >= 0 && action < 8) {
        const int p = neighbor(e.player, action);
        if (p >= 0 && bit(s.floor, p)) {
            const int id = occupant(e, p, lane);
            if (id >= 0) {
                // 80% hit, uniform 1..4 damage (learn.cu:520-531)
                if (rng_r(e.rng, 5) != 0) {
                    const int h = (int16_t)(mget(e.ha, e.hb, id) - (1 + rng_r(e.rng, 4)));
                    if (h <= 0) {
                        mset(e.ha, e.hb, id, 0, lane);
                        mset(e.ea, e.eb, id, -30000, lane);
                        if (lane == 0) bit_clear(s.occ, p);
                        __syncwarp();
                        e.killed++;
                        reward_milli += 1000;
                    } else {
                        mset(e.ha, e.hb, id, h, lane);
                    }
                }
            } else {
                e.player = p;
            }
        }
    }
    reward_milli += EXPLORE_MILLI * reveal(e, s, list, lane);
    const bool clear = e.killed == c.count;
    if (!clear) {
        const uint16_t *dist = field(t, e.map_id, e.player);
        // SLEEP_ON (learn.cu:553-562): wake within Chebyshev 6, sleepers hold
        // -30000, then every live monster gains its speed
        const bool a_live = lane < c.count && e.ha > 0, b_live = lane < 8 && lane + 32 < c.count && e.hb > 0;
        if (a_live && !e.wa && cheb(e.pa, e.player) <= 6) {
            e.wa = 1;
            e.ea = 70;
        }
        if (b_live && !e.wb && cheb(e.pb, e.player) <= 6) {
            e.wb = 1;
            e.eb = 70;
        }
        if (a_live && !e.wa) e.ea = -30000;
        if (b_live && !e.wb) e.eb = -30000;
        if (a_live) e.ea = (int16_t)(e.ea + kind_of(c, lane % 6).speed);
        if (b_live) e.eb = (int16_t)(e.eb + kind_of(c, (lane + 32) % 6).speed);
        while (e.hp > 0) {
            const int id = scan_ready(e, c.count, lane);
            if (id < 0) break;
            act(e, c, s, dist, id, lane);
        }
    }
    e.ticks++;
    const bool death = e.hp <= 0, timeout = !clear && !death && e.ticks >= limit;
    if (clear) reward_milli += CLEAR_MILLI;
    if (death) reward_milli -= DEATH_MILLI;
    const float reward = 0.001f * (float)reward_milli;
    const bool done = clear || death || timeout;
    float o = 0.f;
    switch (lane) {
        case 0: o = reward; break;
        case 1: o = done; break;
        case 2: o = clear; break;
        case 3: o = (float)e.killed; break;
        case 4: o = (float)imax(0, e.hp); break;
        case 5: o = (float)e.ticks; break;
        case 6: o = death; break;
        case 7: o = timeout; break;
    }
    if (done) {
        e.episode++;
        reset(e, c, t, t.map_filter, s, list, lane);
    }
    return o;
}

// ------------------------------------------------------------------ observe
// Nearest frontier through remembered floor (learn.cu:180-203, FAST_FRONTIER):
// layered BFS from the player over viewed & floor, stopping at the first layer
// that holds a listed frontier cell; the chosen cell is the first one of that
// layer in list order (learn.cu:400-418). Returns it (-1: none reachable) and
// its distance; reach/m0/m1 keep the layers for the walk-back.
__device__ int nearest_frontier(const Env &e, Smem &s, const int16_t *list, int lane, int &dmin) {
    dmin = 0;
    if (e.fcount <= 0) return -1;
    uint32_t *cur = s.u.bfs.a, *nxt = s.u.bfs.b, *m0 = s.u.bfs.m0, *m1 = s.u.bfs.m1;
    for (int i = lane; i < PL; i += 32) {
        s.reach[i] = 0u;
        cur[i] = 0u;
        nxt[i] = 0u;
        m0[i] = 0u;
        m1[i] = 0u;
    }
    __syncwarp();
    if (lane == 0) {
        bit_or(s.reach, e.player);
        bit_or(cur, e.player);
    }
    __syncwarp();
    if (bit(s.front, e.player)) return e.player;
    const int py = e.player / W;
    for (int k = 1;; k++) {
        const int y0 = imax(0, py - k), y1 = imin(H - 1, py + k);
        bool any = false, hit = false;
        for (int y = y0 + lane; y <= y1; y += 32) {
            uint32_t a0 = cur[y * 3], a1 = cur[y * 3 + 1], a2 = cur[y * 3 + 2];
            if (y > 0) {
                a0 |= cur[y * 3 - 3];
                a1 |= cur[y * 3 - 2];
                a2 |= cur[y * 3 - 1];
            }
            if (y < H - 1) {
                a0 |= cur[y * 3 + 3];
                a1 |= cur[y * 3 + 4];
                a2 |= cur[y * 3 + 5];
            }
            const uint32_t d0 = a0 | (a0 << 1) | (a0 >> 1) | (a1 << 31);
            const uint32_t d1 = a1 | (a1 << 1) | (a0 >> 31) | (a1 >> 1) | (a2 << 31);
            const uint32_t d2 = a2 | (a2 << 1) | (a1 >> 31) | (a2 >> 1);
            const uint32_t dd[3] = {d0, d1, d2};
#pragma unroll
            for (int w = 0; w < 3; w++) {
                const int r = y * 3 + w;
                const uint32_t n = dd[w] & s.floor[r] & s.viewed[r] & ~s.reach[r];
                nxt[r] = n;
                s.reach[r] |= n;
                if (k % 3 == 1) m0[r] |= n;
                if (k % 3 == 2) m1[r] |= n;
                any |= n != 0u;
                hit |= (n & s.front[r]) != 0u;
            }
        }
        __syncwarp();
        if (__any_sync(FULL, hit)) {
            dmin = k;
            // candidates: layer k & frontier; one of them -> it, else the first in list order
            int cnt = 0, first = -1;
            for (int y = y0 + lane; y <= y1; y += 32)
#pragma unroll
                for (int w = 0; w < 3; w++) {
                    const uint32_t cm = nxt[y * 3 + w] & s.front[y * 3 + w];
                    cnt += __popc(cm);
                    if (cm && first < 0) first = y * W + 32 * w + __ffs(cm) - 1;
                }
            cnt = __reduce_add_sync(FULL, cnt);
            if (cnt == 1) return __reduce_max_sync(FULL, (unsigned)(first + 1)) - 1;
            for (int base = 0; base < e.fcount; base += 32) {
                const int j = base + lane;
                const int v = j < e.fcount ? (int)list[j] : -1;
                const bool m = v >= 0 && bit(nxt, v) && bit(s.front, v);
                const unsigned b = __ballot_sync(FULL, m);
                if (b) return __shfl_sync(FULL, v, __ffs(b) - 1);
            }
            return -1;
        }
        if (!__any_sync(FULL, any)) return -1;
        uint32_t *tmp = cur;
        cur = nxt;
        nxt = tmp;
    }
}

// route_first_step (learn.cu:205-222): walk back from the target through
// cells one layer closer, first compass direction first; a neighbour's layer
// is one of k-1, k, k+1, so its distance mod 3 decides.
__device__ int route_first_step(const Env &e, const Smem &s, int target, int dmin, int lane) {
    if (target < 0 || dmin < 1) return -1;
    const uint32_t *m0 = s.u.bfs.m0, *m1 = s.u.bfs.m1;
    int p = target;
    for (int k = dmin; k > 1; k--) {
        const int q = neighbor(p, lane & 7);
        const int want = (k - 1) % 3;
        const bool m = lane < 8 && q >= 0 && bit(s.reach, q) && ((int)bit(m0, q) | (int)bit(m1, q) << 1) == want;
        const unsigned b = __ballot_sync(FULL, m);
        if (!b) return -1;
        p = neighbor(p, __ffs(b) - 1);
    }
    const unsigned b = __ballot_sync(FULL, lane < 8 && neighbor(e.player, lane) == p);
    return b ? __ffs(b) - 1 : -1;
}

// learn.cu:328-498 for this build: the 9x9 floor and monster-HP windows, 40
// monster records, the player block, the 11x11 remembered ring, the nearest
// frontier pointer and the route cue; mask = passable neighbours + wait.
__device__ void observe(const Env &e, const D1Config &c, Smem &s, const int16_t *list, float *obs, float *mask,
                        uint16_t *legal, int lane) {
    int dmin;
    const int best = nearest_frontier(e, s, list, lane, dmin);
    int unseen = 0, bdx = 0, bdy = 0, dir = -1;
    if (best >= 0) {
        const int q = neighbor(best, lane & 7);
        const unsigned b = __ballot_sync(FULL, lane < 8 && q >= 0 && !bit(s.viewed, q));
        unseen = __popc(b);
        if (b) {
            const int qf = neighbor(best, __ffs(b) - 1);
            bdx = qf % W - best % W;
            bdy = qf / W - best / W;
        }
        dir = route_first_step(e, s, best, dmin, lane);
    }
    __syncwarp();
    float *o = s.u.obs;
    for (int j = lane; j < OBS; j += 32) o[j] = 0.f;
    __syncwarp();
    const int px = e.player % W, py = e.player / W;
    for (int j = lane; j < 81; j += 32) {
        const int x = px + j % 9 - 4, y = py + j / 9 - 4;
        if (x >= 0 && x < W && y >= 0 && y < H && bit(s.floor, y * W + x)) o[j] = 1.f;
    }
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int id = h ? lane + 32 : lane;
        const int mp = h ? e.pb : e.pa, mh = h ? e.hb : e.ha;
        if ((h == 0 || lane < 8) && id < c.count && mh > 0) {
            const int dx = mp % W - px, dy = mp / W - py;
            if (iabs(dx) <= 4 && iabs(dy) <= 4) o[81 + (dy + 4) * 9 + dx + 4] = mh / 16.f;
            float *r = o + 162 + id * 5;
            r[0] = dx / 80.f;
            r[1] = dy / 70.f;
            r[2] = mh / 16.f;
            r[3] = (id % 6) / 5.f;
            r[4] = 1.f;
        }
    }
    if (lane == 0) o[BASE_OBS - 4] = e.hp / (float)c.hp;
    if (lane == 1) o[BASE_OBS - 3] = e.ticks / 256.f;
    if (lane == 2) o[BASE_OBS - 2] = px / 80.f;
    if (lane == 3) o[BASE_OBS - 1] = py / 70.f;
    for (int j = lane; j < 40; j += 32) {
        int x, y;
        if (j < 11) { y = -5; x = j - 5; }
        else if (j < 22) { y = 5; x = j - 16; }
        else if (j < 31) { x = -5; y = j - 26; }
        else { x = 5; y = j - 35; }
        const int cx = px + x, cy = py + y;
        if (cx >= 0 && cx < W && cy >= 0 && cy < H) {
            const int p = cy * W + cx;
            if (bit(s.viewed, p)) o[BASE_OBS + j] = bit(s.floor, p) ? 1.f : -1.f;
        }
    }
    if (best >= 0) {
        float v = 0.f;
        switch (lane) {
            case 0: v = 1.f; break;
            case 1: v = (best % W - px) / (float)W; break;
            case 2: v = (best / W - py) / (float)H; break;
            case 3: v = dmin / (float)(W + H); break;
            case 4: v = unseen / 8.f; break;
            case 5: v = (float)bdx; break;
            case 6: v = (float)bdy; break;
        }
        if (lane < 7) o[BASE_OBS + 40 + lane] = v;
        if (dir >= 0 && lane == 0) o[BASE_OBS + 47 + dir] = 1.f;
    }
    __syncwarp();
    for (int j = lane; j < OBS; j += 32) obs[j] = o[j];
    const int q = neighbor(e.player, lane & 7);
    const bool pass = lane == 8 || (lane < 8 && q >= 0 && bit(s.floor, q));
    if (lane < ACTIONS) mask[lane] = pass ? 1.f : 0.f;
    const unsigned lb = __ballot_sync(FULL, pass);
    if (legal && lane == 0) *legal = (uint16_t)(lb & 0x1FFu);
}

// ------------------------------------------------------------------ rows
// from_row: take the floor plane from the row (rows the library wrote), else
// pack it from the tables (rows built by hand).
__device__ void load(const uint8_t *row, Env &e, Smem &s, const D1RouteTables &t, int lane, bool from_row) {
    const uint64_t *q = reinterpret_cast<const uint64_t *>(row);
    e.rng.state = q[0];
    e.rng.inc = q[1];
    e.episode = q[2];
    const int2 h0 = *reinterpret_cast<const int2 *>(row + 24), h1 = *reinterpret_cast<const int2 *>(row + 32);
    const int2 h2 = *reinterpret_cast<const int2 *>(row + 40), h3 = *reinterpret_cast<const int2 *>(row + 48);
    e.hp = h0.x;
    e.regen = h0.y;
    e.blocks = h1.x;
    e.player = h1.y;
    e.ticks = h2.x;
    e.killed = h2.y;
    e.map_id = h3.x;
    e.fcount = h3.y;
    const int16_t *pos = reinterpret_cast<const int16_t *>(row + OFF_POS);
    const int16_t *en = reinterpret_cast<const int16_t *>(row + OFF_ENERGY);
    const int16_t *hp = reinterpret_cast<const int16_t *>(row + OFF_HP);
    const uint8_t *aw = row + OFF_AWAKE;
    e.pa = pos[lane];
    e.ea = en[lane];
    e.ha = hp[lane];
    e.wa = aw[lane];
    const int l8 = lane & 7;
    e.pb = pos[32 + l8];
    e.eb = en[32 + l8];
    e.hb = lane < 8 ? hp[32 + l8] : 0;
    e.wb = aw[32 + l8];
    const uint32_t *v = reinterpret_cast<const uint32_t *>(row + OFF_VIEWED);
    for (int i = lane; i < PL; i += 32) {
        s.viewed[i] = v[i];
        s.occ[i] = 0u;
        s.front[i] = 0u;
    }
    e.dirty_all = false;
    e.dirty_y0 = -100;
    if (from_row) {
        const uint32_t *f = reinterpret_cast<const uint32_t *>(row + OFF_FLOOR);
        for (int i = lane; i < PL; i += 32) s.floor[i] = f[i];
        __syncwarp();
    } else {
        load_floor(s, t, e.map_id, lane);  // ends with __syncwarp
    }
    if (e.ha > 0) bit_or(s.occ, e.pa);
    if (e.hb > 0) bit_or(s.occ, e.pb);
    const int16_t *list = reinterpret_cast<const int16_t *>(row + OFF_LIST);
    for (int j = lane; j < e.fcount; j += 32) bit_or(s.front, list[j]);
    __syncwarp();
}

__device__ void store(uint8_t *row, const Env &e, const Smem &s, int lane) {
    if (lane == 0) {
        uint64_t *q = reinterpret_cast<uint64_t *>(row);
        q[0] = e.rng.state;
        q[1] = e.rng.inc;
        q[2] = e.episode;
        *reinterpret_cast<int2 *>(row + 24) = make_int2(e.hp, e.regen);
        *reinterpret_cast<int2 *>(row + 32) = make_int2(e.blocks, e.player);
        *reinterpret_cast<int2 *>(row + 40) = make_int2(e.ticks, e.killed);
        *reinterpret_cast<int2 *>(row + 48) = make_int2(e.map_id, e.fcount);
    }
    int16_t *pos = reinterpret_cast<int16_t *>(row + OFF_POS);
    int16_t *en = reinterpret_cast<int16_t *>(row + OFF_ENERGY);
    int16_t *hp = reinterpret_cast<int16_t *>(row + OFF_HP);
    uint8_t *aw = row + OFF_AWAKE;
    pos[lane] = (int16_t)e.pa;
    en[lane] = (int16_t)e.ea;
    hp[lane] = (int16_t)e.ha;
    aw[lane] = (uint8_t)e.wa;
    if (lane < 8) {
        pos[32 + lane] = (int16_t)e.pb;
        en[32 + lane] = (int16_t)e.eb;
        hp[32 + lane] = (int16_t)e.hb;
        aw[32 + lane] = (uint8_t)e.wb;
    }
    uint32_t *v = reinterpret_cast<uint32_t *>(row + OFF_VIEWED);
    if (e.dirty_all) {
        uint32_t *f = reinterpret_cast<uint32_t *>(row + OFF_FLOOR);
        for (int i = lane; i < PL; i += 32) {
            v[i] = s.viewed[i];
            f[i] = s.floor[i];
        }
    } else if (e.dirty_y0 > -100) {
        const int y0 = imax(0, e.dirty_y0), y1 = imin(H - 1, e.dirty_y0 + 8);
        for (int i = y0 * 3 + lane; i < (y1 + 1) * 3; i += 32) v[i] = s.viewed[i];
    }
}

__global__ void __launch_bounds__(WARPS * 32)
    init_kernel(uint8_t *state, int n, D1Config c, D1RouteTables t, uint64_t seed, float *obs, float *mask,
                uint16_t *legal) {
    __shared__ Smem sm[WARPS];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    Smem &s = sm[w];
    uint8_t *row = state + (size_t)env * ROW;
    for (int i = lane; i < OFF_LIST / 4; i += 32) reinterpret_cast<uint32_t *>(row)[i] = 0u;
    __syncwarp();
    Env e;
    e.rng.seed(mix64(seed + (uint64_t)env), (uint64_t)env + 1);
    e.episode = 0;
    e.pa = e.ea = e.ha = e.wa = e.pb = e.eb = e.hb = e.wb = 0;
    e.dirty_y0 = -100;
    // balanced initial maps for evaluation (learn.cu:626-627)
    const int filter = t.map_filter == -2 ? env % t.n_maps : t.map_filter;
    int16_t *list = reinterpret_cast<int16_t *>(row + OFF_LIST);
    reset(e, c, t, filter, s, list, lane);
    observe(e, c, s, list, obs + (size_t)env * OBS, mask + (size_t)env * ACTIONS, legal ? legal + env : nullptr,
            lane);
    store(row, e, s, lane);
}

__global__ void __launch_bounds__(WARPS * 32)
    step_kernel(uint8_t *state, int n, D1Config c, D1RouteTables t, const int64_t *actions, int limit, float *obs,
                float *mask, float *out, const bool *active, uint16_t *legal) {
    __shared__ Smem sm[WARPS];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    if (active && !active[env]) return;
    Smem &s = sm[w];
    uint8_t *row = state + (size_t)env * ROW;
    int16_t *list = reinterpret_cast<int16_t *>(row + OFF_LIST);
    Env e;
    load(row, e, s, t, lane, true);
    const float o = transition(e, c, t, s, list, (int)actions[env], limit, lane);
    if (lane < OUT) out[(size_t)env * OUT + lane] = o;
    observe(e, c, s, list, obs + (size_t)env * OBS, mask + (size_t)env * ACTIONS, legal ? legal + env : nullptr,
            lane);
    store(row, e, s, lane);
}

__global__ void __launch_bounds__(WARPS * 32)
    observe_kernel(const uint8_t *state, int n, D1Config c, D1RouteTables t, float *obs, float *mask,
                   uint16_t *legal) {
    __shared__ Smem sm[WARPS];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    Smem &s = sm[w];
    const uint8_t *row = state + (size_t)env * ROW;
    Env e;
    load(row, e, s, t, lane, false);
    observe(e, c, s, reinterpret_cast<const int16_t *>(row + OFF_LIST), obs + (size_t)env * OBS,
            mask + (size_t)env * ACTIONS, legal ? legal + env : nullptr, lane);
}

// learn.cu:599-621: weakest adjacent monster (first compass direction on
// ties), else a step down the distance field toward the nearest monster.
__global__ void __launch_bounds__(WARPS * 32)
    heuristic_kernel(const uint8_t *state, int n, D1Config c, D1RouteTables t, int64_t *actions) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    const uint8_t *row = state + (size_t)env * ROW;
    const int player = reinterpret_cast<const int *>(row + 36)[0];
    const int map = reinterpret_cast<const int *>(row + 48)[0];
    const int16_t *pos = reinterpret_cast<const int16_t *>(row + OFF_POS);
    const int16_t *hp = reinterpret_cast<const int16_t *>(row + OFF_HP);
    Env e;
    e.pa = pos[lane];
    e.ha = hp[lane];
    e.pb = pos[32 + (lane & 7)];
    e.hb = lane < 8 ? hp[32 + (lane & 7)] : 0;
    int best = -1, bhp = 10000;
    for (int d = 0; d < 8; d++) {
        const int p = neighbor(player, d);
        if (p < 0) continue;
        const int id = occupant(e, p, lane);
        if (id >= 0) {
            const int h = mget(e.ha, e.hb, id);
            if (h < bhp) {
                bhp = h;
                best = d;
            }
        }
    }
    if (best < 0) {
        const uint16_t *ds = field(t, map, player);
        // nearest live monster by the player's field, smaller id on ties
        const unsigned ka = e.ha > 0 ? ((unsigned)ds[e.pa] << 6) | (unsigned)lane : 0xFFFFFFFFu;
        const unsigned kb = lane < 8 && e.hb > 0 ? ((unsigned)ds[e.pb] << 6) | (unsigned)(lane + 32) : 0xFFFFFFFFu;
        const unsigned key = __reduce_min_sync(FULL, ka < kb ? ka : kb);
        best = 8;
        if (key != 0xFFFFFFFFu && (key >> 6) < 65535u) {
            const int id = (int)(key & 63u);
            const int target = mget(e.pa, e.pb, id);
            const uint16_t *dt = field(t, map, target);
            const int q = neighbor(player, lane & 7);
            const bool fl = lane < 8 && q >= 0 && t.floor[(size_t)map * N + q];
            const unsigned v = fl ? ((unsigned)dt[q] << 3) | (unsigned)lane : 0xFFFFFFFFu;
            const unsigned m = __reduce_min_sync(FULL, v);
            if (m != 0xFFFFFFFFu && (m >> 3) < (unsigned)dt[player]) best = (int)(m & 7u);
        }
    }
    if (lane == 0) actions[env] = best;
}

__global__ void compact_kernel(const uint8_t *state, int n, int64_t *rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * COMPACT) return;
    const int env = i / COMPACT, f = i % COMPACT;
    const uint8_t *row = state + (size_t)env * ROW;
    int64_t v;
    if (f < 3) v = (int64_t)reinterpret_cast<const uint64_t *>(row)[f];
    else if (f < 11) v = reinterpret_cast<const int *>(row + 24)[f - 3];
    else {
        const int g = (f - 11) / ENEMIES, k = (f - 11) % ENEMIES;
        if (g == 3) v = row[OFF_AWAKE + k];
        else v = reinterpret_cast<const int16_t *>(row + (g == 0 ? OFF_POS : g == 1 ? OFF_ENERGY : OFF_HP))[k];
    }
    rows[i] = v;
}

__global__ void memory_kernel(const uint8_t *state, int n, uint32_t *viewed, int16_t *frontier) {
    const int env = blockIdx.x, lane = threadIdx.x;
    if (env >= n) return;
    const uint8_t *row = state + (size_t)env * ROW;
    const int count = reinterpret_cast<const int *>(row + 52)[0];
    const uint32_t *v = reinterpret_cast<const uint32_t *>(row + OFF_VIEWED);
    const int16_t *list = reinterpret_cast<const int16_t *>(row + OFF_LIST);
    if (viewed)
        for (int i = lane; i < PL; i += blockDim.x) viewed[(size_t)env * PL + i] = v[i];
    if (frontier)
        for (int i = lane; i < N; i += blockDim.x) frontier[(size_t)env * N + i] = i < count ? list[i] : (int16_t)-1;
}

inline int blocks_for(int n) { return (n + WARPS - 1) / WARPS; }

}  // namespace route
}  // namespace d1

using namespace d1;

extern "C" {

int d1_route_state_bytes(void) { return route::ROW; }
int d1_route_obs_size(void) { return route::OBS; }
int d1_route_action_size(void) { return route::ACTIONS; }
int d1_route_out_size(void) { return route::OUT; }
int d1_route_config_bytes(void) { return (int)sizeof(D1Config); }
int d1_route_compact_size(void) { return route::COMPACT; }

static int route_check(int n, const D1Config *c, const D1RouteTables *t) {
    if (n < 0 || !c || !t || c->count < 0 || c->count > route::ENEMIES || t->n_maps <= 0 || !t->floor || !t->cells ||
        !t->index || !t->distance || !t->map_ncells || !t->distance_offsets || t->map_filter < -2 ||
        t->map_filter >= t->n_maps || (reinterpret_cast<uintptr_t>(t->floor) & 15))
        return D1_ERR_BAD_ARGUMENT;
    return 0;
}

int d1_route_init(void *state, int n, const D1Config *c, const D1RouteTables *t, uint64_t seed, float *obs,
                  float *mask, uint16_t *legal, void *stream) {
    if (int e = route_check(n, c, t)) return e;
    if (n == 0) return 0;
    if (!state || !obs || !mask) return D1_ERR_BAD_ARGUMENT;
    route::init_kernel<<<route::blocks_for(n), route::WARPS * 32, 0, (cudaStream_t)stream>>>(
        (uint8_t *)state, n, *c, *t, seed, obs, mask, legal);
    return (int)cudaGetLastError();
}

int d1_route_step(void *state, int n, const D1Config *c, const D1RouteTables *t, const int64_t *actions, int limit,
                  float *obs, float *mask, float *out, const bool *active, uint16_t *legal, void *stream) {
    if (int e = route_check(n, c, t)) return e;
    if (n == 0) return 0;
    if (!state || !actions || !obs || !mask || !out) return D1_ERR_BAD_ARGUMENT;
    route::step_kernel<<<route::blocks_for(n), route::WARPS * 32, 0, (cudaStream_t)stream>>>(
        (uint8_t *)state, n, *c, *t, actions, limit, obs, mask, out, active, legal);
    return (int)cudaGetLastError();
}

int d1_route_observe(const void *state, int n, const D1Config *c, const D1RouteTables *t, float *obs, float *mask,
                     uint16_t *legal, void *stream) {
    if (int e = route_check(n, c, t)) return e;
    if (n == 0) return 0;
    if (!state || !obs || !mask) return D1_ERR_BAD_ARGUMENT;
    route::observe_kernel<<<route::blocks_for(n), route::WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)state, n, *c, *t, obs, mask, legal);
    return (int)cudaGetLastError();
}

int d1_route_heuristic(const void *state, int n, const D1Config *c, const D1RouteTables *t, int64_t *actions,
                       void *stream) {
    if (int e = route_check(n, c, t)) return e;
    if (n == 0) return 0;
    if (!state || !actions) return D1_ERR_BAD_ARGUMENT;
    route::heuristic_kernel<<<route::blocks_for(n), route::WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)state, n, *c, *t, actions);
    return (int)cudaGetLastError();
}

int d1_route_compact(const void *state, int n, int64_t *rows, void *stream) {
    if (n < 0 || (n > 0 && (!state || !rows))) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    const int total = n * route::COMPACT;
    route::compact_kernel<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>((const uint8_t *)state, n, rows);
    return (int)cudaGetLastError();
}

int d1_route_memory(const void *state, int n, uint32_t *viewed, int16_t *frontier, void *stream) {
    if (n < 0 || (n > 0 && !state)) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    route::memory_kernel<<<n, 256, 0, (cudaStream_t)stream>>>((const uint8_t *)state, n, viewed, frontier);
    return (int)cudaGetLastError();
}

}  // extern "C"
