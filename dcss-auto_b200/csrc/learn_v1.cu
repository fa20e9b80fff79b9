// Reference-compatible D:1 task ("v1") on sm_100a: the behaviour of the
// reference's default learn.cu build (gpu-d1/src/learn.cu with no -D flags) over
// the rules of gpu-d1/src/sim.h, re-laid-out for a warp per environment.
//
// State row (128 B per env, one coalesced read and write per step):
//   0  u64 rng.state   8 u64 rng.inc   16 u64 episode
//   24 i32 hp, regen, blocks, player, ticks, killed
//   48 i16 pos[8]      64 i16 energy[8]   80 i16 hp[8]      96..127 unused
// The reference keeps an int16 occupancy grid of 5600 cells per env (11.2 KB);
// here occupancy is a ballot over the lane-distributed monster positions.
#include "d1_common.cuh"
#include "d1_bfs.cuh"

namespace d1 {
namespace v1 {

constexpr int ENEMIES = 8, OBS = 206, ACTIONS = 9, OUT = 8, ROW = 128, COMPACT = 33;
constexpr int WARPS_PER_BLOCK = 8;

// Per-warp shared scratch of the repair search: its list (cell, first step)
// and a membership bit plane (row y = words 3y..3y+2).
struct Scratch {
    uint32_t inlist[PLANE];
    int16_t cell[24], first[24];
};

struct State {
    Pcg rng;
    uint64_t episode;
    int hp, regen, blocks, player, ticks, killed;
    int m_pos, m_energy, m_hp;  // this lane's monster (lane < 8), hp 0 beyond count
    Scratch *sc;
};

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
__device__ __forceinline__ bool floor_at(const D1Tables &t, int p) { return p >= 0 && p < N && t.floor[p]; }
__device__ __forceinline__ const uint16_t *field(const D1Tables &t, int player) {
    return t.distance + (size_t)t.index[player] * N;
}

__device__ __forceinline__ void load(const uint8_t *row, int lane, State &s) {
    const uint64_t *q = reinterpret_cast<const uint64_t *>(row);
    s.rng.state = q[0];
    s.rng.inc = q[1];
    s.episode = q[2];
    const int2 a = *reinterpret_cast<const int2 *>(row + 24);  // hp, regen
    const int2 b = *reinterpret_cast<const int2 *>(row + 32);  // blocks, player
    const int2 e = *reinterpret_cast<const int2 *>(row + 40);  // ticks, killed
    s.hp = a.x;
    s.regen = a.y;
    s.blocks = b.x;
    s.player = b.y;
    s.ticks = e.x;
    s.killed = e.y;
    const int16_t *m = reinterpret_cast<const int16_t *>(row + 48);
    int l = lane & 7;
    s.m_pos = m[l];
    s.m_energy = m[8 + l];
    s.m_hp = lane < ENEMIES ? m[16 + l] : 0;
}
__device__ __forceinline__ void store(uint8_t *row, int lane, const State &s) {
    if (lane == 0) {
        uint64_t *q = reinterpret_cast<uint64_t *>(row);
        q[0] = s.rng.state;
        q[1] = s.rng.inc;
        q[2] = s.episode;
        *reinterpret_cast<int2 *>(row + 24) = make_int2(s.hp, s.regen);
        *reinterpret_cast<int2 *>(row + 32) = make_int2(s.blocks, s.player);
        *reinterpret_cast<int2 *>(row + 40) = make_int2(s.ticks, s.killed);
    }
    if (lane < ENEMIES) {
        int16_t *m = reinterpret_cast<int16_t *>(row + 48);
        m[lane] = (int16_t)s.m_pos;
        m[8 + lane] = (int16_t)s.m_energy;
        m[16 + lane] = (int16_t)s.m_hp;
    }
}

// gpu-d1/src/learn.cu:291-327 (default build).
__device__ void reset(State &s, const D1Config &c, const D1Tables &t, int lane) {
    s.player = t.cells[rng_r(s.rng, t.ncells)];
    s.hp = c.hp;
    s.regen = 0;
    s.blocks = 0;
    s.ticks = 0;
    s.killed = 0;
    s.m_hp = 0;  // the occupancy grid is cleared before placement
    for (int i = 0; i < c.count; i++) {
        int p;
        do {
            p = t.cells[rng_r(s.rng, t.ncells)];
        } while (p == s.player || occupant(s.m_pos, s.m_hp, p) >= 0);
        int e = 70 + rng_r(s.rng, 10);
        if (lane == i) {
            s.m_pos = p;
            s.m_hp = monster_hp0(i % 6);
            s.m_energy = e;
        }
    }
}

// gpu-d1/src/sim.h:207-253: distance-field step with random rotation, reservoir
// ties (walk_pick) and the bounded 24-node repair search. The eight neighbour
// tests run one per lane.
__device__ int choose_move(State &s, const D1Config &c, const D1Tables &t, const uint16_t *dist, int p, int lane) {
    const int bd = dist[p];
    int rotation = rng_r(s.rng, 4);
    const int d = lane & 7;
    int q = neighbor(p, d);
    const unsigned occd = occupied_dirs(p, s.m_pos, lane < c.count && s.m_hp > 0);  // all lanes
    const bool ok = q >= 0 && t.floor[q] && q != s.player && !((occd >> d) & 1u);
    const unsigned cand = __ballot_sync(FULL, lane < 8 && ok && (int)dist[q] < bd);
    if (cand) return __shfl_sync(FULL, q, walk_pick(s.rng, cand, rotation));
    if (!c.repair) return -1;
    // Repair search (sim.h:225-252): FIFO over free floor from p, at most 24
    // nodes on the list, returning the first step of the first cell met (list
    // order, then compass order) that is closer to the player than p. A head's
    // 8 neighbours are tested at once: the first closer one in compass order is
    // the one the serial walk would meet first, and the others join the list in
    // compass order while there is room.
    uint32_t *inl = s.sc->inlist;
    int16_t *lc = s.sc->cell, *lf = s.sc->first;
    for (int r = lane; r < PLANE; r += 32) inl[r] = 0u;
    __syncwarp();
    if (lane == 0) {
        lc[0] = (int16_t)p;
        lf[0] = -1;
        inl[(p / W) * ROWW + (p % W) / 32] = 1u << ((p % W) & 31);
    }
    __syncwarp();
    const int dp = dist[p];
    int len = 1;
    for (int head = 0; head < len; head++) {
        const int ch = lc[head], fh = lf[head];
        const int qn = neighbor(ch, d);
        const unsigned occd = occupied_dirs(ch, s.m_pos, lane < c.count && s.m_hp > 0);
        const bool okn = lane < 8 && qn >= 0 && t.floor[qn] && qn != s.player &&
                         !((inl[(qn / W) * ROWW + (qn % W) / 32] >> ((qn % W) & 31)) & 1u) && !((occd >> d) & 1u);
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
            atomicOr(&inl[(qn / W) * ROWW + (qn % W) / 32], 1u << ((qn % W) & 31));
        }
        len = imin(24, len + __popc(cand));
        __syncwarp();
    }
    return -1;
}

// gpu-d1/src/sim.h:254-269
__device__ void act(State &s, const D1Config &c, const D1Tables &t, const uint16_t *dist, int id, int lane) {
    if (lane == id) s.m_energy -= 10;
    int mp = __shfl_sync(FULL, s.m_pos, id);
    if (cheb(mp, s.player) == 1) {
        D1Kind k = kind_of(c, id % 6);
        incoming_attack(s.rng, c, k.damage, k.tohit, k.bypass, 1, s.hp, s.blocks);
        return;
    }
    int q = choose_move(s, c, t, dist, mp, lane);
    if (q >= 0 && lane == id) s.m_pos = q;
}

// gpu-d1/src/learn.cu:505-598 (default build). Returns the outcome row in
// registers: lane j < 8 holds out[j].
__device__ float transition(State &s, const D1Config &c, const D1Tables &t, int action, int limit, int lane) {
    float reward = -0.001f;
    s.blocks = 0;
    s.regen += c.regen;
    while (s.regen >= 100) {
        s.hp = imin(c.hp, s.hp + 1);
        s.regen -= 100;
    }
    if (action >= 0 && action < 8) {
        int p = neighbor(s.player, action);
        if (floor_at(t, p)) {
            int id = occupant(s.m_pos, s.m_hp, p);
            if (id >= 0) {
                if (rng_r(s.rng, 5) != 0) {
                    int dmg = 1 + rng_r(s.rng, 4);
                    if (lane == id) s.m_hp = (int16_t)(s.m_hp - dmg);
                    if (__shfl_sync(FULL, s.m_hp, id) <= 0) {
                        if (lane == id) {
                            s.m_hp = 0;
                            s.m_energy = -30000;
                        }
                        s.killed++;
                        reward += 1;
                    }
                }
            } else
                s.player = p;
        }
    }
    const bool clear = s.killed == c.count;
    if (!clear) {
        const uint16_t *dist = field(t, s.player);
        if (lane < c.count && s.m_hp > 0) s.m_energy += kind_of(c, lane % 6).speed;
        while (s.hp > 0) {
            int id = scan_ready(s.m_energy, lane, c.count);
            if (id < 0) break;
            act(s, c, t, dist, id, lane);
        }
    }
    s.ticks++;
    const bool death = s.hp <= 0, timeout = !clear && !death && s.ticks >= limit;
    if (clear) reward += 3.f;
    if (death) reward -= 0.001f * 1000;
    const bool done = clear || death || timeout;
    float o = 0.f;
    switch (lane) {
        case 0: o = reward; break;
        case 1: o = done; break;
        case 2: o = clear; break;
        case 3: o = (float)s.killed; break;
        case 4: o = (float)imax(0, s.hp); break;
        case 5: o = (float)s.ticks; break;
        case 6: o = death; break;
        case 7: o = timeout; break;
    }
    if (done) {
        s.episode++;
        reset(s, c, t, lane);
    }
    return o;
}

// gpu-d1/src/learn.cu:328-347 and 497-498 (default build), written as a gather:
// lane l produces obs[l + 32k]; every row is one coalesced 128 B store per k.
// The monster table is first broadcast into per-lane registers (unrolled, constant
// indices) so that the lane-divergent branches below need no shuffles.
__device__ void observe(const State &s, const D1Config &c, const D1Tables &t, float *o, float *mask, int lane) {
    const int px0 = s.player % W, py0 = s.player / W;
    int mp[ENEMIES], mh[ENEMIES];
#pragma unroll
    for (int k = 0; k < ENEMIES; k++) {
        mp[k] = __shfl_sync(FULL, s.m_pos, k);
        mh[k] = k < c.count ? __shfl_sync(FULL, s.m_hp, k) : 0;
    }
    for (int j = lane; j < OBS; j += 32) {
        float v = 0.f;
        if (j < 162) {
            int jj = j < 81 ? j : j - 81;
            int px = px0 + jj % 9 - 4, py = py0 + jj / 9 - 4;
            bool in = px >= 0 && px < W && py >= 0 && py < H;
            int p = py * W + px;
            if (j < 81) {
                v = (in && t.floor[p]) ? 1.f : 0.f;
            } else if (in) {
                int hp = 0;
#pragma unroll
                for (int k = 0; k < ENEMIES; k++)
                    if (mh[k] > 0 && mp[k] == p) hp = mh[k];
                if (hp) v = hp / 16.f;
            }
        } else if (j < 202) {
            int i = (j - 162) / 5, f = (j - 162) % 5, pi = 0, hi = 0;
#pragma unroll
            for (int k = 0; k < ENEMIES; k++)
                if (k == i) {
                    pi = mp[k];
                    hi = mh[k];
                }
            if (hi > 0) {
                if (f == 0) v = (pi % W - px0) / 80.f;
                else if (f == 1) v = (pi / W - py0) / 70.f;
                else if (f == 2) v = hi / 16.f;
                else if (f == 3) v = (i % 6) / 5.f;
                else v = 1.f;
            }
        } else {
            if (j == 202) v = s.hp / (float)c.hp;
            else if (j == 203) v = s.ticks / 256.f;
            else if (j == 204) v = px0 / 80.f;
            else v = py0 / 70.f;
        }
        o[j] = v;
    }
    if (lane < ACTIONS) mask[lane] = lane == 8 ? 1.f : (floor_at(t, neighbor(s.player, lane)) ? 1.f : 0.f);
}

// gpu-d1/src/learn.cu:599-621
__device__ int heuristic(const State &s, const D1Config &c, const D1Tables &t, int lane) {
    // Weakest adjacent monster, first compass direction on ties.
    const int d = lane & 7;
    int p = neighbor(s.player, d);
    int occ_hp = 0;
    for (int k = 0; k < c.count; k++) {
        int pk = __shfl_sync(FULL, s.m_pos, k), hk = __shfl_sync(FULL, s.m_hp, k);
        if (p >= 0 && hk > 0 && pk == p) occ_hp = hk;
    }
    int best = -1, bhp = 10000;
    for (int dd = 0; dd < 8; dd++) {
        int h = __shfl_sync(FULL, occ_hp, dd);
        if (h > 0 && h < bhp) {
            bhp = h;
            best = dd;
        }
    }
    if (best >= 0) return best;
    const uint16_t *ds = field(t, s.player);
    int target = -1, bd = 65535;
    for (int i = 0; i < c.count; i++) {
        int pi = __shfl_sync(FULL, s.m_pos, i), hi = __shfl_sync(FULL, s.m_hp, i);
        if (hi > 0 && ds[pi] < bd) {
            bd = ds[pi];
            target = pi;
        }
    }
    if (target < 0) return 8;
    ds = field(t, target);
    bd = ds[s.player];
    best = 8;
    for (int dd = 0; dd < 8; dd++) {
        int q = neighbor(s.player, dd);
        if (floor_at(t, q) && ds[q] < bd) {
            bd = ds[q];
            best = dd;
        }
    }
    return best;
}

__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32)
    init_kernel(uint8_t *state, int n, D1Config c, D1Tables t, uint64_t seed, float *obs, float *mask) {
    const int env = blockIdx.x * WARPS_PER_BLOCK + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (env >= n) return;
    State s;
    s.rng.seed(mix64(seed + (uint64_t)env), (uint64_t)env + 1);
    s.episode = 0;
    s.m_pos = 0;
    s.m_energy = 0;
    reset(s, c, t, lane);
    observe(s, c, t, obs + (size_t)env * OBS, mask + (size_t)env * ACTIONS, lane);
    uint8_t *row = state + (size_t)env * ROW;
    if (lane < ROW / 4) reinterpret_cast<uint32_t *>(row)[lane] = 0;
    __syncwarp();
    store(row, lane, s);
}

__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32)
    step_kernel(uint8_t *state, int n, D1Config c, D1Tables t, const int64_t *actions, int limit, float *obs,
                float *mask, float *out, const bool *active) {
    const int env = blockIdx.x * WARPS_PER_BLOCK + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (env >= n) return;
    if (active && !active[env]) return;
    __shared__ Scratch scr[WARPS_PER_BLOCK];
    uint8_t *row = state + (size_t)env * ROW;
    State s;
    s.sc = &scr[threadIdx.x >> 5];
    load(row, lane, s);
    float o = transition(s, c, t, (int)actions[env], limit, lane);
    if (lane < OUT) out[(size_t)env * OUT + lane] = o;
    observe(s, c, t, obs + (size_t)env * OBS, mask + (size_t)env * ACTIONS, lane);
    store(row, lane, s);
}

__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32)
    heuristic_kernel(const uint8_t *state, int n, D1Config c, D1Tables t, int64_t *actions) {
    const int env = blockIdx.x * WARPS_PER_BLOCK + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (env >= n) return;
    State s;
    load(state + (size_t)env * ROW, lane, s);
    int a = heuristic(s, c, t, lane);
    if (lane == 0) actions[env] = a;
}

__global__ void compact_kernel(const uint8_t *state, int n, int64_t *rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n * COMPACT) return;
    const int env = i / COMPACT, f = i % COMPACT;
    const uint8_t *row = state + (size_t)env * ROW;
    int64_t v;
    if (f < 3) v = (int64_t)reinterpret_cast<const uint64_t *>(row)[f];
    else if (f < 9) v = reinterpret_cast<const int *>(row + 24)[f - 3];
    else v = reinterpret_cast<const int16_t *>(row + 48)[f - 9];
    rows[i] = v;
}

// Device restatement of learn.cu:677-707 on one warp; result in *status.
__device__ int g_semantic_status;
__global__ void semantic_kernel(D1Config c, D1Tables t) {
    const int lane = threadIdx.x & 31;
    __shared__ Scratch scr;
    c.count = 1;
    State s;
    s.sc = &scr;
    s.rng.seed(123, 1);
    s.episode = 0;
    s.m_pos = 0;
    s.m_energy = 0;
    reset(s, c, t, lane);
    int p = -1, q = -1, dir = -1;
    for (int j = 0; j < t.ncells && p < 0; j++)
        for (int d = 0; d < 8; d++) {
            int z = neighbor(t.cells[j], d);
            if (floor_at(t, z)) {
                p = t.cells[j];
                q = z;
                dir = d;
                break;
            }
        }
    int status = 0;
    if (p < 0) status = 1;
    float o;
    if (!status) {
        s.player = p;
        if (lane == 0) {
            s.m_pos = q;
            s.m_hp = 0;
            s.m_energy = -30000;
        }
        s.killed = 0;
        o = transition(s, c, t, dir, 256, lane);
        if (!(s.player == q && __shfl_sync(FULL, o, 1) == 0.f)) status = 2;
    }
    for (int k = 0; !status && k < 100; k++) {
        s.player = p;
        if (lane == 0) {
            s.m_pos = q;
            s.m_hp = 1;
            s.m_energy = 79;
        }
        s.hp = c.hp;
        s.regen = 0;
        s.killed = 0;
        s.ticks = 0;
        o = transition(s, c, t, dir, 256, lane);
        float o0 = __shfl_sync(FULL, o, 0), o2 = __shfl_sync(FULL, o, 2), o3 = __shfl_sync(FULL, o, 3),
              o4 = __shfl_sync(FULL, o, 4);
        if (o2 != 0.f) {
            if (!(o0 > 3.9f && o3 == 1.f && o4 == (float)c.hp)) status = 3;
            break;
        }
        if (k >= 99) status = 4;
    }
    if (!status) {
        reset(s, c, t, lane);
        s.ticks = 255;
        if (lane == 0) s.m_energy = -30000;
        o = transition(s, c, t, 8, 256, lane);
        float o1 = __shfl_sync(FULL, o, 1), o6 = __shfl_sync(FULL, o, 6), o7 = __shfl_sync(FULL, o, 7);
        if (!(o1 == 1.f && o7 == 1.f && o6 == 0.f && s.ticks == 0)) status = 5;
    }
    if (!status) {
        reset(s, c, t, lane);
        s.hp = -100;
        s.regen = 0;
        o = transition(s, c, t, 8, 256, lane);
        float o4 = __shfl_sync(FULL, o, 4), o6 = __shfl_sync(FULL, o, 6);
        if (!(o6 == 1.f && o4 == 0.f && s.hp == c.hp)) status = 6;
    }
    if (lane == 0) g_semantic_status = status;
}

// One warp per source cell: layered bitset BFS over 8-neighbour floor.
__global__ void __launch_bounds__(4 * 32)
    distance_kernel(const uint8_t *floor, const int16_t *cells, int ncells, uint16_t *distance) {
    __shared__ BfsBits bits[4];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int src = blockIdx.x * 4 + w;
    BfsBits &b = bits[w];
    load_floor_bits(floor, b.floor, lane);
    if (src >= ncells) return;
    uint16_t *row = distance + (size_t)src * N;
    for (int p = lane; p < N; p += 32) row[p] = 65535;
    __syncwarp();
    bfs_layers(b, cells[src], lane, 0x7fffffff, [&](int p, int k) { row[p] = (uint16_t)k; });
}

inline int blocks_for(int n) { return (n + WARPS_PER_BLOCK - 1) / WARPS_PER_BLOCK; }

}  // namespace v1
}  // namespace d1

using namespace d1;

extern "C" {

int learn_state_bytes(void) { return v1::ROW; }
int learn_obs_size(void) { return v1::OBS; }
int learn_action_size(void) { return v1::ACTIONS; }
int learn_out_size(void) { return v1::OUT; }
int learn_config_bytes(void) { return (int)sizeof(D1Config); }

static int v1_check(int n, const D1Config *c, const D1Tables *t) {
    if (n < 0 || !c || !t || c->count < 0 || c->count > v1::ENEMIES || t->ncells <= 0 || t->ncells > N)
        return D1_ERR_BAD_ARGUMENT;
    return 0;
}

int learn_init(void *state, int n, const D1Config *c, const D1Tables *t, uint64_t seed, float *obs, float *mask,
               void *stream, int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    if (int e = v1_check(n, c, t)) return e;
    if (n == 0) return 0;
    v1::init_kernel<<<v1::blocks_for(n), v1::WARPS_PER_BLOCK * 32, 0, (cudaStream_t)stream>>>(
        (uint8_t *)state, n, *c, *t, seed, obs, mask);
    return (int)cudaGetLastError();
}

int learn_step(void *state, int n, const D1Config *c, const D1Tables *t, const int64_t *actions, int limit, float *obs,
               float *mask, float *out, void *stream, int gpu) {
    return learn_step_active(state, n, c, t, actions, limit, obs, mask, out, nullptr, stream, gpu);
}

int learn_step_active(void *state, int n, const D1Config *c, const D1Tables *t, const int64_t *actions, int limit,
                      float *obs, float *mask, float *out, const bool *active, void *stream, int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    if (int e = v1_check(n, c, t)) return e;
    if (n == 0) return 0;
    v1::step_kernel<<<v1::blocks_for(n), v1::WARPS_PER_BLOCK * 32, 0, (cudaStream_t)stream>>>(
        (uint8_t *)state, n, *c, *t, actions, limit, obs, mask, out, active);
    return (int)cudaGetLastError();
}

int learn_heuristic(void *state, int n, const D1Config *c, const D1Tables *t, int64_t *actions, void *stream, int gpu) {
    if (!gpu) return D1_ERR_NO_HOST_PATH;
    if (int e = v1_check(n, c, t)) return e;
    if (n == 0) return 0;
    v1::heuristic_kernel<<<v1::blocks_for(n), v1::WARPS_PER_BLOCK * 32, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)state, n, *c, *t, actions);
    return (int)cudaGetLastError();
}

int learn_semantic_test(const D1Config *c, const D1Tables *t) {
    if (int e = v1_check(1, c, t)) return e;
    int status = -1;
    v1::semantic_kernel<<<1, 32>>>(*c, *t);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&status, v1::g_semantic_status, sizeof(int));
    return e != cudaSuccess ? (int)e : status;
}

int learn_compact_state(const void *state, int n, int64_t *rows, void *stream) {
    if (n < 0) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    int total = n * v1::COMPACT;
    v1::compact_kernel<<<(total + 255) / 256, 256, 0, (cudaStream_t)stream>>>((const uint8_t *)state, n, rows);
    return (int)cudaGetLastError();
}

int learn_distance_table(const uint8_t *floor, const int16_t *cells, int ncells, uint16_t *distance, void *stream) {
    if (ncells < 0 || ncells > N) return D1_ERR_BAD_ARGUMENT;
    if (ncells == 0) return 0;
    v1::distance_kernel<<<(ncells + 3) / 4, 4 * 32, 0, (cudaStream_t)stream>>>(floor, cells, ncells, distance);
    return (int)cudaGetLastError();
}

}  // extern "C"
