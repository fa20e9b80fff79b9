/* TEST INFRASTRUCTURE ONLY -- plain-C CPU oracle for the D:1 env step.
 * Loaded by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as a
 * checker; the product library never links or calls it.
 *
 * Every function cites the reference lines it restates. Citations are relative to
 * the reference project root (gpu-d1/...).
 */
#include "d1_oracle.h"

#include <stdlib.h>
#include <string.h>
#include <math.h>

#define W 80
#define H 70
#define N 5600

/* ------------------------------------------------------------------ */
/* Shared integer rules: gpu-d1/src/sim.h                              */
/* ------------------------------------------------------------------ */
static int mn(int a, int b) { return a < b ? a : b; }
static int mx(int a, int b) { return a > b ? a : b; }
static int ab(int a) { return a < 0 ? -a : a; }
/* sim.h:14 */
static int cheb(int a, int b) { return mx(ab(a % W - b % W), ab(a / W - b / W)); }

/* sim.h:15-20 splitmix64 finalizer. */
static uint64_t mix64(uint64_t x) {
    x += 0x9e3779b97f4a7c15ULL;
    x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
    x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
    return x ^ (x >> 31);
}

typedef struct { uint64_t state, inc; } Pcg32;

/* sim.h:23-28 PCG32 XSH-RR step. */
static uint32_t pcg_next(Pcg32 *g) {
    uint64_t old = g->state;
    g->state = old * 6364136223846793005ULL + (g->inc | 1);
    uint32_t x = (uint32_t)(((old >> 18) ^ old) >> 27), r = (uint32_t)(old >> 59);
    return (x >> r) | (x << ((0u - r) & 31));
}
/* sim.h:29-35 */
static void pcg_seed(Pcg32 *g, uint64_t s, uint64_t seq) {
    g->state = 0;
    g->inc = (seq << 1) | 1;
    pcg_next(g);
    g->state += s;
    pcg_next(g);
}

/* The bounded draw, average and random rounding are written once over an abstract
 * 32-bit source so that the v1 (PCG32) and spec (Philox) streams share them. */
typedef uint32_t (*Next32)(void *);
/* sim.h:36-51 unbiased multiply-high with rejection. */
static int rng_r(Next32 next, void *g, int bound) {
    if (bound <= 1) return 0;
    uint32_t x = next(g);
    uint64_t m = (uint64_t)x * (uint32_t)bound;
    uint32_t low = (uint32_t)m;
    if (low < (uint32_t)bound) {
        uint32_t t = (0u - (uint32_t)bound) % (uint32_t)bound;
        while (low < t) {
            x = next(g);
            m = (uint64_t)x * (uint32_t)bound;
            low = (uint32_t)m;
        }
    }
    return (int)(m >> 32);
}
/* sim.h:52-55 */
static int rng_avg(Next32 next, void *g, int n) {
    int a = rng_r(next, g, n);
    return (a + rng_r(next, g, n + 1)) / 2;
}
/* sim.h:56-59 */
static int rng_round(Next32 next, void *g, int n, int d) {
    int rem = n % d;
    return n / d + (rem && rng_r(next, g, d) < rem);
}
static uint32_t pcg_next_v(void *g) { return pcg_next((Pcg32 *)g); }

/* sim.h:201-206 compass order N, E, S, W, NE, SE, SW, NW. */
static const int DX[8] = {0, 1, 0, -1, 1, 1, -1, -1};
static const int DY[8] = {-1, 0, 1, 0, -1, 1, 1, -1};
static int neighbor(int p, int d) {
    int x = p % W + DX[d], y = p / W + DY[d];
    return x >= 0 && x < W && y >= 0 && y < H ? y * W + x : -1;
}

/* Monster-side melee against the player: sim.h:130-163. `hp` and `blocks` are the
 * player's; `kind` is the attacker's. */
static void incoming_attack(Next32 nx, void *g, const D1Config *c, const D1Kind *k, int *hp, int *blocks) {
    int hit = rng_r(nx, g, k->tohit + 1);
    int ev = rng_round(nx, g, c->ev100, 100);
    ev = rng_avg(nx, g, 2 * ev);
    int margin = hit - ev;
    if (rng_r(nx, g, 100) < 5) margin = (rng_r(nx, g, 2) ? 1 : -1) * 1000;
    int bypass = rng_r(nx, g, k->bypass);
    int sh = rng_round(nx, g, c->sh100, 100);
    int block = rng_avg(nx, g, sh * 2) / 3 - 1;
    if (block >= bypass && *blocks < c->shield_limit) {
        (*blocks)++;
        return;
    }
    if (margin < 0) return;
    int damage = 1 + rng_r(nx, g, k->damage);
    int ac = rng_round(nx, g, c->ac100, 100);
    int gac = rng_round(nx, g, c->ac100, 100);
    int gdr = c->gdr[gac - c->ac100 / 100];
    int saved = rng_r(nx, g, ac + 1);
    int half = rng_round(nx, g, ac, 2);
    saved = mx(saved, mn(gdr * k->damage / 100, half));
    damage = mx(0, damage - saved);
    *hp -= damage;
}

/* ------------------------------------------------------------------ */
/* v1 task: gpu-d1/src/learn.cu default build                          */
/* ------------------------------------------------------------------ */
typedef struct {
    Pcg32 rng;
    int hp, regen, blocks;
    uint64_t episode;
    int player, ticks, killed;
    int16_t pos[OV1_ENEMIES], energy[OV1_ENEMIES], mhp[OV1_ENEMIES];
    int16_t occ[N]; /* the reference's occupancy grid, kept as-is */
} V1;

int oracle_v1_state_bytes(void) { return (int)sizeof(V1); }

static int floor_at(const D1Tables *t, int p) { return p >= 0 && p < N && t->floor[p]; }
/* learn.cu:168-176 (single map) */
static const uint16_t *field(const D1Tables *t, int player) { return t->distance + (size_t)t->index[player] * N; }

/* sim.h:165-174 stable max-energy pick, smaller id first on ties. */
static int v1_scan(const V1 *s, int n) {
    int best = -1;
    for (int i = 0; i < n; i++)
        if (s->energy[i] >= 80 &&
            (best < 0 || s->energy[i] > s->energy[best] || (s->energy[i] == s->energy[best] && i < best)))
            best = i;
    return best;
}

/* sim.h:207-253 distance-field step with random rotation, reservoir ties and the
 * bounded 24-node repair search. */
static int v1_choose_move(V1 *s, const D1Config *c, const uint16_t *dist, const uint8_t *floor, int id) {
    int p = s->pos[id], best = -1, bd = dist[p], ties = 0, rotation = rng_r(pcg_next_v, &s->rng, 4);
    for (int z = 0; z < 8; z++) {
        int d = z < 4 ? (z + rotation) % 4 : 4 + (z + rotation) % 4;
        int q = neighbor(p, d);
        if (q < 0 || !floor[q] || q == c->player || s->occ[q] >= 0) continue;
        int dq = dist[q];
        if (dq < bd) {
            bd = dq;
            best = q;
            ties = 1;
        } else if (dq == bd && best >= 0 && rng_r(pcg_next_v, &s->rng, ++ties) == 0)
            best = q;
    }
    if (best >= 0 || !c->repair) return best;
    int cells[24], first[24], len = 1;
    cells[0] = p;
    first[0] = -1;
    for (int head = 0; head < len; head++)
        for (int d = 0; d < 8; d++) {
            int q = neighbor(cells[head], d);
            if (q < 0 || !floor[q] || q == c->player || s->occ[q] >= 0) continue;
            int seen = 0;
            for (int j = 0; j < len; j++)
                if (cells[j] == q) { seen = 1; break; }
            if (seen) continue;
            int step = head == 0 ? q : first[head];
            if (dist[q] < dist[p]) return step;
            if (len < 24) {
                cells[len] = q;
                first[len] = step;
                len++;
            }
        }
    return -1;
}

/* sim.h:254-269 */
static void v1_act(V1 *s, const D1Config *c, const uint16_t *dist, const uint8_t *floor, int id) {
    s->energy[id] -= 10;
    if (cheb(s->pos[id], c->player) == 1) {
        incoming_attack(pcg_next_v, &s->rng, c, &c->kinds[id % 6], &s->hp, &s->blocks);
        return;
    }
    int q = v1_choose_move(s, c, dist, floor, id);
    if (q >= 0) {
        s->occ[s->pos[id]] = -1;
        s->pos[id] = (int16_t)q;
        s->occ[q] = (int16_t)id;
    }
}

/* learn.cu:291-327 (default build: single map, no sleep, no exploration memory). */
static void v1_reset(V1 *s, const D1Config *c, const D1Tables *t) {
    static const int mhp[6] = {8, 10, 12, 16, 12, 10};
    for (int p = 0; p < N; p++) s->occ[p] = -1;
    s->player = t->cells[rng_r(pcg_next_v, &s->rng, t->ncells)];
    s->hp = c->hp;
    s->regen = 0;
    s->blocks = 0;
    s->ticks = 0;
    s->killed = 0;
    for (int i = 0; i < c->count; i++) {
        int p;
        do { p = t->cells[rng_r(pcg_next_v, &s->rng, t->ncells)]; } while (p == s->player || s->occ[p] >= 0);
        s->pos[i] = (int16_t)p;
        s->occ[p] = (int16_t)i;
        s->mhp[i] = (int16_t)mhp[i % 6];
        s->energy[i] = (int16_t)(70 + rng_r(pcg_next_v, &s->rng, 10));
    }
}

/* learn.cu:328-347 and 497-498 (default build). */
static void v1_observe(const V1 *s, const D1Config *c, const D1Tables *t, float *o, float *mask) {
    for (int j = 0; j < OV1_OBS; j++) o[j] = 0;
    for (int y = -4; y <= 4; y++)
        for (int x = -4; x <= 4; x++) {
            int px = s->player % W + x, py = s->player / W + y, j = (y + 4) * 9 + x + 4;
            if (px < 0 || px >= W || py < 0 || py >= H) continue;
            int p = py * W + px;
            o[j] = (float)floor_at(t, p);
            int id = s->occ[p];
            if (id >= 0) o[81 + j] = s->mhp[id] / 16.f;
        }
    for (int i = 0; i < c->count; i++)
        if (s->mhp[i] > 0) {
            int j = 162 + i * 5;
            o[j] = (s->pos[i] % W - s->player % W) / 80.f;
            o[j + 1] = (s->pos[i] / W - s->player / W) / 70.f;
            o[j + 2] = s->mhp[i] / 16.f;
            o[j + 3] = (i % 6) / 5.f;
            o[j + 4] = 1;
        }
    o[202] = s->hp / (float)c->hp;
    o[203] = s->ticks / 256.f;
    o[204] = s->player % W / 80.f;
    o[205] = s->player / W / 70.f;
    for (int d = 0; d < 8; d++) mask[d] = (float)floor_at(t, neighbor(s->player, d));
    mask[8] = 1;
}

/* learn.cu:505-598 (default build: float reward, no sleep, no exploration). */
static void v1_transition(V1 *s, D1Config c, const D1Tables *t, int action, int limit, float *out) {
    for (int j = 0; j < OV1_OUT; j++) out[j] = 0;
    float reward = -0.001f;
    s->blocks = 0;
    s->regen += c.regen;
    while (s->regen >= 100) {
        s->hp = mn(c.hp, s->hp + 1);
        s->regen -= 100;
    }
    if (action >= 0 && action < 8) {
        int p = neighbor(s->player, action);
        if (floor_at(t, p)) {
            int id = s->occ[p];
            if (id >= 0) {
                if (rng_r(pcg_next_v, &s->rng, 5) != 0) {
                    s->mhp[id] -= (int16_t)(1 + rng_r(pcg_next_v, &s->rng, 4));
                    if (s->mhp[id] <= 0) {
                        s->mhp[id] = 0;
                        s->occ[p] = -1;
                        s->energy[id] = -30000;
                        s->killed++;
                        reward += 1;
                    }
                }
            } else
                s->player = p;
        }
    }
    int clear = s->killed == c.count;
    c.player = s->player;
    const uint16_t *dist = field(t, s->player);
    if (!clear) {
        for (int i = 0; i < c.count; i++)
            if (s->mhp[i] > 0) s->energy[i] += (int16_t)c.kinds[i % 6].speed;
        while (s->hp > 0) {
            int id = v1_scan(s, c.count);
            if (id < 0) break;
            v1_act(s, &c, dist, t->floor, id);
        }
    }
    s->ticks++;
    int death = s->hp <= 0, timeout = !clear && !death && s->ticks >= limit;
    if (clear) reward += 3.f;
    if (death) reward -= 0.001f * 1000;
    out[0] = reward;
    out[1] = (float)(clear || death || timeout);
    out[2] = (float)clear;
    out[3] = (float)s->killed;
    out[4] = (float)mx(0, s->hp);
    out[5] = (float)s->ticks;
    out[6] = (float)death;
    out[7] = (float)timeout;
    if (out[1] != 0) {
        s->episode++;
        v1_reset(s, &c, t);
    }
}

/* learn.cu:599-621 */
static int v1_heuristic(const V1 *s, const D1Config *c, const D1Tables *t) {
    int best = -1, bhp = 10000;
    for (int d = 0; d < 8; d++) {
        int p = neighbor(s->player, d);
        if (p >= 0 && s->occ[p] >= 0 && s->mhp[s->occ[p]] < bhp) {
            bhp = s->mhp[s->occ[p]];
            best = d;
        }
    }
    if (best >= 0) return best;
    const uint16_t *ds = field(t, s->player);
    int target = -1, bd = 65535;
    for (int i = 0; i < c->count; i++)
        if (s->mhp[i] > 0 && ds[s->pos[i]] < bd) {
            bd = ds[s->pos[i]];
            target = s->pos[i];
        }
    if (target < 0) return 8;
    ds = field(t, target);
    bd = ds[s->player];
    best = 8;
    for (int d = 0; d < 8; d++) {
        int p = neighbor(s->player, d);
        if (floor_at(t, p) && ds[p] < bd) {
            bd = ds[p];
            best = d;
        }
    }
    return best;
}

/* learn.cu:649-659 (host path) */
int oracle_v1_init(void *states, int n, const D1Config *c, const D1Tables *t, uint64_t seed, float *obs,
                   float *mask) {
    V1 *s = (V1 *)states;
    if (c->count < 0 || c->count > OV1_ENEMIES) return 1;
    for (int i = 0; i < n; i++) {
        memset(&s[i], 0, sizeof(V1));
        pcg_seed(&s[i].rng, mix64(seed + (uint64_t)i), (uint64_t)i + 1);
        v1_reset(&s[i], c, t);
        v1_observe(&s[i], c, t, obs + (size_t)i * OV1_OBS, mask + (size_t)i * OV1_ACTIONS);
    }
    return 0;
}

/* learn.cu:661-670 (host path; `active` may be NULL) */
int oracle_v1_step(void *states, int n, const D1Config *c, const D1Tables *t, const int64_t *actions, int limit,
                   float *obs, float *mask, float *out, const uint8_t *active) {
    V1 *s = (V1 *)states;
    for (int i = 0; i < n; i++) {
        if (active && !active[i]) continue;
        v1_transition(&s[i], *c, t, (int)actions[i], limit, out + (size_t)i * OV1_OUT);
        v1_observe(&s[i], c, t, obs + (size_t)i * OV1_OBS, mask + (size_t)i * OV1_ACTIONS);
    }
    return 0;
}

/* learn.cu:671-675 */
int oracle_v1_heuristic(void *states, int n, const D1Config *c, const D1Tables *t, int64_t *actions) {
    V1 *s = (V1 *)states;
    for (int i = 0; i < n; i++) actions[i] = v1_heuristic(&s[i], c, t);
    return 0;
}

static void compact_row(int64_t *r, uint64_t st, uint64_t inc, uint64_t episode, int hp, int regen, int blocks,
                        int player, int ticks, int killed, const int16_t *pos, const int16_t *energy,
                        const int16_t *mhp) {
    r[0] = (int64_t)st;
    r[1] = (int64_t)inc;
    r[2] = (int64_t)episode;
    r[3] = hp;
    r[4] = regen;
    r[5] = blocks;
    r[6] = player;
    r[7] = ticks;
    r[8] = killed;
    for (int i = 0; i < OV1_ENEMIES; i++) {
        r[9 + i] = pos[i];
        r[17 + i] = energy[i];
        r[25 + i] = mhp[i];
    }
}

int oracle_v1_compact(const void *states, int n, int64_t *rows) {
    const V1 *s = (const V1 *)states;
    for (int i = 0; i < n; i++)
        compact_row(rows + (size_t)i * OV1_COMPACT, s[i].rng.state, s[i].rng.inc, s[i].episode, s[i].hp,
                    s[i].regen, s[i].blocks, s[i].player, s[i].ticks, s[i].killed, s[i].pos, s[i].energy,
                    s[i].mhp);
    return 0;
}

/* Byte offsets of the reference State (learn.cu:106-129 over sim.h:78-83, x86-64):
 * World{RNG 16, hp, regen, blocks, fixture, episode u64, Stats 13 x u64} = 144 B,
 * then player, ticks, killed, map_id, pos[8], energy[8], occ[5600], hp[8]. */
int oracle_v1_compact_from_reference(const void *ref_states, int n, int state_bytes, int64_t *rows) {
    if (state_bytes != 11408) return 1;
    for (int i = 0; i < n; i++) {
        const uint8_t *b = (const uint8_t *)ref_states + (size_t)i * state_bytes;
        uint64_t st, inc, episode;
        int32_t hp, regen, blocks, player, ticks, killed;
        int16_t pos[8], energy[8], mhp[8];
        memcpy(&st, b + 0, 8);
        memcpy(&inc, b + 8, 8);
        memcpy(&hp, b + 16, 4);
        memcpy(&regen, b + 20, 4);
        memcpy(&blocks, b + 24, 4);
        memcpy(&episode, b + 32, 8);
        memcpy(&player, b + 144, 4);
        memcpy(&ticks, b + 148, 4);
        memcpy(&killed, b + 152, 4);
        memcpy(pos, b + 160, 16);
        memcpy(energy, b + 176, 16);
        memcpy(mhp, b + 192 + 2 * N, 16);
        compact_row(rows + (size_t)i * OV1_COMPACT, st, inc, episode, hp, regen, blocks, player, ticks, killed,
                    pos, energy, mhp);
    }
    return 0;
}

/* learn.cu:677-707, restated with return codes instead of asserts. */
int oracle_v1_semantic_test(const D1Config *cp, const D1Tables *t) {
    D1Config c = *cp;
    c.count = 1;
    V1 s;
    memset(&s, 0, sizeof s);
    pcg_seed(&s.rng, 123, 1);
    v1_reset(&s, &c, t);
    int p = -1, q = -1, dir = -1;
    for (int j = 0; j < t->ncells && p < 0; j++)
        for (int d = 0; d < 8; d++) {
            int z = neighbor(t->cells[j], d);
            if (floor_at(t, z)) {
                p = t->cells[j];
                q = z;
                dir = d;
                break;
            }
        }
    if (p < 0) return 1;
    float out[OV1_OUT];
    for (int j = 0; j < N; j++) s.occ[j] = -1;
    s.player = p;
    s.pos[0] = (int16_t)q;
    s.mhp[0] = 0;
    s.energy[0] = -30000;
    s.killed = 0;
    v1_transition(&s, c, t, dir, 256, out);
    if (!(s.player == q && out[1] == 0)) return 2;
    for (int k = 0; k < 100; k++) {
        for (int j = 0; j < N; j++) s.occ[j] = -1;
        s.player = p;
        s.pos[0] = (int16_t)q;
        s.occ[q] = 0;
        s.mhp[0] = 1;
        s.energy[0] = 79;
        s.hp = c.hp;
        s.regen = 0;
        s.killed = 0;
        s.ticks = 0;
        v1_transition(&s, c, t, dir, 256, out);
        if (out[2] != 0) {
            if (!(out[0] > 3.9f && out[3] == 1 && out[4] == c.hp)) return 3;
            break;
        }
        if (k >= 99) return 4;
    }
    v1_reset(&s, &c, t);
    s.ticks = 255;
    s.energy[0] = -30000;
    v1_transition(&s, c, t, 8, 256, out);
    if (!(out[1] == 1 && out[7] == 1 && out[6] == 0 && s.ticks == 0)) return 5;
    v1_reset(&s, &c, t);
    s.hp = -100;
    s.regen = 0;
    v1_transition(&s, c, t, 8, 256, out);
    if (!(out[6] == 1 && out[4] == 0 && s.hp == c.hp)) return 6;
    return 0;
}

/* gpu-d1/scripts/learn_env.py:25-39: BFS from every reachable cell over 8-neighbour
 * floor, 65535 for unreachable. */
int oracle_distance_table(const uint8_t *floor, const int16_t *cells, int ncells, uint16_t *distance) {
    int *queue = (int *)malloc(sizeof(int) * N);
    if (!queue) return 1;
    for (int i = 0; i < ncells; i++) {
        uint16_t *ds = distance + (size_t)i * N;
        for (int p = 0; p < N; p++) ds[p] = 65535;
        int head = 0, tail = 0;
        ds[cells[i]] = 0;
        queue[tail++] = cells[i];
        while (head < tail) {
            int p = queue[head++];
            for (int d = 0; d < 8; d++) {
                int q = neighbor(p, d);
                if (q >= 0 && floor[q] && ds[q] == 65535) {
                    ds[q] = (uint16_t)(ds[p] + 1);
                    queue[tail++] = q;
                }
            }
        }
    }
    free(queue);
    return 0;
}

/* ================================================================== */
/* spec task: the BASELINE configuration (generated maps, Philox,      */
/* 12 semantic actions, one-hot 15x15x8 + 32 observation).             */
/* Rules reused from the reference: sim.h:130-269 (melee, scheduler,   */
/* pursuit, repair search), learn.cu:505-598 (player move/attack,      */
/* regeneration, reward accounting), semantic-actions-v1 learn.cu      */
/* :190-216 (15x15 LOS view, LOS+6-tile wake), :296-331 (reveal),      */
/* :418-450 (attack-nearest, REST gating), :554-563 (sleep energy),    */
/* d1-stairs-v2 learn.cu:732 (descend ends the episode with a clear).  */
/* The generator, stream, action set and encoding have no reference:  */
/* parity for those parts is against this restatement only.            */
/* ================================================================== */
#define PLANE 210
#define MAXM OSPEC_MAXM

static struct {
    int n;
    int ex[512], ey[512];
    uint64_t blk[512];
} RAYS;

int oracle_set_rays(const int32_t *ex, const int32_t *ey, const uint64_t *blockers, int n) {
    if (n < 0 || n > 512) return 1;
    RAYS.n = n;
    for (int i = 0; i < n; i++) {
        RAYS.ex[i] = ex[i];
        RAYS.ey[i] = ey[i];
        RAYS.blk[i] = blockers[i];
    }
    return 0;
}

/* Philox4x32-10: ten rounds of the two 32x32->64 multiplies with the Weyl key
 * schedule (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as
 * 1, 2, 3", SC'11). */
void oracle_philox(const uint32_t in[4], const uint32_t key[2], uint32_t out[4]) {
    uint32_t c0 = in[0], c1 = in[1], c2 = in[2], c3 = in[3], k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0, n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1, n3 = (uint32_t)p0;
        c0 = n0;
        c1 = n1;
        c2 = n2;
        c3 = n3;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

typedef struct {
    uint64_t ctr;              /* draws consumed from this env's stream */
    uint32_t env, seed_lo, seed_hi, episode;
    int hp, regen, blocks, player, ticks, killed, stairs, nmon, floor_seen;
    int16_t pos[MAXM], energy[MAXM], mhp[MAXM];
    uint8_t kind[MAXM], awake[MAXM];
    uint32_t floor[PLANE], viewed[PLANE];
    uint32_t vis[15];          /* derived: LOS window from the player, row dy+7, bit dx+7 */
} Spec;

int oracle_spec_state_bytes(void) { return (int)sizeof(Spec); }

/* Draw n of env e under run seed s: word (n & 3) of
 * Philox4x32-10(ctr = {lo(n>>2), hi(n>>2), hi(s), 0}, key = {e, lo(s)}). */
static uint32_t spec_next(void *g) {
    Spec *s = (Spec *)g;
    uint64_t b = s->ctr >> 2;
    uint32_t ctr[4] = {(uint32_t)b, (uint32_t)(b >> 32), s->seed_hi, 0}, key[2] = {s->env, s->seed_lo}, o[4];
    oracle_philox(ctr, key, o);
    uint32_t v = o[s->ctr & 3];
    s->ctr++;
    return v;
}
static int sr(Spec *s, int bound) { return rng_r(spec_next, s, bound); }

static int bit_at(const uint32_t *plane, int p) {
    int x = p % W, y = p / W;
    return (plane[y * 3 + x / 32] >> (x % 32)) & 1;
}
static void bit_set(uint32_t *plane, int p) {
    int x = p % W, y = p / W;
    plane[y * 3 + x / 32] |= 1u << (x % 32);
}
static int sfloor(const Spec *s, int p) { return p >= 0 && p < N && bit_at(s->floor, p); }

static void carve(Spec *s, int x0, int y0, int x1, int y1) {
    if (x0 > x1) { int t = x0; x0 = x1; x1 = t; }
    if (y0 > y1) { int t = y0; y0 = y1; y1 = t; }
    for (int y = y0; y <= y1; y++)
        for (int x = x0; x <= x1; x++) bit_set(s->floor, y * W + x);
}

/* 4-9 rooms with sides 4-12 inside the one-cell wall border; room k is joined to
 * room k-1 by an L corridor between their centres, horizontal-first or
 * vertical-first by a coin flip. */
static void spec_gen_map(Spec *s) {
    memset(s->floor, 0, sizeof s->floor);
    int rooms = 4 + sr(s, 6), pcx = 0, pcy = 0;
    for (int k = 0; k < rooms; k++) {
        int w = 4 + sr(s, 9), h = 4 + sr(s, 9);
        int x0 = 1 + sr(s, W - w - 1), y0 = 1 + sr(s, H - h - 1);
        carve(s, x0, y0, x0 + w - 1, y0 + h - 1);
        int cx = x0 + w / 2, cy = y0 + h / 2;
        if (k > 0) {
            if (sr(s, 2) == 0) {
                carve(s, pcx, pcy, cx, pcy);
                carve(s, cx, pcy, cx, cy);
            } else {
                carve(s, pcx, pcy, pcx, cy);
                carve(s, pcx, cy, cx, cy);
            }
        }
        pcx = cx;
        pcy = cy;
    }
}

static int popc32(uint32_t v) { return __builtin_popcount(v); }
static int floor_count(const Spec *s) {
    int n = 0;
    for (int w = 0; w < PLANE; w++) n += popc32(s->floor[w]);
    return n;
}
/* The k-th floor cell in row-major order. */
static int kth_floor(const Spec *s, int k) {
    for (int w = 0; w < PLANE; w++) {
        int c = popc32(s->floor[w]);
        if (k < c) {
            uint32_t v = s->floor[w];
            for (int b = 0; b < 32; b++)
                if ((v >> b) & 1) {
                    if (k == 0) return (w / 3) * W + (w % 3) * 32 + b;
                    k--;
                }
        }
        k -= c;
    }
    return -1;
}

static int s_occupant(const Spec *s, int p) {
    for (int i = 0; i < s->nmon; i++)
        if (s->mhp[i] > 0 && s->pos[i] == p) return i;
    return -1;
}

/* Native ray-fan LOS (gpu-d1/scripts/compile_corpus.py:67-81): per quadrant, a
 * ray dies when any in-map wall lies on it; live rays reveal their end cell when
 * that cell is on the map. The origin is always seen. */
static void los_core(const uint8_t *floor_u8, const uint32_t *floor_bits, int origin, uint32_t vis[15]) {
    static const int SX[4] = {1, -1, -1, 1}, SY[4] = {1, 1, -1, -1};
    int px = origin % W, py = origin / W;
    memset(vis, 0, 15 * sizeof(uint32_t));
    vis[7] |= 1u << 7;
    for (int q = 0; q < 4; q++) {
        uint64_t opq = 0;
        for (int y = 0; y < 8; y++)
            for (int x = 0; x < 8; x++) {
                int cx = px + SX[q] * x, cy = py + SY[q] * y;
                if (cx < 0 || cx >= W || cy < 0 || cy >= H) continue;
                int p = cy * W + cx;
                int fl = floor_u8 ? floor_u8[p] != 0 : bit_at(floor_bits, p);
                if (!fl) opq |= 1ull << (y * 8 + x);
            }
        for (int r = 0; r < RAYS.n; r++) {
            if (RAYS.blk[r] & opq) continue;
            int cx = px + SX[q] * RAYS.ex[r], cy = py + SY[q] * RAYS.ey[r];
            if (cx < 0 || cx >= W || cy < 0 || cy >= H) continue;
            vis[SY[q] * RAYS.ey[r] + 7] |= 1u << (SX[q] * RAYS.ex[r] + 7);
        }
    }
}

int oracle_los_mask(const uint8_t *floor, int origin, uint32_t *mask10) {
    uint32_t vis[15];
    if (RAYS.n == 0) return 1;
    los_core(floor, NULL, origin, vis);
    memset(mask10, 0, 10 * sizeof(uint32_t));
    for (int dy = -7; dy <= 7; dy++)
        for (int dx = -7; dx <= 7; dx++)
            if ((vis[dy + 7] >> (dx + 7)) & 1) {
                int bit = (dy + 8) * 17 + dx + 8;
                mask10[bit / 32] |= 1u << (bit % 32);
            }
    return 0;
}

static void spec_los(Spec *s) { los_core(NULL, s->floor, s->player, s->vis); }
static int s_visible(const Spec *s, int p) {
    int dx = p % W - s->player % W, dy = p / W - s->player / W;
    if (dx < -7 || dx > 7 || dy < -7 || dy > 7) return 0;
    return (s->vis[dy + 7] >> (dx + 7)) & 1;
}
/* Mark every visible cell remembered; count newly seen floor (semantic-actions-v1
 * learn.cu:296-331 with MARK_WALLS: `seen` is `viewed` restricted to floor). */
static int spec_reveal(Spec *s) {
    int newly = 0;
    for (int dy = -7; dy <= 7; dy++)
        for (int dx = -7; dx <= 7; dx++) {
            if (!((s->vis[dy + 7] >> (dx + 7)) & 1)) continue;
            int p = (s->player / W + dy) * W + s->player % W + dx;
            if (bit_at(s->viewed, p)) continue;
            bit_set(s->viewed, p);
            if (bit_at(s->floor, p)) newly++;
        }
    s->floor_seen += newly;
    return newly;
}
static int s_visible_awake(const Spec *s) {
    for (int i = 0; i < s->nmon; i++)
        if (s->mhp[i] > 0 && s->awake[i] && s_visible(s, s->pos[i])) return 1;
    return 0;
}
/* semantic-actions-v1 learn.cu:423-428: weakest visible adjacent monster, first
 * compass direction on ties. */
static int s_adjacent_attack(const Spec *s) {
    int best = -1, hp = 100000;
    for (int d = 0; d < 8; d++) {
        int p = neighbor(s->player, d);
        if (p < 0) continue;
        int id = s_occupant(s, p);
        if (id >= 0 && s->mhp[id] > 0 && s_visible(s, p) && s->mhp[id] < hp) {
            hp = s->mhp[id];
            best = d;
        }
    }
    return best;
}

static void spec_reset(Spec *s, const D1SpecConfig *c) {
    spec_gen_map(s);
    int nf = floor_count(s);
    s->stairs = kth_floor(s, sr(s, nf));
    int tries = 0;
    do { s->player = kth_floor(s, sr(s, nf)); } while (s->player == s->stairs && ++tries < 4096);
    for (int i = 0; i < MAXM; i++) {
        s->pos[i] = 0;
        s->energy[i] = 0;
        s->mhp[i] = 0;
        s->kind[i] = 0;
        s->awake[i] = 0;
    }
    s->nmon = 0;
    int target = c->min_monsters + sr(s, c->max_monsters - c->min_monsters + 1);
    for (int i = 0; i < target; i++) {
        int kind = sr(s, 4), hp = c->min_mhp + sr(s, c->max_mhp - c->min_mhp + 1), p, bad;
        tries = 0;
        do {
            p = kth_floor(s, sr(s, nf));
            bad = p == s->player || p == s->stairs || s_occupant(s, p) >= 0;
        } while (bad && ++tries < 4096);
        if (bad) break;
        s->pos[i] = (int16_t)p;
        s->mhp[i] = (int16_t)hp;
        s->kind[i] = (uint8_t)kind;
        s->energy[i] = (int16_t)(70 + sr(s, 10));
        s->awake[i] = 0;
        s->nmon = i + 1;
    }
    if (c->ogre) {
        for (int t = 0; t < 64; t++) {
            int p = kth_floor(s, sr(s, nf));
            if (cheb(p, s->player) >= 12 && p != s->stairs && s_occupant(s, p) < 0) {
                int i = s->nmon++;
                s->pos[i] = (int16_t)p;
                s->mhp[i] = (int16_t)c->ogre_hp;
                s->kind[i] = 4;
                s->energy[i] = (int16_t)(70 + sr(s, 10));
                s->awake[i] = 0;
                break;
            }
        }
    }
    s->hp = c->hp;
    s->regen = 0;
    s->blocks = 0;
    s->ticks = 0;
    s->killed = 0;
    s->floor_seen = 0;
    memset(s->viewed, 0, sizeof s->viewed);
    spec_los(s);
    spec_reveal(s); /* the first view earns no reward */
}

/* Full FIFO BFS from the player over 8-neighbour floor (the distance field the
 * reference precomputes per player cell, learn.cu:168-176). */
static void spec_bfs(const Spec *s, uint16_t *ds) {
    static _Thread_local int queue[N]; /* per host thread: the CPU baseline steps env slices in parallel */
    for (int p = 0; p < N; p++) ds[p] = 65535;
    int head = 0, tail = 0;
    ds[s->player] = 0;
    queue[tail++] = s->player;
    while (head < tail) {
        int p = queue[head++];
        for (int d = 0; d < 8; d++) {
            int q = neighbor(p, d);
            if (q >= 0 && bit_at(s->floor, q) && ds[q] == 65535) {
                ds[q] = (uint16_t)(ds[p] + 1);
                queue[tail++] = q;
            }
        }
    }
}

/* sim.h:207-253 on the generated map. */
static int spec_choose_move(Spec *s, const uint16_t *dist, int id) {
    int p = s->pos[id], best = -1, bd = dist[p], ties = 0, rotation = sr(s, 4);
    for (int z = 0; z < 8; z++) {
        int d = z < 4 ? (z + rotation) % 4 : 4 + (z + rotation) % 4;
        int q = neighbor(p, d);
        if (q < 0 || !bit_at(s->floor, q) || q == s->player || s_occupant(s, q) >= 0) continue;
        int dq = dist[q];
        if (dq < bd) {
            bd = dq;
            best = q;
            ties = 1;
        } else if (dq == bd && best >= 0 && sr(s, ++ties) == 0)
            best = q;
    }
    if (best >= 0) return best;
    int cells[24], first[24], len = 1;
    cells[0] = p;
    first[0] = -1;
    for (int head = 0; head < len; head++)
        for (int d = 0; d < 8; d++) {
            int q = neighbor(cells[head], d);
            if (q < 0 || !bit_at(s->floor, q) || q == s->player || s_occupant(s, q) >= 0) continue;
            int seen = 0;
            for (int j = 0; j < len; j++)
                if (cells[j] == q) { seen = 1; break; }
            if (seen) continue;
            int step = head == 0 ? q : first[head];
            if (dist[q] < dist[p]) return step;
            if (len < 24) {
                cells[len] = q;
                first[len] = step;
                len++;
            }
        }
    return -1;
}

static void spec_act(Spec *s, const D1SpecConfig *c, const uint16_t *dist, int id) {
    s->energy[id] -= 10;
    if (cheb(s->pos[id], s->player) == 1) {
        const D1Kind *k = &c->kinds[s->kind[id]];
        int dmin = s->kind[id] == 4 ? c->ogre_min_damage : 1;
        D1Config pc;
        memset(&pc, 0, sizeof pc);
        pc.ev100 = c->ev100;
        pc.sh100 = c->sh100;
        pc.ac100 = c->ac100;
        pc.shield_limit = c->shield_limit;
        pc.gdr[0] = c->gdr[0];
        pc.gdr[1] = c->gdr[1];
        D1Kind kk = *k;
        /* incoming_attack rolls 1 + r(damage); the ogre's range starts at dmin. */
        if (dmin == 1) {
            incoming_attack(spec_next, s, &pc, &kk, &s->hp, &s->blocks);
        } else {
            /* sim.h:130-163 with damage = dmin + r(damage - dmin + 1). */
            Next32 nx = spec_next;
            int hit = rng_r(nx, s, kk.tohit + 1);
            int ev = rng_round(nx, s, pc.ev100, 100);
            ev = rng_avg(nx, s, 2 * ev);
            int margin = hit - ev;
            if (rng_r(nx, s, 100) < 5) margin = (rng_r(nx, s, 2) ? 1 : -1) * 1000;
            int bypass = rng_r(nx, s, kk.bypass);
            int sh = rng_round(nx, s, pc.sh100, 100);
            int block = rng_avg(nx, s, sh * 2) / 3 - 1;
            if (block >= bypass && s->blocks < pc.shield_limit) {
                s->blocks++;
                return;
            }
            if (margin < 0) return;
            int damage = dmin + rng_r(nx, s, kk.damage - dmin + 1);
            int ac = rng_round(nx, s, pc.ac100, 100);
            int gac = rng_round(nx, s, pc.ac100, 100);
            int gdr = pc.gdr[gac - pc.ac100 / 100];
            int saved = rng_r(nx, s, ac + 1);
            int half = rng_round(nx, s, ac, 2);
            saved = mx(saved, mn(gdr * kk.damage / 100, half));
            damage = mx(0, damage - saved);
            s->hp -= damage;
        }
        return;
    }
    int q = spec_choose_move(s, dist, id);
    if (q >= 0) s->pos[id] = (int16_t)q;
}

static int spec_scan(const Spec *s) {
    int best = -1;
    for (int i = 0; i < s->nmon; i++)
        if (s->energy[i] >= 80 &&
            (best < 0 || s->energy[i] > s->energy[best] || (s->energy[i] == s->energy[best] && i < best)))
            best = i;
    return best;
}

enum { PRIM_WAIT = 8, PRIM_DESCEND = 9 };
/* saw_awake: an awake monster was in view at some point of the turn -- after the
 * player's move, after any monster's action, or at its end (the interrupt signal
 * of the reference's rest macro, semantic-actions-v1 learn.cu:680-681,708,729,819). */
typedef struct { float reward; int done, descended, death, timeout, saw_awake; } Prim;

/* One physical turn: learn.cu:505-598 with the sleep/exploration variants of
 * semantic-actions-v1 learn.cu:638-730 and the stairs clear of d1-stairs-v2. */
static Prim spec_primitive(Spec *s, const D1SpecConfig *c, int d) {
    static _Thread_local uint16_t dist[N];
    Prim r = {0};
    int reward_milli = -1;
    s->blocks = 0;
    s->regen += c->regen;
    while (s->regen >= 100) {
        s->hp = mn(c->hp, s->hp + 1);
        s->regen -= 100;
    }
    if (d >= 0 && d < 8) {
        int p = neighbor(s->player, d);
        if (sfloor(s, p)) {
            int id = s_occupant(s, p);
            if (id >= 0) {
                if (sr(s, 5) != 0) {
                    s->mhp[id] = (int16_t)(s->mhp[id] - (1 + sr(s, 4)));
                    if (s->mhp[id] <= 0) {
                        s->mhp[id] = 0;
                        s->energy[id] = -30000;
                        s->killed++;
                        reward_milli += c->kill_milli;
                    }
                }
            } else {
                s->player = p;
                spec_los(s);
            }
        }
    }
    int descended = d == PRIM_DESCEND && s->player == s->stairs && s->hp > 0;
    reward_milli += c->explore_milli * spec_reveal(s);
    r.saw_awake = s_visible_awake(s);
    if (!descended) {
        for (int i = 0; i < s->nmon; i++)
            if (s->mhp[i] > 0 && !s->awake[i] && cheb(s->pos[i], s->player) <= 6 && s_visible(s, s->pos[i])) {
                s->awake[i] = 1;
                s->energy[i] = 70;
            }
        for (int i = 0; i < s->nmon; i++)
            if (s->mhp[i] > 0 && !s->awake[i]) s->energy[i] = -30000;
        for (int i = 0; i < s->nmon; i++)
            if (s->mhp[i] > 0) s->energy[i] = (int16_t)(s->energy[i] + c->kinds[s->kind[i]].speed);
        spec_bfs(s, dist);
        while (s->hp > 0) {
            int id = spec_scan(s);
            if (id < 0) break;
            spec_act(s, c, dist, id);
            if (s->awake[id] && s_visible(s, s->pos[id])) r.saw_awake = 1;
        }
    }
    s->ticks++;
    int death = s->hp <= 0, timeout = !descended && !death && s->ticks >= c->limit;
    if (descended) reward_milli += c->descend_milli;
    if (death) reward_milli -= c->death_milli;
    r.reward = 0.001f * (float)reward_milli;
    r.done = descended || death || timeout;
    r.descended = descended;
    r.death = death;
    r.timeout = timeout;
    r.saw_awake |= s_visible_awake(s);
    return r;
}

/* Actions: 0-7 move/attack N,E,S,W,NE,SE,SW,NW; 8 wait; 9 rest; 10 attack the
 * weakest visible adjacent monster; 11 descend. An action that is not legal
 * becomes one wait turn and is flagged invalid. REST repeats wait turns until HP
 * is full, an awake monster was in view during a turn, or the episode ends
 * (semantic-actions-v1 learn.cu:803-826). */
static void spec_decision(Spec *s, const D1SpecConfig *c, int a, float *out) {
    float total = 0.f;
    int elapsed = 0, invalid = 0;
    Prim r;
    for (;;) {
        int d = PRIM_WAIT;
        if (a >= 0 && a < 8) d = a;
        else if (a == 8) d = PRIM_WAIT;
        else if (a == 9) invalid = s->hp >= c->hp || s_visible_awake(s) || c->regen <= 0;
        else if (a == 10) {
            d = s_adjacent_attack(s);
            if (d < 0) {
                d = PRIM_WAIT;
                invalid = 1;
            }
        } else if (a == 11) {
            if (s->player == s->stairs) d = PRIM_DESCEND;
            else invalid = 1;
        } else
            invalid = 1;
        r = spec_primitive(s, c, d);
        elapsed++;
        total += r.reward;
        if (r.done || invalid || a != 9) break;
        if (r.saw_awake || s->hp >= c->hp) break;
    }
    out[0] = total;
    out[1] = (float)r.done;
    out[2] = (float)r.descended;
    out[3] = (float)s->killed;
    out[4] = (float)mx(0, s->hp);
    out[5] = (float)s->ticks;
    out[6] = (float)r.death;
    out[7] = (float)r.timeout;
    out[8] = (float)elapsed;
    out[9] = (float)invalid;
    if (r.done) {
        s->episode++;
        spec_reset(s, c);
    }
}

/* One-hot channel per 15x15 window cell: 0 unknown/off-map, 1 remembered wall,
 * 2 remembered floor out of view, 3 visible floor, 4 stairs, 5 visible sleeping
 * monster, 6 visible awake monster, 7 visible ogre. Then 32 scalars. */
static void spec_observe(const Spec *s, const D1SpecConfig *c, float *o, uint16_t *legal) {
    const int px = s->player % W, py = s->player / W;
    for (int j = 0; j < OSPEC_OBS; j++) o[j] = 0;
    for (int wy = 0; wy < 15; wy++)
        for (int wx = 0; wx < 15; wx++) {
            int cx = px + wx - 7, cy = py + wy - 7, ch = 0;
            if (cx >= 0 && cx < W && cy >= 0 && cy < H) {
                int p = cy * W + cx;
                if (bit_at(s->viewed, p)) {
                    if (!bit_at(s->floor, p)) ch = 1;
                    else {
                        int vis = (s->vis[wy] >> wx) & 1, id = vis ? s_occupant(s, p) : -1;
                        if (id >= 0) ch = s->kind[id] == 4 ? 7 : s->awake[id] ? 6 : 5;
                        else if (p == s->stairs) ch = 4;
                        else ch = vis ? 3 : 2;
                    }
                }
            }
            o[(wy * 15 + wx) * 8 + ch] = 1.f;
        }
    float *f = o + 1800;
    int nvis = 0, nvis_awake = 0, near = -1, neard = 1000, nadj = 0, weakest = 0, ogre = -1;
    for (int i = 0; i < s->nmon; i++) {
        if (s->mhp[i] <= 0 || !s_visible(s, s->pos[i])) continue;
        nvis++;
        nvis_awake += s->awake[i];
        int d = cheb(s->pos[i], s->player);
        if (d < neard) {
            neard = d;
            near = i;
        }
        if (d == 1) {
            nadj++;
            if (weakest == 0 || s->mhp[i] < weakest) weakest = s->mhp[i];
        }
        if (s->kind[i] == 4) ogre = i;
    }
    int rest_ok = s->hp < c->hp && c->regen > 0 && !s_visible_awake(s);
    int attack_ok = s_adjacent_attack(s) >= 0;
    int known = bit_at(s->viewed, s->stairs);
    f[0] = s->hp / (float)c->hp;
    f[1] = s->regen / 100.f;
    f[2] = s->ticks / (float)c->limit;
    f[3] = s->killed / 10.f;
    f[4] = px / 80.f;
    f[5] = py / 70.f;
    f[6] = nvis / 10.f;
    f[7] = nvis_awake / 10.f;
    if (near >= 0) {
        f[8] = 1.f;
        f[9] = (s->pos[near] % W - px) / 7.f;
        f[10] = (s->pos[near] / W - py) / 7.f;
        f[11] = s->mhp[near] / 16.f;
        f[12] = (float)s->awake[near];
        f[13] = s->kind[near] / 4.f;
    }
    f[14] = (float)known;
    if (known) {
        f[15] = (s->stairs % W - px) / 80.f;
        f[16] = (s->stairs / W - py) / 70.f;
    }
    f[17] = (float)(s->player == s->stairs);
    f[18] = nadj / 8.f;
    f[19] = weakest / 16.f;
    f[20] = (float)rest_ok;
    f[21] = (float)attack_ok;
    f[22] = s->floor_seen / 1024.f;
    f[23] = s->blocks / 2.f;
    f[24] = 1.f;
    if (ogre >= 0) {
        f[25] = 1.f;
        f[26] = (s->pos[ogre] % W - px) / 7.f;
        f[27] = (s->pos[ogre] / W - py) / 7.f;
        f[28] = (float)s->awake[ogre];
        f[29] = s->mhp[ogre] / 30.f;
    }
    uint16_t bits = 1u << 8;
    for (int d = 0; d < 8; d++)
        if (sfloor(s, neighbor(s->player, d))) bits |= (uint16_t)(1u << d);
    if (rest_ok) bits |= 1u << 9;
    if (attack_ok) bits |= 1u << 10;
    if (s->player == s->stairs) bits |= 1u << 11;
    *legal = bits;
}

int oracle_spec_init(void *states, int n, const D1SpecConfig *c, uint64_t seed, int first_env, float *obs,
                     uint16_t *legal) {
    Spec *s = (Spec *)states;
    if (RAYS.n == 0 || c->max_monsters > 10 || c->min_monsters < 0 || c->min_monsters > c->max_monsters) return 1;
    for (int i = 0; i < n; i++) {
        memset(&s[i], 0, sizeof(Spec));
        s[i].env = (uint32_t)(first_env + i);
        s[i].seed_lo = (uint32_t)seed;
        s[i].seed_hi = (uint32_t)(seed >> 32);
        spec_reset(&s[i], c);
        spec_observe(&s[i], c, obs + (size_t)i * OSPEC_OBS, legal + i);
    }
    return 0;
}

int oracle_spec_step(void *states, int n, const D1SpecConfig *c, const int64_t *actions, float *obs, uint16_t *legal,
                     float *out) {
    Spec *s = (Spec *)states;
    for (int i = 0; i < n; i++) {
        spec_decision(&s[i], c, (int)actions[i], out + (size_t)i * OSPEC_OUT);
        spec_observe(&s[i], c, obs + (size_t)i * OSPEC_OBS, legal + i);
    }
    return 0;
}

int oracle_spec_observe(const void *states, int n, const D1SpecConfig *c, float *obs, uint16_t *legal) {
    const Spec *s = (const Spec *)states;
    for (int i = 0; i < n; i++) spec_observe(&s[i], c, obs + (size_t)i * OSPEC_OBS, legal + i);
    return 0;
}

/* Rule hook for tests: the direction attack-nearest would strike from this
 * state (-1 when no visible monster is adjacent). */
int oracle_spec_attack_dir(const void *state) { return s_adjacent_attack((const Spec *)state); }

int oracle_spec_compact(const void *states, int n, int64_t *rows) {
    const Spec *s = (const Spec *)states;
    for (int i = 0; i < n; i++) {
        int64_t *r = rows + (size_t)i * OSPEC_COMPACT;
        const Spec *e = &s[i];
        r[0] = (int64_t)e->ctr;
        r[1] = e->env;
        r[2] = e->episode;
        r[3] = e->hp;
        r[4] = e->regen;
        r[5] = e->blocks;
        r[6] = e->player;
        r[7] = e->ticks;
        r[8] = e->killed;
        r[9] = e->stairs;
        r[10] = e->nmon;
        r[11] = e->floor_seen;
        for (int k = 0; k < MAXM; k++) {
            r[12 + k] = e->pos[k];
            r[23 + k] = e->energy[k];
            r[34 + k] = e->mhp[k];
            r[45 + k] = e->kind[k] * 2 + e->awake[k];
        }
    }
    return 0;
}

int oracle_spec_planes(const void *states, int n, uint32_t *floor, uint32_t *viewed) {
    const Spec *s = (const Spec *)states;
    for (int i = 0; i < n; i++) {
        memcpy(floor + (size_t)i * PLANE, s[i].floor, sizeof s[i].floor);
        memcpy(viewed + (size_t)i * PLANE, s[i].viewed, sizeof s[i].viewed);
    }
    return 0;
}

/* ================================================================== */
/* Action sampling: masked categorical over 12 logits                  */
/* (gpu-d1/scripts/run_ring_ablations.py:221-223 masks illegal logits  */
/* to -1e9 and samples torch.distributions.Categorical; torch's        */
/* multinomial stream is not a stable specification, so the draw is    */
/* defined here: inverse CDF over exp(l - max) in action order with one */
/* Philox uniform per (env, step)).                                    */
/* ================================================================== */
static float o_bits_float(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}
/* e^x for x <= 0: Cody-Waite reduction with the Cephes ln2 split, degree-7
 * Taylor polynomial, exponent-field scaling (every op separately rounded). */
static float o_exp_nonpos(float x) {
    if (x < -87.0f) return 0.0f;
    const float k = __builtin_rintf(x * 1.44269504088896341f);
    float r = x + -(k * 0.693359375f);
    r = r + -(k * -2.12194440e-4f);
    float p = 1.0f / 5040.0f;
    p = p * r + 1.0f / 720.0f;
    p = p * r + 1.0f / 120.0f;
    p = p * r + 1.0f / 24.0f;
    p = p * r + 1.0f / 6.0f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    return p * o_bits_float((uint32_t)((int)k + 127) << 23);
}

int oracle_exp_nonpos(const float *x, int n, float *y) {
    for (int i = 0; i < n; i++) y[i] = o_exp_nonpos(x[i]);
    return 0;
}

int oracle_sample_actions(const float *logits, const uint16_t *legal, int n, uint64_t seed, uint64_t step,
                          int first_env, int64_t *action, float *logp) {
    for (int i = 0; i < n; i++) {
        const float *l = logits + (size_t)i * 12;
        uint32_t bits = legal ? legal[i] : 0xfffu;
        float m = -3.402823466e38f, z[12], total = 0.f;
        for (int j = 0; j < 12; j++)
            if ((bits >> j) & 1u) m = l[j] > m ? l[j] : m;
        for (int j = 0; j < 12; j++) {
            z[j] = ((bits >> j) & 1u) ? o_exp_nonpos(l[j] + -m) : 0.f;
            total = total + z[j];
        }
        uint32_t ctr[4] = {(uint32_t)step, (uint32_t)(step >> 32), (uint32_t)(seed >> 32), 1u};
        uint32_t key[2] = {(uint32_t)(first_env + i), (uint32_t)seed}, o[4];
        oracle_philox(ctr, key, o);
        const float t = ((float)(o[0] >> 8) * (1.0f / 16777216.0f)) * total;
        int a = -1, last = 0;
        float run = 0.f;
        for (int j = 0; j < 12; j++) {
            if (!((bits >> j) & 1u)) continue;
            last = j;
            run = run + z[j];
            if (a < 0 && t < run) a = j;
        }
        if (a < 0) a = last;
        action[i] = a;
        logp[i] = (l[a] - m) - logf(total);
    }
    return 0;
}

/* ---- conv policy inputs and the autoregressive head ---- */

/* D4 element g acting on a crop offset (dx, dy): rotation r = g % 4 gives
 * (dx, dy), (dy, -dx), (-dx, -dy), (-dy, dx); g >= 4 then negates x. This is the
 * sampling rule of gpu-d1/branches/vision15-centered-map-v1/src/fast_maps.cu:7-9. */
static void d4_offset(int g, int dx, int dy, int *sx, int *sy) {
    const int r = g & 3;
    int a = r == 0 ? dx : r == 1 ? dy : r == 2 ? -dx : -dy;
    int b = r == 0 ? dy : r == 1 ? -dx : r == 2 ? -dy : dx;
    if (g >= 4) a = -a;
    *sx = a;
    *sy = b;
}

/* Egocentric 63x63 crop (rows of pitch 64, column 63 zero) of each env under D4
 * element g. Pixel (x, y) shows map cell (px + sx, py + sy) with (sx, sy) =
 * d4_offset(g, x - 31, y - 31), coded in a u16:
 *   bits 0-2  the one-hot class of the 15x15 observation (0 unknown, 1 wall,
 *             2 remembered floor, 3 visible floor, 4 stairs, 5 asleep, 6 awake,
 *             7 ogre); visibility is the LOS window, monsters only when visible
 *   bit 3     the cell is on the 80x70 map
 *   bits 4-8  hp (<= 31) of the visible monster standing there. */
int oracle_spec_crop(const void *states, int n, int g, uint16_t *out) {
    if (g < 0 || g > 7) return 1;
    const Spec *ss = (const Spec *)states;
    for (int i = 0; i < n; i++) {
        const Spec *s = &ss[i];
        const int px = s->player % W, py = s->player / W;
        uint16_t *o = out + (size_t)i * 63 * 64;
        for (int y = 0; y < 63; y++) {
            for (int x = 0; x < 64; x++) {
                uint16_t code = 0;
                if (x < 63) {
                    int sx, sy;
                    d4_offset(g, x - 31, y - 31, &sx, &sy);
                    const int cx = px + sx, cy = py + sy;
                    if (cx >= 0 && cx < W && cy >= 0 && cy < H) {
                        const int p = cy * W + cx;
                        int cls = 0, hp = 0;
                        if (bit_at(s->viewed, p)) {
                            if (!bit_at(s->floor, p)) cls = 1;
                            else {
                                const int vis = sx >= -7 && sx <= 7 && sy >= -7 && sy <= 7 &&
                                                ((s->vis[sy + 7] >> (sx + 7)) & 1);
                                const int id = vis ? s_occupant(s, p) : -1;
                                if (id >= 0) {
                                    cls = s->kind[id] == 4 ? 7 : s->awake[id] ? 6 : 5;
                                    hp = s->mhp[id] > 31 ? 31 : s->mhp[id];
                                } else if (p == s->stairs) cls = 4;
                                else cls = vis ? 3 : 2;
                            }
                        }
                        code = (uint16_t)(cls | 8 | (hp << 4));
                    }
                }
                o[y * 64 + x] = code;
            }
        }
    }
    return 0;
}

/* Validity of the verbs and of the targets of the two directional verbs from
 * the spec env's legal bits (0-7 passable neighbour, 8 wait, 9 rest allowed,
 * 10 an adjacent visible monster, 11 on the stairs):
 *   verb 0 MOVE     targets 0-7 = passable directions, target 8 never
 *   verb 1 ATTACK   targets 0-7 = passable directions, 8 = nearest; all need bit 10
 *   verb 2 WAIT, 3 REST, 4 DESCEND (bits 8, 9, 11); verbs 5-11 are not offered on D:1.
 * A directional verb is valid when any of its targets is (type_mask of
 * autoregressive-actions-v1/scripts/tactical_models.py:10-12). */
static void ar_masks(uint32_t bits, int vvalid[12], int tvalid[2][9]) {
    for (int t = 0; t < 9; t++) {
        tvalid[0][t] = t < 8 ? (int)((bits >> t) & 1u) : 0;
        tvalid[1][t] = ((bits >> 10) & 1u) ? (t < 8 ? (int)((bits >> t) & 1u) : 1) : 0;
    }
    for (int v = 0; v < 12; v++) vvalid[v] = 0;
    for (int k = 0; k < 2; k++)
        for (int t = 0; t < 9; t++) vvalid[k] |= tvalid[k][t];
    vvalid[2] = (int)((bits >> 8) & 1u);
    vvalid[3] = (int)((bits >> 9) & 1u);
    vvalid[4] = (int)((bits >> 11) & 1u);
}

static const int AR_ENV_ACTION[28] = {0, 1, 2, 3, 4, 5, 6, 7, -1,        /* MOVE t */
                                      0, 1, 2, 3, 4, 5, 6, 7, 10,        /* ATTACK t (bump), nearest */
                                      8, 9, 11, -1, -1, -1, -1, -1, -1, -1};  /* WAIT REST DESCEND, D:1-absent */

/* Inverse-CDF draw over the valid entries of l[0..k): returns the index and the
 * max / normaliser used (the flat sampler's arithmetic). */
static int ar_draw(const float *l, const int *ok, int k, float u, float *m_out, float *total_out) {
    float m = -3.402823466e38f, z[12], total = 0.f;
    for (int j = 0; j < k; j++)
        if (ok[j]) m = l[j] > m ? l[j] : m;
    for (int j = 0; j < k; j++) {
        z[j] = ok[j] ? o_exp_nonpos(l[j] + -m) : 0.f;
        total = total + z[j];
    }
    const float t = u * total;
    int a = -1, last = 0;
    float run = 0.f;
    for (int j = 0; j < k; j++) {
        if (!ok[j]) continue;
        last = j;
        run = run + z[j];
        if (a < 0 && t < run) a = j;
    }
    *m_out = m;
    *total_out = total;
    return a < 0 ? last : a;
}

/* Entropy of the masked categorical over l[0..k) (masked entries carry no mass). */
static float ar_entropy(const float *l, const int *ok, int k, float *p_out) {
    float m = -3.402823466e38f, total = 0.f;
    for (int j = 0; j < k; j++)
        if (ok[j]) m = l[j] > m ? l[j] : m;
    for (int j = 0; j < k; j++) total += ok[j] ? expf(l[j] - m) : 0.f;
    const float lz = logf(total);
    float h = 0.f;
    for (int j = 0; j < k; j++) {
        float p = 0.f;
        if (ok[j]) {
            const float lp = l[j] - m - lz;
            p = expf(lp);
            h -= p * lp;
        }
        if (p_out) p_out[j] = p;
    }
    return h;
}

/* Autoregressive verb x target sampling (type-first factorisation of
 * autoregressive-actions-v1/scripts/tactical_models.py:8-30 with 12 verbs and 9
 * targets). The verb is drawn with uniform word 0, the target of a directional
 * verb with word 1 of Philox(ctr = {lo(step), hi(step), hi(seed), 2},
 * key = {env, lo(seed)}); a directional verb with no valid target samples all
 * nine (the reference's safe dummy conditional). joint = 9v + t for v < 2, else
 * 16 + v. logp = log p(verb) + log p(target | verb); entropy = H(verb) +
 * sum over directional verbs of p(verb) H(target | verb). */
int oracle_sample_ar(const float *vl, const float *tl, const uint16_t *legal, int n, uint64_t seed, uint64_t step,
                     int first_env, int64_t *joint, int64_t *env_action, float *logp, float *entropy) {
    for (int i = 0; i < n; i++) {
        const float *l = vl + (size_t)i * 12, *lt = tl + (size_t)i * 18;
        int vvalid[12], tvalid[2][9], safe[2][9];
        ar_masks(legal[i], vvalid, tvalid);
        for (int k = 0; k < 2; k++) {
            int any = 0;
            for (int t = 0; t < 9; t++) any |= tvalid[k][t];
            for (int t = 0; t < 9; t++) safe[k][t] = tvalid[k][t] || !any;
        }
        uint32_t ctr[4] = {(uint32_t)step, (uint32_t)(step >> 32), (uint32_t)(seed >> 32), 2u};
        uint32_t key[2] = {(uint32_t)(first_env + i), (uint32_t)seed}, o[4];
        oracle_philox(ctr, key, o);
        const float uv = (float)(o[0] >> 8) * (1.0f / 16777216.0f), ut = (float)(o[1] >> 8) * (1.0f / 16777216.0f);
        float mv, tv, mt = 0.f, tt = 1.f;
        const int v = ar_draw(l, vvalid, 12, uv, &mv, &tv);
        int t = 0;
        float lp = (l[v] - mv) - logf(tv);
        if (v < 2) {
            t = ar_draw(lt + 9 * v, safe[v], 9, ut, &mt, &tt);
            lp += (lt[9 * v + t] - mt) - logf(tt);
        }
        const int j = v < 2 ? 9 * v + t : 16 + v;
        joint[i] = j;
        if (env_action) env_action[i] = AR_ENV_ACTION[j];
        logp[i] = lp;
        if (entropy) {
            float pv[12];
            float h = ar_entropy(l, vvalid, 12, pv);
            for (int k = 0; k < 2; k++)
                if (pv[k] > 0.f) h += pv[k] * ar_entropy(lt + 9 * k, safe[k], 9, NULL);
            entropy[i] = h;
        }
    }
    return 0;
}

/* Random baseline (the reference samples the legal mask uniformly,
 * gpu-d1/scripts/train_clear.py:52-53): the k-th set bit of legal & (2^nact - 1)
 * with k = floor(word * count / 2^32), word = Philox word 0 of
 * (ctr = {lo(step), hi(step), hi(seed), 3}, key = {first_env + i, lo(seed)}). */
int oracle_sample_uniform_legal(const uint16_t *legal, int nact, int n, uint64_t seed, uint64_t step, int first_env,
                                int64_t *action) {
    for (int i = 0; i < n; i++) {
        uint32_t bits = (uint32_t)legal[i] & ((1u << nact) - 1u);
        int count = 0;
        for (int j = 0; j < nact; j++) count += (bits >> j) & 1u;
        if (!count) {
            action[i] = -1;
            continue;
        }
        uint32_t ctr[4] = {(uint32_t)step, (uint32_t)(step >> 32), (uint32_t)(seed >> 32), 3u};
        uint32_t key[2] = {(uint32_t)(first_env + i), (uint32_t)seed}, o[4];
        oracle_philox(ctr, key, o);
        uint32_t k = (uint32_t)(((uint64_t)o[0] * (uint32_t)count) >> 32);
        int a = -1;
        for (int j = 0; j < nact; j++)
            if ((bits >> j) & 1u) {
                if (k == 0) {
                    a = j;
                    break;
                }
                k--;
            }
        action[i] = a;
    }
    return 0;
}
