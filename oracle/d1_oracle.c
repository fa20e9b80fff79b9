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
