/* TEST INFRASTRUCTURE ONLY -- the CPU oracle for the D:1 env-step hot path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg load this
 * library, and only as the checker. The product (libd1.so) never links it.
 *
 * Two task modes are restated here in plain C:
 *   v1    the reference's default learn.cu build (gpu-d1/src/learn.cu with no -D
 *         flags: 9 actions, 8 enemies, 206 observations, 8 outcome values), over
 *         the rules of gpu-d1/src/sim.h. Pinned against the reference itself
 *         compiled for the host (oracle/_ref/learn_v1.so) by tests/test_oracle.py.
 *   spec  the BASELINE task (generated rooms+corridors maps, Philox4x32-10, 12
 *         semantic actions, one-hot 15x15x8 + 32 observation). The reference has
 *         no code for the map generator, Philox stream, action set or encoding,
 *         so those parts are parity-unpinned; the combat, scheduler, pursuit,
 *         LOS, wake, REST and attack-nearest rules reuse the v1-pinned helpers
 *         and the reference's native LOS ray fan (pinned against native LOS).
 */
#pragma once
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Reference ABI structs (gpu-d1/src/sim.h:61-67, gpu-d1/src/learn.cu:130-139). */
typedef struct { int speed, damage, tohit, bypass; } D1Kind;
typedef struct {
    int count, player, hp, ac100, ev100, sh100, shield_limit, regen, repair, gdr[2];
    D1Kind kinds[6];
} D1Config;
typedef struct {
    const uint8_t *floor;
    const int16_t *cells, *index;
    const uint16_t *distance;
    int ncells;
} D1Tables;

/* ---- v1 (reference default build) ---- */
enum { OV1_ENEMIES = 8, OV1_OBS = 206, OV1_ACTIONS = 9, OV1_OUT = 8, OV1_COMPACT = 33 };
int oracle_v1_state_bytes(void);
int oracle_v1_init(void *states, int n, const D1Config *c, const D1Tables *t, uint64_t seed,
                   float *obs, float *mask);
int oracle_v1_step(void *states, int n, const D1Config *c, const D1Tables *t, const int64_t *actions,
                   int limit, float *obs, float *mask, float *out, const uint8_t *active);
int oracle_v1_heuristic(void *states, int n, const D1Config *c, const D1Tables *t, int64_t *actions);
/* Compact canonical view: rng.state, rng.inc, episode, hp, regen, blocks, player,
 * ticks, killed, pos[8], energy[8], hp[8]  (33 x int64 per env). */
int oracle_v1_compact(const void *states, int n, int64_t *rows);
/* Same compact view read from the reference's own State bytes (learn.cu:106-129). */
int oracle_v1_compact_from_reference(const void *ref_states, int n, int state_bytes, int64_t *rows);
int oracle_v1_semantic_test(const D1Config *c, const D1Tables *t);
/* Host all-pairs BFS distance table, the restatement of gpu-d1/scripts/learn_env.py:25-39. */
int oracle_distance_table(const uint8_t *floor, const int16_t *cells, int ncells, uint16_t *distance);


/* ---- spec (BASELINE task) ---- */
typedef struct {
    int hp, ac100, ev100, sh100, shield_limit, regen, gdr[2]; /* player */
    int min_monsters, max_monsters, min_mhp, max_mhp;        /* regular monsters per episode */
    int ogre, ogre_hp, ogre_min_damage;                       /* one sleeping ogre when ogre != 0 */
    int limit;                                                /* physical-turn deadline */
    int explore_milli, kill_milli, descend_milli, death_milli;
    D1Kind kinds[5];                                          /* rat, jackal, goblin, kobold, ogre */
} D1SpecConfig;
enum { OSPEC_MAXM = 11, OSPEC_OBS = 1832, OSPEC_ACTIONS = 12, OSPEC_OUT = 10, OSPEC_COMPACT = 56 };
/* The native LOS ray fan: n rays ending at (ex, ey) in the 8x8 quadrant, blocked
 * by any opaque cell in `blockers` (bit y*8+x). Must be set before any spec call. */
int oracle_set_rays(const int32_t *ex, const int32_t *ey, const uint64_t *blockers, int n);
/* LOS from `origin` on a u8[5600] floor map, in the reference's 17x17 mask format
 * (bit (dy+8)*17 + dx+8, 10 x u32), for pinning against native LOS tables. */
int oracle_los_mask(const uint8_t *floor, int origin, uint32_t *mask10);
/* Philox4x32-10 block (Salmon et al., SC'11): out = philox(ctr, key). */
void oracle_philox(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
int oracle_spec_state_bytes(void);
/* env ids are `first_env + i`; obs is float [n, 1832]; legal is u16 [n] bits. */
int oracle_spec_init(void *states, int n, const D1SpecConfig *c, uint64_t seed, int first_env, float *obs,
                     uint16_t *legal);
int oracle_spec_step(void *states, int n, const D1SpecConfig *c, const int64_t *actions, float *obs, uint16_t *legal,
                     float *out);
/* Observation and legal bits of states as they are (no step). */
int oracle_spec_observe(const void *states, int n, const D1SpecConfig *c, float *obs, uint16_t *legal);
/* 56 x int64 per env: ctr, env, episode, hp, regen, blocks, player, ticks, killed,
 * stairs, nmon, floor_seen, then pos[11], energy[11], hp[11], kind*2+awake [11].
 */
int oracle_spec_attack_dir(const void *state);
int oracle_spec_compact(const void *states, int n, int64_t *rows);
/* Copies the floor and remembered (viewed) bit planes, u32[n, 210] each. */
int oracle_spec_planes(const void *states, int n, uint32_t *floor, uint32_t *viewed);
/* Masked categorical sampling over 12 logits (see d1_oracle.c). */
int oracle_exp_nonpos(const float *x, int n, float *y);
int oracle_sample_actions(const float *logits, const uint16_t *legal, int n, uint64_t seed, uint64_t step,
                          int first_env, int64_t *action, float *logp);
/* Uniform draw over the legal actions (random baseline; see d1_oracle.c). */
int oracle_sample_uniform_legal(const uint16_t *legal, int nact, int n, uint64_t seed, uint64_t step, int first_env,
                                int64_t *action);
/* Conv-policy inputs: 63x63 u16 crops (pitch 64) under D4 element g (see d1_oracle.c). */
int oracle_spec_crop(const void *states, int n, int g, uint16_t *out);
/* Autoregressive verb (12) x target (9) sampling: verb_logits [n, 12],
 * target_logits [n, 2, 9]; outputs joint index, env action, log-prob, entropy. */
int oracle_sample_ar(const float *verb_logits, const float *target_logits, const uint16_t *legal, int n,
                     uint64_t seed, uint64_t step, int first_env, int64_t *joint, int64_t *env_action, float *logp,
                     float *entropy);

#ifdef __cplusplus
}
#endif
