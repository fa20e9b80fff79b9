/* libd1.so -- B200-native (sm_100a) batched D:1 environment step and PPO hot path.
 *
 * Plain C ABI: pointers and sizes only. Every buffer argument is DEVICE memory
 * owned by the caller (allocated once, reused every step); the library never
 * allocates on the hot path, never synchronises, and launches on the caller's
 * stream. Every entry point returns 0 on success or a nonzero code: a CUDA error
 * number from the launch, or one of the D1_ERR_* codes below.
 *
 * There is no host execution path: a call that asks for one (gpu == 0) returns
 * D1_ERR_NO_HOST_PATH instead of silently running on the CPU.
 */
#ifndef D1_H
#define D1_H
#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>

#ifdef __cplusplus
extern "C" {
#endif

#define D1_ERR_NO_HOST_PATH 9001 /* gpu == 0: this library has no CPU path */
#define D1_ERR_BAD_ARGUMENT 9002 /* size, count or pointer outside the supported range */
#define D1_ERR_TOO_LARGE 9003    /* request exceeds a fixed internal capacity */

/* Monster kind and run configuration, byte-identical to the reference structs
 * (gpu-d1/src/sim.h:61-67): 11 ints + 6 kinds of 4 ints = 140 bytes. */
typedef struct { int speed, damage, tohit, bypass; } D1Kind;
typedef struct {
    int count, player, hp, ac100, ev100, sh100, shield_limit, regen, repair, gdr[2];
    D1Kind kinds[6];
} D1Config;

/* Static map tables for the single fixture map, byte-identical to the reference
 * (gpu-d1/src/learn.cu:130-139, single-map build). All pointers are device memory:
 * floor u8[5600], cells i16[ncells] (reachable floor), index i16[5600],
 * distance u16[ncells * 5600] (row i = BFS distance from cells[i]). */
typedef struct {
    const uint8_t *floor;
    const int16_t *cells, *index;
    const uint16_t *distance;
    int ncells;
} D1Tables;

/* ======================================================================
 * Reference-compatible task ("v1"): the reference's default learn.cu build,
 * 9 actions (8 compass moves/attacks + wait), up to 8 monsters, 206 float
 * observations, 9 mask floats and 8 outcome floats per env.
 * Same names, argument meaning and error behaviour as the reference exports.
 * ====================================================================== */

#ifndef D1_ROUTE_LIBRARY  /* libd1_route.so exports learn_* with the route task (d1_route.h) */
/* Bytes of one env's opaque state row (reference: gpu-d1/src/learn.cu:644). */
int learn_state_bytes(void);
/* 206 (learn.cu:645). */
int learn_obs_size(void);
/* 9 (learn.cu:646). */
int learn_action_size(void);
/* 8 (learn.cu:647). */
int learn_out_size(void);
/* sizeof(D1Config) == 140 (learn.cu:648). */
int learn_config_bytes(void);
/* Seed env i with PCG32(mix(seed + i), i + 1), reset it and write its first
 * observation and mask (reference: learn.cu:649-660). state: u8[n, state_bytes];
 * obs f32[n, 206]; mask f32[n, 9]. `c` and `t` are host pointers to structs whose
 * table pointers are device memory. */
int learn_init(void *state, int n, const D1Config *c, const D1Tables *t, uint64_t seed, float *obs, float *mask,
               void *stream, int gpu);
/* One decision for every env: transition + auto-reset + observation
 * (reference: learn.cu:661-665). actions i64[n]; out f32[n, 8]. */
int learn_step(void *state, int n, const D1Config *c, const D1Tables *t, const int64_t *actions, int limit, float *obs,
               float *mask, float *out, void *stream, int gpu);
/* As learn_step, but envs with active[i] == false are left byte-for-byte untouched
 * (reference: learn.cu:666-670). */
int learn_step_active(void *state, int n, const D1Config *c, const D1Tables *t, const int64_t *actions, int limit,
                      float *obs, float *mask, float *out, const bool *active, void *stream, int gpu);
/* Pursuit baseline action per env (reference: learn.cu:671-675). */
int learn_heuristic(void *state, int n, const D1Config *c, const D1Tables *t, int64_t *actions, void *stream, int gpu);
/* Deterministic rule checks (move, last kill without retaliation, timeout,
 * death reset), run on the device (reference: learn.cu:677-707, which ran them on
 * the host). Returns 0 when all pass, else the number of the failed check. Blocks
 * until the check kernel finishes. */
int learn_semantic_test(const D1Config *c, const D1Tables *t);
#endif

/* Extras with no reference counterpart, used by the Python wrapper and tests. */
/* Canonical compact view of each env (33 x i64: rng.state, rng.inc, episode, hp,
 * regen, blocks, player, ticks, killed, pos[8], energy[8], hp[8]) -- the fields of
 * the reference State that determine every future step. rows: device i64[n, 33]. */
int learn_compact_state(const void *state, int n, int64_t *rows, void *stream);
/* All-pairs BFS distance table over 8-neighbour floor, one warp per source cell
 * (replaces the Python BFS of gpu-d1/scripts/learn_env.py:25-39).
 * floor u8[5600], cells i16[ncells] -> distance u16[ncells, 5600] (65535 = unreachable). */
int learn_distance_table(const uint8_t *floor, const int16_t *cells, int ncells, uint16_t *distance, void *stream);


/* ======================================================================
 * Route-cue task ("route"): the reference's selected fast build of its
 * headline PPO benchmark -- gpu-d1/src/learn.cu with LEARN_ENEMIES=40,
 * MULTI_MAP, SLEEP_ON, EXPLORE_REWARD (2 milli per newly seen floor cell),
 * MARK_WALLS, FRONTIER_RING_MEMORY_WALLS_OBS, KNOWN_FRONTIER,
 * FRONTIER_ROUTE_CUE_OBS and FAST_FRONTIER (gpu-d1/scripts/
 * run_ring_ablations.py:141-157; gpu-d1/PERFORMANCE.md:16). 9 actions, up to 40
 * sleeping monsters, 421 float observations (learn.cu:66-74: 9x9 floor and
 * monster-HP windows, 40 monster records, the player block, the 11x11
 * remembered ring, the nearest-frontier pointer through remembered floor and
 * an 8-way one-hot first step of the route to it), 9 mask and 8 outcome floats.
 * The exports of libd1_route.so carry the reference's learn_* names with these
 * semantics (the reference builds one learn.so per variant); libd1.so exports
 * the same entry points as d1_route_*.
 * ====================================================================== */

/* Multi-map tables, byte-identical to learn.cu:130-139 with MULTI_MAP (the
 * layout gpu-d1/scripts/learn_env_ring_multi.py:11-17 fills). Device pointers:
 * floor u8[n_maps * 5600] (16-byte aligned), cells i16[n_maps * 5600] (map m's
 * cells at m * 5600, -1 padded), index i16[n_maps * 5600], distance u16[sum of
 * ncells * 5600] (map m's rows from distance_offsets[m]), map_ncells
 * i32[n_maps], distance_offsets i32[n_maps]. map_filter: >= 0 plays that map
 * only, -1 draws a map per episode, -2 gives env i map i % n_maps on the first
 * episode (learn.cu:626-627). ncells is unused (the reference keeps it). */
typedef struct {
    const uint8_t *floor;
    const int16_t *cells, *index;
    const uint16_t *distance;
    int ncells;
    const int *map_ncells, *distance_offsets;
    int n_maps, map_filter;
} D1RouteTables;

/* Row bytes (13,312), 421, 9, 8, sizeof(D1Config), and the compact view's
 * width (171). Reference: learn.cu:644-648 of this build. */
int d1_route_state_bytes(void);
int d1_route_obs_size(void);
int d1_route_action_size(void);
int d1_route_out_size(void);
int d1_route_config_bytes(void);
int d1_route_compact_size(void);
/* learn_init of this build (learn.cu:649-660): env i is seeded
 * PCG(mix(seed + i), i + 1), placed and observed. obs f32[n, 421], mask
 * f32[n, 9]; legal (optional) receives the mask as u16 bits. */
int d1_route_init(void *state, int n, const D1Config *c, const D1RouteTables *t, uint64_t seed, float *obs,
                  float *mask, uint16_t *legal, void *stream);
/* learn_step / learn_step_active of this build (learn.cu:661-670): one
 * decision per env (actions i64[n]: 0-7 move/attack, 8 wait), outcomes
 * out f32[n, 8] = reward, done, clear, kills, hp, ticks, death, timeout, and
 * auto-reset; limit is the decision deadline (1024 in the reference wrapper).
 * active (optional, bool[n]) leaves inactive envs and their rows untouched. */
int d1_route_step(void *state, int n, const D1Config *c, const D1RouteTables *t, const int64_t *actions, int limit,
                  float *obs, float *mask, float *out, const bool *active, uint16_t *legal, void *stream);
/* learn_heuristic of this build (learn.cu:599-621, 671-675). */
int d1_route_heuristic(const void *state, int n, const D1Config *c, const D1RouteTables *t, int64_t *actions,
                       void *stream);
/* Extras with no reference counterpart. Observe rows as they are (the
 * reference's observe(), learn.cu:328-498), e.g. rows built by hand. Row
 * layout: u64 rng.state, rng.inc, episode; i32 hp, regen, blocks, player,
 * ticks, killed, map_id, frontier_count at byte 24; i16 pos[40] at 64,
 * energy[40] at 144, hp[40] at 224; u8 awake[40] at 304; the viewed plane
 * u32[210] at 352 (row y = words 3y..3y+2, bit x % 32 of word x / 32); the
 * map's floor plane u32[210] at 1216 (ignored here: the tables' floor is
 * used; the step reads the row's copy, written at reset); the frontier list
 * i16[5600] at 2112. */
int d1_route_observe(const void *state, int n, const D1Config *c, const D1RouteTables *t, float *obs, float *mask,
                     uint16_t *legal, void *stream);
/* Compact view, i64[n, 171]: rng.state, rng.inc, episode, hp, regen, blocks,
 * player, ticks, killed, map_id, frontier_count, pos[40], energy[40], hp[40],
 * awake[40] -- the reference State's fields apart from its three 5600-cell
 * arrays, which d1_route_memory exports: viewed u32[n, 210] bit planes and the
 * frontier list i16[n, 5600] (-1 past the count). Either output may be NULL. */
int d1_route_compact(const void *state, int n, int64_t *rows, void *stream);
int d1_route_memory(const void *state, int n, uint32_t *viewed, int16_t *frontier, void *stream);


/* ======================================================================
 * BASELINE task ("spec"): generated 80x70 rooms+corridors maps, a per-env
 * Philox4x32-10 stream keyed by the global env id, 12 semantic actions
 * (0-7 move/attack N,E,S,W,NE,SE,SW,NW; 8 wait; 9 rest; 10 attack the weakest
 * visible adjacent monster; 11 descend), 1832 bf16 observations (one-hot 15x15
 * LOS window x 8 channels + 32 scalars), a u16 legal-action bit mask and 10
 * outcome floats per env. No reference entry point exists for this task; its
 * rules reuse the reference's (see each kernel's comments).
 * ====================================================================== */
typedef struct {
    int hp, ac100, ev100, sh100, shield_limit, regen, gdr[2]; /* player */
    int min_monsters, max_monsters, min_mhp, max_mhp;        /* regular monsters per episode, <= 10 */
    int ogre, ogre_hp, ogre_min_damage;                       /* one sleeping ogre when ogre != 0 */
    int limit;                                                /* physical-turn deadline */
    int explore_milli, kill_milli, descend_milli, death_milli;
    D1Kind kinds[5];                                          /* rat, jackal, goblin, kobold, ogre */
} D1SpecConfig;

/* 7680 */
int d1_spec_state_bytes(void);
/* 1832 */
int d1_spec_obs_size(void);
/* 12 */
int d1_spec_action_size(void);
/* 10: reward, done, descended, killed, hp, turns, death, timeout, elapsed turns, invalid */
int d1_spec_out_size(void);
/* sizeof(D1SpecConfig) */
int d1_spec_config_bytes(void);
/* Register the LOS ray fan (a device array kept by the caller for the library's
 * lifetime, 16-byte aligned): n records of 4 x u32 {blocker mask bits 0-31,
 * bits 32-63 (bit y*8+x of the 8x8 quadrant), end-cell bit index ey*8+ex, 0}.
 * n <= 320. Must be called before any other d1_spec_* compute call. */
int d1_spec_set_rays(const void *rays, int n);
/* Generate env i's first map from Philox(key = {first_env + i, lo32(seed)}),
 * reset it and write its observation. state u8[n, 7680]; obs bf16[n, 1832];
 * legal u16[n]. */
int d1_spec_init(void *state, int n, const D1SpecConfig *c, uint64_t seed, int first_env, void *obs_bf16,
                 uint16_t *legal, void *stream);
/* One semantic decision per env with auto-reset; envs with active[i] == false
 * (when active is not NULL) are left untouched. actions i64[n]; out f32[n, 10]. */
int d1_spec_step(void *state, int n, const D1SpecConfig *c, const int64_t *actions, void *obs_bf16, uint16_t *legal,
                 float *out, const bool *active, void *stream);
/* d1_spec_init / d1_spec_step that also (or only) write the compact
 * observation: cobs u8[n, 320] -- the channel 0-7 of each of the 225 window
 * cells as a byte (zeros to byte 255), then the 32 scalars as bf16 at byte 256.
 * obs_bf16 and cobs may each be NULL. 320 B instead of 3,664 B per env: the
 * rollout buffer keeps this form and the update expands it
 * (d1_ppo_gather_cobs). */
int d1_spec_init_ex(void *state, int n, const D1SpecConfig *c, uint64_t seed, int first_env, void *obs_bf16,
                    void *cobs, uint16_t *legal, void *stream);
int d1_spec_step_ex(void *state, int n, const D1SpecConfig *c, const int64_t *actions, void *obs_bf16, void *cobs,
                    uint16_t *legal, float *out, const bool *active, void *stream);
/* d1_spec_step_ex with outcome value j of env i at out[i * out_env + j *
 * out_col] (out_env, out_col >= 1): out_col = B, out_env = 1 stores the outcomes
 * column by column ([10, B]), so that GAE reads rewards and dones as coalesced
 * planes. No reference counterpart. */
int d1_spec_step_strided(void *state, int n, const D1SpecConfig *c, const int64_t *actions, void *obs_bf16,
                         void *cobs, uint16_t *legal, float *out, int64_t out_env, int64_t out_col, const bool *active,
                         void *stream);
/* Observation, compact row and legal bits of rows as they are, without a step
 * (rows built or edited by hand, e.g. for rule tests). No reference counterpart
 * (the reference's observe() is internal to its step). Row layout: u64 draws
 * consumed; u32 env, seed lo, seed hi, episode; i32 hp, regen, blocks, player,
 * ticks, killed, stairs, nmon, floor_seen at byte 24; u16 LOS window rows[15]
 * at 64 (row dy+7, bit dx+7); i16 pos[16] at 128, energy[16] at 160, hp[16] at
 * 192; u8 kind[16] at 224, awake[16] at 240; the floor plane u32[210] at 256
 * and the remembered plane u32[210] at 1096 (row y = words 3y..3y+2). */
int d1_spec_observe(void *state, int n, const D1SpecConfig *c, void *obs_bf16, void *cobs, uint16_t *legal,
                    void *stream);
/* Canonical compact view, 56 x i64 per env: Philox draw count, env id, episode,
 * hp, regen, blocks, player, turns, killed, stairs, monster count, floor seen,
 * then pos[11], energy[11], hp[11], kind*2+awake[11]. */
int d1_spec_compact(const void *state, int n, int64_t *rows, void *stream);
/* Floor and remembered-cell bit planes, u32[n, 210] each (row y = words 3y..3y+2). */
int d1_spec_planes(const void *state, int n, uint32_t *floor, uint32_t *viewed, void *stream);
/* Map compiler: the LOS masks of one 80x70 map for all 5600 origins in the
 * reference's corpus format (gpu-d1/scripts/compile_corpus.py:67-85; 17x17
 * window, bit (dy+8)*17 + dx+8, 10 x u32 per origin). floor u8[5600] (nonzero =
 * floor), masks u32[5600, 10]; uses the ray fan of d1_spec_set_rays. */
int d1_los_table(const uint8_t *floor, uint32_t *masks, void *stream);
/* Conv-policy input: the egocentric 63x63 crop of each env
 * under D4 element g (0-7), u16 [n, 63, 64] (column 63 zero). Pixel (x, y) shows
 * the map cell at offset d4(g, x - 31, y - 31) from the player, d4 = rotation by
 * g % 4 quarter turns ((dx, dy) -> (dy, -dx)), then an x mirror for g >= 4 (the
 * sampling rule of gpu-d1/branches/vision15-centered-map-v1/src/fast_maps.cu:4-17).
 * Code bits 0-2: the observation's one-hot class (0 unknown, 1 wall, 2 remembered
 * floor, 3 visible floor, 4 stairs, 5 asleep, 6 awake, 7 ogre); bit 3: on the
 * map; bits 4-8: hp of the visible monster there. The conv stack expands it to
 * 10 channels (8 one-hot, hp / 32, on-map). d1_spec_step/init accept
 * obs_bf16 == NULL when only the crop (and legal bits) are wanted. */
int d1_spec_crop(const void *state, int n, int g, uint16_t *crop, void *stream);

/* ======================================================================
 * Policy and PPO kernels (no reference counterpart as kernels: the reference
 * runs these as PyTorch ops, gpu-d1/scripts/run_ring_ablations.py:209-223 and
 * :346-372).
 * ====================================================================== */
/* Head and sampler: for each row of h bf16[n, hidden] (hidden == 256) computes
 * logits = h . wh[0:12]^T + bh[0:12] and value = h . wh[12] + bh[12]
 * (wh bf16[13, hidden], bh f32[13]); when `action` is not NULL draws
 * action ~ softmax(logits over the legal bits of legal[row]) with one Philox
 * uniform keyed by (first_env + row, seed, step) and writes log p(action).
 * Any of action/logp/value/logits may be NULL. */
int d1_policy_head_sample(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                          const uint16_t *legal, uint64_t seed, uint64_t step, int first_env, int64_t *action,
                          float *logp, float *value, float *logits, void *stream);
/* Layer 2, the head and the draw in one persistent tcgen05 launch, from h1
 * bf16 [n, 256] (row pitch ldh elements, 16-byte aligned) as layer 1 leaves
 * it: h2 = relu(h1 W2^T + b2) (w2 bf16 [256, 256]), logits and value = h2
 * Wh^T + bh (wh bf16 [13, 256]), then the masked draw of
 * d1_policy_head_sample (same Philox counter: first_env + row, seed, step;
 * the step is *step_dev when step_dev is not NULL, read when the kernel runs).
 * action NULL: value (and logits) only. Replaces d1_gemm (layer 2) +
 * d1_policy_head_sample, the reference's policy forward and
 * Categorical(logits).sample() (gpu-d1/scripts/run_ring_ablations.py:350). */
int d1_policy_tail_sample(const void *h1, int n, int ldh, const void *w2, const float *b2, const void *wh,
                          const float *bh, const uint16_t *legal, uint64_t seed, uint64_t step,
                          const int64_t *step_dev, int first_env, int64_t *action, float *logp, float *value,
                          float *logits, void *stream);
/* Nonzero when a d1_policy_tail_sample launch gave up on a bounded wait;
 * reading clears it. Synchronises the device. */
int d1_policy_tail_error(void);
/* As d1_policy_head_sample with the step read from device memory (*step_dev)
 * when the kernel runs, so a captured CUDA graph that also advances the counter
 * (d1_counter_add) draws fresh uniforms on every replay. */
int d1_policy_head_sample_dev(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                              const uint16_t *legal, uint64_t seed, const int64_t *step_dev, int first_env,
                              int64_t *action, float *logp, float *value, float *logits, void *stream);
/* Greedy variant of the head (the reference's dist.probs.argmax(-1) evaluation
 * mode, gpu-d1/scripts/train_clear.py:57): action = the first legal action of
 * maximal logit; logp and value as in d1_policy_head_sample (may be NULL). */
int d1_policy_head_greedy(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                          const uint16_t *legal, int64_t *action, float *logp, float *value, void *stream);
/* Tensor-core dense layer (tcgen05 + TMA): C = act(A . B^T + bias) [* (mask > 0)] with
 * A bf16[M, K] (row pitch lda), B bf16[N, K] (row pitch ldb), fp32 accumulation,
 * act = ReLU when relu != 0; when mask (bf16 [M, ldm]) is given, entries whose mask
 * value is not positive are zeroed (the ReLU derivative of the backward pass).
 * Writes any of: c bf16[M, ldc] row-major, ct
 * bf16[N, ldct] (C transposed), cf fp32 (row-major, pitch ldcf, one [M, ldcf]
 * slab per K split). splits > 1 splits K across CTAs and requires c == ct ==
 * NULL; the number of slabs written is d1_gemm_splits(K, splits). Bases and
 * pitches must be 16-byte aligned (TMA). When no transposed output is asked
 * for, N > 128 and each split spans at least 512 of K, the call runs the 2-SM
 * pair kernel (d1_gemm_pair); otherwise one CTA per 128 x 256 tile
 * (d1_gemm_single). Both give bit-identical results. */
int d1_gemm(const void *a, int lda, const void *b, int ldb, int M, int N, int K, const float *bias, int relu,
            const void *mask, int ldm, void *c, int ldc, void *ct, int ldct, float *cf, int ldcf, int splits,
            void *stream);
/* Number of fp32 slabs a split-K call writes for (K, splits); D1_ERR_BAD_ARGUMENT
 * when K <= 0. */
int d1_gemm_splits(int K, int splits);
/* As d1_gemm with B stored [K, N] (row pitch ldb >= N, N contiguous: "MN-major")
 * instead of [N, K], so a weight gradient A^T-style product can read a row-major
 * activation matrix without a transposed copy. Outputs c (bf16) and/or cf
 * (fp32 split-K slabs) only. */
int d1_gemm_bkn(const void *a, int lda, const void *b_kn, int ldb, int M, int N, int K, const float *bias, int relu,
                void *c, int ldc, float *cf, int ldcf, int splits, void *stream);
/* Gathered operands (TMA tile::gather4): with a_rows, row m of A is row
 * a_rows[m] of the K-major table a [a_table_rows, K]; with b_rows (b_mn = 1),
 * K-row k of B is row b_rows[k] of the table b [b_table_rows, N]. Other
 * arguments as d1_gemm_ex (no transposed output). Measured for the PPO
 * minibatch (rows of the rollout buffer): no faster than gathering X once into
 * an L2-resident copy for layer 1, and 4x slower for dW1, whose tiles re-read
 * the rows piecewise from HBM -- the update therefore gathers X once. */
int d1_gemm_rows(const void *a, int lda, int a_mn, const int64_t *a_rows, int a_table_rows, const void *b, int ldb,
                 int b_mn, const int64_t *b_rows, int b_table_rows, int M, int N, int K, const float *bias, int relu,
                 const void *mask, int ldm, void *c, int ldc, float *cf, int ldcf, int splits, void *stream);
/* 2-SM form of d1_gemm_ex: each cluster of two CTAs computes a 256 x 256 tile
 * with tcgen05.mma.cta_group::2, each CTA streaming its 128 rows of A and its
 * half of B, so an SM reads 32 KB per 64-deep K block instead of 48 KB. Same
 * arguments as d1_gemm_ex without the transposed output. */
int d1_gemm_pair(const void *a, int lda, int a_mn, const void *b, int ldb, int b_mn, int M, int N, int K,
                 const float *bias, int relu, const void *mask, int ldm, void *c, int ldc, float *cf, int ldcf,
                 int splits, void *stream);
/* Pair-kernel products with one operand expanded from compact observation rows
 * (d1_spec_step_ex's 320-byte cobs rows) inside the kernel, so the one-hot
 * matrix never exists in memory. Row r of the expanded matrix X is the
 * 1832-feature one-hot observation of compact row idx[r] (idx == NULL: row r)
 * followed by the ones column (1, 0, ..., 0) at 1832..1839.
 * d1_gemm_cobs_a: c[M, N] (bf16) = act(X[:, :1832] . B^T + bias), B [N, 1832]
 * K-major (the policy's first layer on a minibatch).
 * d1_gemm_cobs_b: fp32 split-K slabs of A^T-form products A . X[:, :N] with A
 * stored [K, M] (M contiguous, e.g. dh1 [samples, 256]) and the K samples'
 * rows of X, N <= 1840 (the weight and bias gradient of that layer).
 * Bit-identical to d1_gemm_ex on the expanded matrix. */
int d1_gemm_cobs_a(const void *cobs, const int64_t *idx, int M, const void *b, int ldb, int N, const float *bias,
                   int relu, void *c, int ldc, void *stream);
int d1_gemm_cobs_b(const void *a, int lda, const void *cobs, const int64_t *idx, int M, int N, int K, float *cf,
                   int ldcf, int splits, void *stream);
/* d1_gemm_ex on the one-CTA kernel whatever the shape (the pair kernel's
 * comparison point). */
int d1_gemm_single(const void *a, int lda, int a_mn, const void *b, int ldb, int b_mn, int M, int N, int K,
                   const float *bias, int relu, const void *mask, int ldm, void *c, int ldc, void *ct, int ldct,
                   float *cf, int ldcf, int splits, void *stream);
/* The general form: a_mn / b_mn select A stored [K, M] / B stored [K, N]
 * (M / N contiguous) instead of [M, K] / [N, K]; other arguments as d1_gemm. */
int d1_gemm_ex(const void *a, int lda, int a_mn, const void *b, int ldb, int b_mn, int M, int N, int K,
               const float *bias, int relu, const void *mask, int ldm, void *c, int ldc, void *ct, int ldct, float *cf,
               int ldcf, int splits, void *stream);
/* The policy's second layer with the head and sampler fused into the GEMM
 * epilogue: h = ReLU(A . B^T + bias) with N = 256 (B bf16 [256, K]), never
 * stored; logits/value = bf16(h) . wh^T + bh (wh bf16 [13, 256], bh f32 [13]);
 * then the draw of d1_policy_head_sample (same stream keys and arithmetic).
 * Any of action/logp/value/logits may be NULL (value-only for bootstrapping). */
int d1_gemm_head_sample(const void *a, int lda, const void *b, int ldb, int M, int K, const float *bias,
                        const void *wh_bf16, const float *bh, const uint16_t *legal, uint64_t seed, uint64_t step,
                        int first_env, int64_t *action, float *logp, float *value, float *logits, void *stream);
/* No counterpart in the reference. The split-K weight-gradient product
 * out = A . B^T (fp32 [M, ldo], A bf16 [M, K], B bf16 [N, K], same operand rules as
 * d1_gemm) for callers that cannot allocate device memory (a host framework that
 * owns every byte of HBM, a plugin that must not call cudaMalloc after start-up):
 * the partial-product slabs live in a fixed 16 MiB array inside the library,
 * reserved on every GPU that loads it until the process exits, so the call
 * allocates nothing. Limit: d1_gemm_splits(K, splits) * M * round_up(N, 4) floats
 * <= 4 Mi, else D1_ERR_TOO_LARGE. The first call on a device looks up the array's
 * device address; make that first call before capturing any stream. All calls
 * share the array: calls that overlap on the GPU race and must be serialised by
 * the caller. */
int d1_gemm_wgrad_noalloc(const void *a, int lda, const void *b, int ldb, int M, int N, int K, float *out, int ldo,
                          int splits, void *stream);
/* Conv encoder of the centered-map policy on tcgen05 (the
 * reference runs it as torch Conv2d layers, vision15-centered-map-v1/scripts/
 * tactical_models.py:11-13): three 3x3 stride-2 convs with ReLU,
 * 10 -> 32 -> 64 -> 64 channels, 63x63 -> 31x31 -> 15x15 -> 7x7.
 * Layer 1 reads the u16 crops of d1_spec_crop; layers 2 and 3 read the previous
 * layer's output, written by it in the layer's own input layout
 * (d1_conv_in_bytes(layer) bytes per env); layer 3 writes the flattened NHWC
 * FC input, bf16 [n, 3136] (feature (y*7 + x)*64 + channel). w_packed is the
 * layer's weight in operand layout (d1_conv_weight_bytes(layer) bytes, made by
 * d1_conv_pack_weights from torch's fp32 [Cout, Cin, 3, 3]); bias f32 [Cout].
 * Buffers 16-byte aligned. d1_conv_in_bytes(4) is the FC input row (6272 B). */
int d1_conv_in_bytes(int layer);
int d1_conv_weight_bytes(int layer);
int d1_conv_pack_weights(int layer, const float *w, void *packed, void *stream);
int d1_conv_layer(int layer, const void *in, int n, const void *w_packed, const float *bias, void *out, void *stream);
/* Nonzero when a conv pipeline wait expired; reading clears it. Synchronises. */
int d1_conv_error(void);
/* Autoregressive verb x target head (the reference's
 * ActionDistribution, autoregressive-actions-v1/scripts/tactical_models.py:8-30,
 * with 12 verbs and 9 targets). hb f32 [n, 80] = head GEMM rows [verb logits
 * 0-11, value 12, direction pre-activation 13-76, pad]; cond f32 [2, 64] (the
 * type embedding's first-layer term for MOVE and ATTACK); wt f32 [9, 64], bt f32
 * [9]. Draws the verb, then the target of a directional verb, from Philox words
 * 0 and 1 keyed by (first_env + row, seed, step), and writes the joint index
 * (9*verb + target for MOVE/ATTACK, else 16 + verb), the env action, log p,
 * value and, when given, the entropy and the verb [n, 12] / target [n, 2, 9]
 * logits. Any output may be NULL. */
int d1_ar_head_sample(const float *hb, int n, const float *cond, const float *wt, const float *bt,
                      const uint16_t *legal, uint64_t seed, uint64_t step, int first_env, int64_t *joint,
                      int64_t *env_action, float *logp, float *value, float *entropy, float *verb_logits,
                      float *target_logits, void *stream);
/* Greedy variant (ActionDistribution.greedy, tactical_models.py:22-25): argmax
 * verb, then the argmax target of a directional verb. */
int d1_ar_head_greedy(const float *hb, int n, const float *cond, const float *wt, const float *bt,
                      const uint16_t *legal, int64_t *joint, int64_t *env_action, float *logp, float *value,
                      void *stream);

/* Evaluation and observation wrappers (reference: gpu-d1/scripts/train_clear.py:42-76,
 * run_ring_ablations.py:231-267, vision15-centered-map-v1/scripts/frame_stack.py). */
/* One step of the evaluation bookkeeping for envs with active[i]: returns[i] +=
 * out[i, 0]; when out[i, 1] > 0 the first tcols outcome columns go to
 * terminal[i] and active[i] becomes false. out f32 [n, out_cols]. */
int d1_eval_accumulate(const float *out, int out_cols, int n, bool *active, float *returns, float *terminal,
                       int tcols, void *stream);
/* Random baseline: a uniform draw over the set bits 0..nact-1 of legal[i], the
 * k-th set bit with k = mulhi(word, count), word = Philox word 0 of
 * (ctr = {lo(step), hi(step), hi(seed), 3}, key = {first_env + i, lo(seed)});
 * -1 when no bit is set. */
int d1_sample_uniform_legal(const uint16_t *legal, int nact, int n, uint64_t seed, uint64_t step, int first_env,
                            int64_t *action, void *stream);
/* Frame stack of `frames` observations per env, stack [n, frames, row_bytes]
 * (oldest first), obs [n, row_bytes], row_bytes % 4 == 0. With out == NULL every
 * frame becomes obs (reset). Otherwise frames shift one slot older and obs is
 * appended, except that envs whose episode ended (out[i, 1] > 0, and active[i]
 * when active is given) get obs in every frame. */
int d1_frame_stack(void *stack, const void *obs, int row_bytes, int frames, int n, const float *out, int out_cols,
                   const bool *active, void *stream);
/* Per-episode D4 camera augmentation of the spec observation (reference:
 * gpu-d1/branches/vision15-symmetry-v1/scripts/symmetry.py:19-102, D4 and
 * EpisodeSymmetry). groups u8[n] in 0..7: mirror x when g >= 4, then g % 4
 * quarter turns (x, y) -> (-y, x).
 * d1_spec_d4_observe: camera observation and legal bits of the world ones
 * (cells permuted, coordinate scalars rotated with the reference's scale and
 * offset tables, legal bits 0-7 permuted); obs_out may equal obs (in place),
 * both 16-byte aligned.
 * d1_spec_d4_actions: camera action -> world action (directions 0-7 permuted,
 * others unchanged; the reference's to_world).
 * d1_spec_d4_draw: groups[i] = Philox word 0 >> 29 of (ctr = {lo(step),
 * hi(step), hi(seed), 4}, key = {first_env + i, lo(seed)}) for every env when
 * out == NULL, else only where the episode ended (out[i, 1] > 0, and active[i]
 * when given). */
int d1_spec_d4_observe(const void *obs_bf16, const uint16_t *legal, const uint8_t *groups, int n, void *obs_out_bf16,
                       uint16_t *legal_out, void *stream);
int d1_spec_d4_actions(const int64_t *camera_actions, const uint8_t *groups, int n, int64_t *world_actions,
                       void *stream);
int d1_spec_d4_draw(uint8_t *groups, int n, const float *out, int out_cols, const bool *active, uint64_t seed,
                    uint64_t step, int first_env, void *stream);
/* Nonzero when a GEMM pipeline wait expired (the kernel then skipped its work
 * and freed its tensor memory); reading clears it. Synchronises the device. */
int d1_gemm_error(void);

/* GAE over a rollout (reference: gpu-d1/scripts/run_ring_ablations.py:354-361):
 * reward/done f32 read at [t * r_step + b * r_env] (the env's outcome rows),
 * value f32 [T + 1, B] (row T = bootstrap), outputs adv/ret f32 [T, B]. When
 * `stats` (double[2]) is given, sum(adv) and sum(adv^2) are added to it (the
 * advantage-normalisation statistics; all-reduced across ranks by the caller).
 * mode 0 replays the reference's per-step op order exactly; mode 1 is the
 * segmented scan over time (each thread composes a run of steps in registers,
 * the runs of an env are combined across the 8 warps of a block; within 1e-5
 * relative). The sums are deterministic for a given device (block partials
 * added in block order through a fixed array in the library, so calls on one
 * device must not overlap); with stats in mode 0, B is at most 16,777,216,
 * else D1_ERR_TOO_LARGE. */
int d1_gae(const float *reward, const float *done, int64_t r_step, int64_t r_env, const float *value, int T, int B,
           float gamma, float lambda, float *adv, float *ret, double *stats, int mode, void *stream);
/* Gather + expand of compact observations (d1_spec_step_ex's cobs rows, 320 B
 * each): x[i] (bf16, row pitch ldx) = the 1832-feature one-hot observation of
 * row idx[i], plus the ones column (1, 0, ..., 0) at 1832 with ones_col
 * (ldx >= 1840 then). Equal bit for bit to the one-hot observation the env
 * writes for the same step. */
int d1_ppo_gather_cobs(const void *cobs, const int64_t *idx, int n, void *x, int ldx, int ones_col, void *stream);
/* Length of one block partial written by d1_ppo_loss: dWh[13*256], dbh[13], db2[256],
 * then 8 loss terms (sum pg, sum vf, sum entropy, clipped count, sum approx-kl, 0, 0, 0). */
int d1_ppo_loss_part_len(void);
/* Fused head forward, PPO loss and backward to the last hidden layer for a
 * minibatch of n rows: h2 bf16 [n, 256] (minibatch order), rollout arrays indexed
 * through idx (legal u16, action i64, old_logp/adv/ret/old_value f32), adv
 * normalised with adv_stats (sum, sum of squares over adv_count samples, torch's
 * unbiased std). Loss = mean(pg) + vf_coef*mean(vf) - ent_coef*mean(entropy) with
 * ratio clip `clip` and value clip `vclip` (<= 0: plain squared error). Writes
 * dh2 bf16 [n, 256] and dh2t bf16 [256, ldt] (either may be NULL) and `blocks`
 * partials of d1_ppo_loss_part_len() floats to `part`. */
int d1_ppo_loss(const void *h2, const void *wh, const float *bh, const int64_t *idx, const uint16_t *legal,
                const int64_t *action, const float *old_logp, const float *adv, const float *ret,
                const float *old_value, const double *adv_stats, double adv_count, int n, float clip, float vclip,
                float vf_coef, float ent_coef, void *dh2, void *dh2t, int ldt, float *part, int blocks,
                void *stream);
/* The tail of a minibatch in one tcgen05 launch, from h1 bf16 [n, 256] (the
 * first hidden layer as stored) to dh1: layer 2 (w2 bf16 [256, 256], b2), the
 * head (wh bf16 [13, 256], bh), the loss and dhead exactly as d1_ppo_loss
 * computes them (same rollout arrays, advantage statistics and coefficients),
 * dh2 = relu'(h2) * (dhead Wh) and dh1 = relu'(h1) * (dh2 W2). Writes dh2 and
 * dh1 bf16 [n, 256] (16-byte aligned) and d1_ppo_tail_blocks(n) block partials
 * in d1_ppo_loss's layout (dWh, dbh, db2, loss terms) to `part`. Replaces the
 * layer-2 GEMM, d1_ppo_loss and the dh1 GEMM of the unfused update (the
 * reference's update: gpu-d1/scripts/run_ring_ablations.py:363-372). */
int d1_ppo_tail(const void *h1, const void *w2, const float *b2, const void *wh, const float *bh, const int64_t *idx,
                const uint16_t *legal, const int64_t *action, const float *old_logp, const float *adv,
                const float *ret, const float *old_value, const double *adv_stats, double adv_count, int n,
                float clip, float vclip, float vf_coef, float ent_coef, void *dh2, void *dh1, float *part,
                void *stream);
/* Block partials d1_ppo_tail writes for n rows (one per 128 rows). */
int d1_ppo_tail_blocks(int n);
/* Nonzero when a d1_ppo_tail launch gave up on a bounded wait (it then skipped
 * the rest of its work and freed its tensor memory); reading clears it.
 * Synchronises the device. */
int d1_ppo_tail_error(void);
/* out[i] = sum_s slabs[s * count + i] (split-K partial products, deterministic order). */
int d1_reduce_slabs(const float *slabs, int splits, int64_t count, float *out, void *stream);
/* A parameter segment whose bf16 compute copy the optimizer refreshes: elements
 * [offset, offset + count) form a [rows, cols] matrix; bf16 receives the same
 * layout and bf16_t (when not NULL) its transpose. */
typedef struct { int64_t offset, count; int rows, cols; void *bf16, *bf16_t; } D1AdamSegment;
/* The minibatch order of one epoch: perm[i] (i < n) is a keyed bijection of
 * [0, n) -- an alternating Feistel network over the smallest power of two >= n
 * with cycle walking -- keyed by `seed` and the count *epoch read on the device
 * (advance it with d1_counter_add between epochs, so that a captured epoch draws
 * a new order on every replay). Replaces the reference's per-epoch
 * torch.randperm(T*B, device='cuda') (gpu-d1/scripts/run_ring_ablations.py:364)
 * with one pass and no sort. n <= 2^40. */
int d1_ppo_permute(int64_t *perm, int64_t n, uint64_t seed, const int64_t *epoch, void *stream);
/* *counter += delta on the device (the optimizer's step count lives on the
 * device so that a captured CUDA graph of many updates stays correct). */
int d1_counter_add(int64_t *counter, int64_t delta, void *stream);
/* End of a minibatch in two launches: (1) reduce the gradient's partial
 * products into the flat gradient, with per-block sums of squares; (2) a
 * torch.optim.Adam step (eps outside the sqrt, bias correction with the device
 * step count) on the fp32 master params after scaling the gradient by
 * min(1, max_norm / (||grad|| + 1e-6)) (torch.nn.utils.clip_grad_norm_;
 * max_norm <= 0 disables), refreshing the bf16 copies of `segs` (host array of
 * nseg <= 8); *step advances by one on the device (the step taken is the old
 * *step + 1). param, grad, m and v are 16-byte aligned. Job j
 * (njobs <= 4): element e < rows * cols_in of partial p < nsrc is
 * src[p * stride + e]; element (r, c) of the sum goes to
 * dst[r * cols_out + c] when c < cols_out, to dst_extra[r] when c == cols_out
 * (a bias carried as an extra product column), else nowhere; in_norm = 0 keeps
 * a job (loss statistics) out of the gradient norm. Sums are deterministic
 * (fixed partial and block order). With njobs == 0 the gradient is taken as it
 * is in `grad` (after a cross-rank all-reduce). The block partials live in a
 * file-scope array: calls must not overlap on one device. */
typedef struct {
    const float *src;
    int64_t stride;
    int nsrc, rows, cols_in, cols_out, in_norm;
    float *dst, *dst_extra;
} D1GradJob;
int d1_ppo_step(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step, const D1AdamSegment *segs,
                int nseg, void *stream);
/* Step (1) of d1_ppo_step alone (multi-GPU: reduce, all-reduce, then
 * d1_ppo_step with no jobs). */
int d1_grad_reduce(const D1GradJob *jobs, int njobs, void *stream);
/* d1_ppo_step for data-parallel ranks with the gradient all-reduce done through
 * peer memory instead of a collective library: (1) the reduction writes this
 * rank's gradient into half (epoch & 1) of its exchange buffer xbufs[rank]
 * (epoch = *step + 1) and its last block stores flags[p][rank] = epoch on every
 * peer p (system-scope release); (2) every block waits, bounded, for
 * flags[rank][p] >= epoch from each peer, then sums a contiguous range of all
 * ranks' halves in rank order (peer loads over NVLink), divides by world and
 * writes `grad` -- the same bits on every rank -- with its sums of squares;
 * (3) the Adam step of d1_ppo_step. xbufs[p] / flags[p] are rank p's exchange buffer
 * (2 * xstride floats, xstride >= total, a multiple of 4) and flag array
 * (world u64) as mapped in this process (d1_peer_open); world <= 8. The two
 * halves make a rank's next write safe: before it, every peer has flagged the
 * epoch in between, which it does only after reading. Each wait polls a flag
 * at most wait_limit times (0: 2^24 polls, about a second); a wait that runs
 * out records d1_peer_error and the step then leaves param, m, v, the bf16
 * copies and *step unchanged. */
int d1_ppo_step_peer(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                     float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                     const D1AdamSegment *segs, int nseg, void *const *xbufs, void *const *flags, int64_t xstride,
                     int world, int rank, unsigned wait_limit, void *stream);
/* d1_ppo_step_peer over NVLink SHARP (NVLS): the exchange buffers are bound to
 * one multicast object whose address is `mc` (the same offset maps every
 * rank's buffer), and after the bounded flag waits each block reads its range
 * of the summed gradient with multimem.ld_reduce -- the NVSwitch adds the
 * ranks' values -- instead of reading the N - 1 peer buffers. Publishing,
 * flags, the skip-on-timeout rule and Adam are those of d1_ppo_step_peer. */
int d1_ppo_step_nvls(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                     float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                     const D1AdamSegment *segs, int nseg, void *const *xbufs, void *const *flags, int64_t xstride,
                     const void *mc, int world, int rank, unsigned wait_limit, void *stream);
/* d1_ppo_step_peer with a two-phase exchange, for more ranks: rank j owns
 * slice j of the flat gradient (`slice` elements, a multiple of 4, slice *
 * world >= total). (1) The reduction stores this rank's part of every slice j
 * straight into rank j's inbox, slot [epoch & 1][rank] (peer stores), and
 * raises flags[p][rank] = epoch on every peer; (2) each rank waits for all of
 * its inbox's flags, sums its slice over the ranks in rank order, divides by
 * world and stores the result into slot [epoch & 1][rank] of every rank's
 * gather area, then raises flags[p][8 + rank]; (3) each rank waits for those
 * flags and copies the gathered slices into `grad` (and its sums of squares);
 * (4) Adam. A rank moves 2 (world - 1) / world of the gradient over NVLink
 * instead of reading (world - 1) whole copies. xbufs[p]: rank p's buffer of
 * 4 * world * slice floats (inbox [2][world][slice], then gather
 * [2][world][slice]); flags[p]: its 16 u64 flags. Same bounded waits and
 * failure behaviour as d1_ppo_step_peer; the same bits as the one-shot and
 * NCCL exchanges. Measured slower than the one-shot exchange on 2 and 8
 * B200s (the added flag round outweighs the smaller transfer). No reference
 * counterpart. */
int d1_ppo_step_peer2(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                      float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                      const D1AdamSegment *segs, int nseg, void *const *xbufs, void *const *flags, int64_t slice,
                      int world, int rank, unsigned wait_limit, void *stream);
/* Exchange-buffer set-up through CUDA IPC (not on the hot path): allocate
 * `bytes` of zeroed device memory and its handle (d1_peer_handle_bytes()
 * bytes), map another process's buffer from its handle, unmap, free. */
int d1_peer_handle_bytes(void);
int d1_peer_alloc(int64_t bytes, void **ptr, void *handle);
int d1_peer_open(const void *handle, void **ptr);
int d1_peer_close(void *ptr);
int d1_peer_free(void *ptr);
/* Nonzero when a peer all-reduce gave up waiting for a peer since the last
 * call (that step changed no parameter); reading clears it. Synchronises the
 * device. */
int d1_peer_error(void);
/* Gather x[i, 0..F) = obs[idx[i], 0..F) into rows of pitch ldx; with ones_col,
 * columns F..F+7 of every row are (1, 0, ..., 0), so that a weight-gradient
 * product dh^T x also yields the bias gradient (column sums of dh) in its
 * column F. F and ldx multiples of 8, ldx >= F + 8 with ones_col. */
int d1_ppo_gather_x(const void *obs, int F, const int64_t *idx, int n, void *x, int ldx, int ones_col,
                    void *stream);

#ifdef __cplusplus
}
#endif
#endif /* D1_H */
