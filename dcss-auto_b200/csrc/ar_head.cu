// Autoregressive verb x target head of the centered-map policy (BASELINE
// config 3): the type-first factorisation of the reference's ActionDistribution
// (gpu-d1/branches/autoregressive-actions-v1/scripts/tactical_models.py:8-30,
// Policy.raw :44-48) with 12 verbs and 9 targets.
//
// Input per env: the fp32 head-GEMM row hb[0..79] = [verb logits 0-11, value 12,
// direction pre-activation 13-76 (h . W_dir^T + b_dir), pad]. For each of the two
// directional verbs k (0 MOVE, 1 ATTACK) the conditional target logits are
//   t_k = W_t . tanh(pre + cond_k) + b_t          (cond_k = W_emb . emb_k)
// -- the reference's direction MLP on concat(h, type embedding), with the
// embedding's contribution to the first layer folded into cond_k.
//
// Masks (spec env legal bits: 0-7 passable, 8 wait, 9 rest allowed, 10 adjacent
// visible monster, 11 on stairs): MOVE targets 0-7 = passable directions;
// ATTACK targets 0-7 = passable directions and 8 = nearest, all only with bit
// 10; WAIT, REST, DESCEND = bits 8, 9, 11; verbs 5-11 are not offered on D:1.
// A directional verb is valid when any target is; a directional verb with no
// valid target keeps all nine (the reference's safe dummy conditional).
//
// Sampling: verb by inverse CDF with uniform word 0, then (directional verbs)
// target with word 1 of Philox(ctr = {lo(step), hi(step), hi(seed), 2},
// key = {env, lo(seed)}), using only the portable exp, separately rounded adds
// and multiplies and compares, so the CPU oracle draws the same (verb, target)
// from the same logits bit for bit. joint = 9*verb + target for directional
// verbs, else 16 + verb; the env receives MOVE t -> t, ATTACK t -> t (a bump)
// or 10 (nearest), WAIT 8, REST 9, DESCEND 11.
#include <cuda_bf16.h>

#include "d1_common.cuh"
#include "d1_math.cuh"
#include "d1_philox.cuh"

namespace d1 {
namespace ar {

constexpr int HB = 80, PRE = 64, NV = 12, NT = 9, ROWS = 128;
constexpr int HB_PITCH = HB + 1;

__constant__ int ENV_ACTION[28] = {0, 1, 2, 3, 4, 5, 6, 7, -1, 0, 1, 2, 3, 4,  5,  6,  7,  10,
                                   8, 9, 11, -1, -1, -1, -1, -1, -1, -1};

// Inverse-CDF draw over the `ok` entries of l[0..K) (the flat sampler's arithmetic).
template <int K>
__device__ __forceinline__ int draw(const float *l, uint32_t ok, float u, float &m, float &total) {
    m = -3.402823466e38f;
#pragma unroll
    for (int j = 0; j < K; j++)
        if ((ok >> j) & 1u) m = fmaxf(m, l[j]);
    float z[K];
    total = 0.f;
#pragma unroll
    for (int j = 0; j < K; j++) {
        z[j] = ((ok >> j) & 1u) ? d1_exp_nonpos(D1_ADD(l[j], -m)) : 0.f;
        total = D1_ADD(total, z[j]);
    }
    const float t = D1_MUL(u, total);
    int a = -1, last = 0;
    float run = 0.f;
#pragma unroll
    for (int j = 0; j < K; j++) {
        if ((ok >> j) & 1u) {
            last = j;
            run = D1_ADD(run, z[j]);
            if (a < 0 && t < run) a = j;
        }
    }
    return a < 0 ? last : a;
}

template <int K>
__device__ __forceinline__ float entropy(const float *l, uint32_t ok, float *p_out) {
    float m = -3.402823466e38f, total = 0.f;
#pragma unroll
    for (int j = 0; j < K; j++)
        if ((ok >> j) & 1u) m = fmaxf(m, l[j]);
#pragma unroll
    for (int j = 0; j < K; j++) total += ((ok >> j) & 1u) ? expf(l[j] - m) : 0.f;
    const float lz = logf(total);
    float h = 0.f;
#pragma unroll
    for (int j = 0; j < K; j++) {
        float p = 0.f;
        if ((ok >> j) & 1u) {
            const float lp = l[j] - m - lz;
            p = expf(lp);
            h -= p * lp;
        }
        if (p_out) p_out[j] = p;
    }
    return h;
}

struct Args {
    const float *hb;      // [n, 80]
    const float *cond;    // [2, 64]
    const float *wt;      // [9, 64]
    const float *bt;      // [9]
    const uint16_t *legal;
    int n, first_env;
    uint64_t seed, step;
    int64_t *joint, *env_action;
    float *logp, *value, *entropy;
    float *verb_logits, *target_logits;  // optional debug copies [n, 12], [n, 2, 9]
    int greedy;                          // argmax verb, then argmax target (ActionDistribution.greedy)
};
// First valid index of the maximal logit; `m` and `total` as draw<> computes them.
template <int K>
__device__ __forceinline__ int argmax(const float *l, uint32_t ok, float &m, float &total) {
    m = -3.402823466e38f;
#pragma unroll
    for (int j = 0; j < K; j++)
        if ((ok >> j) & 1u) m = fmaxf(m, l[j]);
    total = 0.f;
    int a = -1;
#pragma unroll
    for (int j = 0; j < K; j++) {
        if ((ok >> j) & 1u) {
            total = D1_ADD(total, d1_exp_nonpos(D1_ADD(l[j], -m)));
            if (a < 0 && l[j] == m) a = j;
        }
    }
    return a < 0 ? 0 : a;
}

// One thread per env; the block's 128 head rows are staged through shared
// memory with coalesced loads (pitch 81 floats: conflict-free row reads).
__global__ void __launch_bounds__(ROWS) ar_kernel(Args a) {
    __shared__ float hb_s[ROWS * HB_PITCH];
    __shared__ float wt_s[NT * PRE], cond_s[2 * PRE], bt_s[NT];
    for (int i = threadIdx.x; i < NT * PRE; i += ROWS) wt_s[i] = a.wt[i];
    for (int i = threadIdx.x; i < 2 * PRE; i += ROWS) cond_s[i] = a.cond[i];
    if (threadIdx.x < NT) bt_s[threadIdx.x] = a.bt[threadIdx.x];
    for (int r0 = blockIdx.x * ROWS; r0 < a.n; r0 += gridDim.x * ROWS) {
        __syncthreads();
        const int rows = min(ROWS, a.n - r0);
        for (int i = threadIdx.x; i < rows * HB; i += ROWS)
            hb_s[(i / HB) * HB_PITCH + i % HB] = a.hb[(size_t)r0 * HB + i];
        __syncthreads();
        const int row = r0 + threadIdx.x;
        if (threadIdx.x >= rows) continue;
        const float *h = hb_s + threadIdx.x * HB_PITCH;
        float vl[NV], tl[2][NT];
#pragma unroll
        for (int j = 0; j < NV; j++) vl[j] = h[j];
        const float value = h[NV];
#pragma unroll
        for (int k = 0; k < 2; k++) {
            float acc[NT];
#pragma unroll
            for (int t = 0; t < NT; t++) acc[t] = bt_s[t];
#pragma unroll 8
            for (int i = 0; i < PRE; i++) {
                const float x = tanhf(h[NV + 1 + i] + cond_s[k * PRE + i]);
#pragma unroll
                for (int t = 0; t < NT; t++) acc[t] = fmaf(wt_s[t * PRE + i], x, acc[t]);
            }
#pragma unroll
            for (int t = 0; t < NT; t++) tl[k][t] = acc[t];
        }
        // masks
        const uint32_t bits = a.legal[row];
        const uint32_t t_move = bits & 0xffu;
        const uint32_t t_att = ((bits >> 10) & 1u) ? ((bits & 0xffu) | 0x100u) : 0u;
        uint32_t vok = (t_move ? 1u : 0u) | (t_att ? 2u : 0u);
        vok |= ((bits >> 8) & 1u) << 2;
        vok |= ((bits >> 9) & 1u) << 3;
        vok |= ((bits >> 11) & 1u) << 4;
        const uint32_t safe0 = t_move ? t_move : 0x1ffu, safe1 = t_att ? t_att : 0x1ffu;
        // draws
        const uint4 o = policy_draw((uint32_t)(a.first_env + row), a.seed, a.step, 2u);
        const float uv = (float)(o.x >> 8) * (1.0f / 16777216.0f), ut = (float)(o.y >> 8) * (1.0f / 16777216.0f);
        float mv, sv;
        const int v = a.greedy ? argmax<NV>(vl, vok, mv, sv) : draw<NV>(vl, vok, uv, mv, sv);
        float lv = vl[0];
#pragma unroll
        for (int j = 1; j < NV; j++)
            if (v == j) lv = vl[j];
        float lp = (lv - mv) - logf(sv);
        int t = 0;
        if (v < 2) {
            float lt[NT];
#pragma unroll
            for (int j = 0; j < NT; j++) lt[j] = v == 0 ? tl[0][j] : tl[1][j];
            float mt, st;
            t = a.greedy ? argmax<NT>(lt, v == 0 ? safe0 : safe1, mt, st) : draw<NT>(lt, v == 0 ? safe0 : safe1, ut, mt, st);
            float lsel = lt[0];
#pragma unroll
            for (int j = 1; j < NT; j++)
                if (t == j) lsel = lt[j];
            lp += (lsel - mt) - logf(st);
        }
        const int joint = v < 2 ? 9 * v + t : 16 + v;
        if (a.joint) a.joint[row] = joint;
        if (a.env_action) a.env_action[row] = ENV_ACTION[joint];
        if (a.logp) a.logp[row] = lp;
        if (a.value) a.value[row] = value;
        if (a.entropy) {
            float pv[NV];
            float ent = entropy<NV>(vl, vok, pv);
            if (pv[0] > 0.f) ent += pv[0] * entropy<NT>(tl[0], safe0, nullptr);
            if (pv[1] > 0.f) ent += pv[1] * entropy<NT>(tl[1], safe1, nullptr);
            a.entropy[row] = ent;
        }
        if (a.verb_logits)
            for (int j = 0; j < NV; j++) a.verb_logits[(size_t)row * NV + j] = vl[j];
        if (a.target_logits)
            for (int k = 0; k < 2; k++)
                for (int j = 0; j < NT; j++) a.target_logits[((size_t)row * 2 + k) * NT + j] = tl[k][j];
    }
}

}  // namespace ar
}  // namespace d1

extern "C" int d1_ar_head_sample(const float *hb, int n, const float *cond, const float *wt, const float *bt,
                                 const uint16_t *legal, uint64_t seed, uint64_t step, int first_env, int64_t *joint,
                                 int64_t *env_action, float *logp, float *value, float *entropy, float *verb_logits,
                                 float *target_logits, void *stream) {
    using namespace d1::ar;
    if (n < 0 || !hb || !cond || !wt || !bt || !legal) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    Args a{hb, cond, wt, bt, legal, n, first_env, seed, step, joint, env_action, logp, value, entropy, verb_logits,
           target_logits, 0};
    int blocks = (n + ROWS - 1) / ROWS;
    if (blocks > 148 * 8) blocks = 148 * 8;
    ar_kernel<<<blocks, ROWS, 0, (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}

extern "C" int d1_ar_head_greedy(const float *hb, int n, const float *cond, const float *wt, const float *bt,
                                 const uint16_t *legal, int64_t *joint, int64_t *env_action, float *logp, float *value,
                                 void *stream) {
    using namespace d1::ar;
    if (n < 0 || !hb || !cond || !wt || !bt || !legal) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    Args a{hb, cond, wt, bt, legal, n, 0, 0, 0, joint, env_action, logp, value, nullptr, nullptr, nullptr, 1};
    int blocks = (n + ROWS - 1) / ROWS;
    if (blocks > 148 * 8) blocks = 148 * 8;
    ar_kernel<<<blocks, ROWS, 0, (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}
