// Masked categorical draw over 12 action logits, shared by the standalone head
// kernel and the GEMM epilogue that fuses the head: inverse CDF over
// exp(logit - max) in action order with one Philox uniform per (env, step)
// (purpose 1), or the first legal action of maximal logit when greedy. Only the
// portable exp, separately rounded adds and multiplies and compares are used,
// so the CPU oracle draws the same action from the same logits bit for bit.
#pragma once
#include <stdint.h>

#include "d1_math.cuh"
#include "d1_philox.cuh"

namespace d1 {

constexpr int SAMPLE_NACT = 12;

__device__ __forceinline__ void sample_masked(const float *l, uint32_t bits, uint32_t env, uint64_t seed,
                                              uint64_t step, bool greedy, int &action, float &logp) {
    float m = -3.402823466e38f;
#pragma unroll
    for (int j = 0; j < SAMPLE_NACT; j++)
        if ((bits >> j) & 1u) m = fmaxf(m, l[j]);
    float z[SAMPLE_NACT], total = 0.f;
#pragma unroll
    for (int j = 0; j < SAMPLE_NACT; j++) {
        z[j] = ((bits >> j) & 1u) ? d1_exp_nonpos(D1_ADD(l[j], -m)) : 0.f;
        total = D1_ADD(total, z[j]);
    }
    int a = -1, last = 0;
    if (greedy) {
#pragma unroll
        for (int j = 0; j < SAMPLE_NACT; j++)
            if (a < 0 && ((bits >> j) & 1u) && l[j] == m) a = j;
    } else {
        const uint4 o = policy_draw(env, seed, step, 1u);
        const float t = D1_MUL((float)(o.x >> 8) * (1.0f / 16777216.0f), total);
        float run = 0.f;
#pragma unroll
        for (int j = 0; j < SAMPLE_NACT; j++) {
            if ((bits >> j) & 1u) {
                last = j;
                run = D1_ADD(run, z[j]);
                if (a < 0 && t < run) a = j;
            }
        }
    }
    if (a < 0) a = last;
    float la = l[0];
#pragma unroll
    for (int j = 1; j < SAMPLE_NACT; j++)
        if (a == j) la = l[j];
    action = a;
    logp = (la - m) - logf(total);
}

}  // namespace d1
