// Policy head and action sampler (sm_100a).
//
// For each env row: 13 dot products of the last hidden layer (bf16, width 256)
// with the head weights -- 12 action logits and the value -- then the masked
// categorical draw of run_ring_ablations.py:221-223/350-351 (illegal logits
// excluded, exactly like masked_fill(-1e9)): inverse-CDF sampling over
// exp(logit - max) in action order with one Philox uniform per (env, step).
// The draw uses only the portable exp of d1_math.cuh, adds and compares, so a
// CPU restatement picks the same action from the same logits bit for bit.
//
// Head weights live in shared memory; partial dot products are combined with
// butterfly shuffles inside groups of eight lanes.
#include <cuda_bf16.h>

#include "d1_common.cuh"
#include "d1_math.cuh"
#include "d1_philox.cuh"

namespace d1 {
namespace head {

constexpr int HID = 256, NOUT = 13, NACT = 12, WARPS = 8;

// Uniform in [0, 1) with 24 random bits: word 0 of
// Philox(ctr = {lo(step), hi(step), hi(seed), 1}, key = {env, lo(seed)}).
__device__ __forceinline__ float sample_uniform(uint32_t env, uint64_t seed, uint64_t step) {
    const uint4 o = policy_draw(env, seed, step, 1u);
    return (float)(o.x >> 8) * (1.0f / 16777216.0f);
}

// Four rows per warp: lanes 8r..8r+7 share row r. Lane part p (0..7) loads the
// 16-byte chunks q = 8c + p (c = 0..3), so each group of eight lanes reads 128
// contiguous bytes per instruction; the head weights are stored with one float
// of padding per 32 to keep those eight lanes on distinct banks.
__device__ __forceinline__ int wpad(int e) { return e + (e >> 5); }
constexpr int WROW = HID + HID / 32;

__global__ void __launch_bounds__(WARPS * 32)
    head_sample_kernel(const __nv_bfloat16 *__restrict__ h, int n, const __nv_bfloat16 *__restrict__ wh,
                       const float *__restrict__ bh, const uint16_t *__restrict__ legal, uint64_t seed, uint64_t step,
                       int first_env, int64_t *__restrict__ action, float *__restrict__ logp,
                       float *__restrict__ value, float *__restrict__ logits_out, int greedy) {
    __shared__ float w_s[NOUT * WROW];
    __shared__ float b_s[NOUT];
    for (int i = threadIdx.x; i < NOUT * HID; i += blockDim.x)
        w_s[(i / HID) * WROW + wpad(i % HID)] = __bfloat162float(wh[i]);
    if (threadIdx.x < NOUT) b_s[threadIdx.x] = bh[threadIdx.x];
    __syncthreads();
    const int lane = threadIdx.x & 31, part = lane & 7, sub = lane >> 3;
    const int groups_total = gridDim.x * WARPS * 4;
    for (int row0 = (blockIdx.x * WARPS + (threadIdx.x >> 5)) * 4; row0 < n; row0 += groups_total) {
        const int row = row0 + sub;
        const bool live = row < n;
        float acc[NOUT];
#pragma unroll
        for (int j = 0; j < NOUT; j++) acc[j] = 0.f;
        if (live) {
            const uint4 *src = reinterpret_cast<const uint4 *>(h + (size_t)row * HID);
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int q = 8 * c + part;
                const uint4 raw = src[q];
                const __nv_bfloat162 *p2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 f = __bfloat1622float2(p2[i]);
                    const int e0 = wpad(q * 8 + 2 * i), e1 = wpad(q * 8 + 2 * i + 1);
#pragma unroll
                    for (int j = 0; j < NOUT; j++) acc[j] += f.x * w_s[j * WROW + e0] + f.y * w_s[j * WROW + e1];
                }
            }
        }
#pragma unroll
        for (int o = 4; o > 0; o >>= 1)
#pragma unroll
            for (int j = 0; j < NOUT; j++) acc[j] += __shfl_xor_sync(FULL, acc[j], o);
        if (!live) continue;
        float l[NACT];
#pragma unroll
        for (int j = 0; j < NACT; j++) l[j] = acc[j] + b_s[j];
        const float v = acc[NACT] + b_s[NACT];
        if (logits_out) {
            // lanes part = 0..7 write logits part and part + 8 (when < 12)
            float m0 = l[0], m1 = l[8];
#pragma unroll
            for (int j = 1; j < 8; j++)
                if (part == j) m0 = l[j];
#pragma unroll
            for (int j = 9; j < NACT; j++)
                if (part + 8 == j) m1 = l[j];
            logits_out[(size_t)row * NACT + part] = m0;
            if (part + 8 < NACT) logits_out[(size_t)row * NACT + part + 8] = m1;
        }
        if (part == 0) {
            if (value) value[row] = v;
            if (action) {
                const uint32_t bits = legal ? legal[row] : 0xfffu;
                float m = -3.402823466e38f;
#pragma unroll
                for (int j = 0; j < NACT; j++)
                    if ((bits >> j) & 1u) m = fmaxf(m, l[j]);
                float z[NACT], total = 0.f;
#pragma unroll
                for (int j = 0; j < NACT; j++) {
                    z[j] = ((bits >> j) & 1u) ? d1_exp_nonpos(D1_ADD(l[j], -m)) : 0.f;
                    total = D1_ADD(total, z[j]);
                }
                int a = -1, last = 0;
                if (greedy) {
                    // first legal action of maximal logit (argmax of the masked probabilities)
#pragma unroll
                    for (int j = 0; j < NACT; j++)
                        if (a < 0 && ((bits >> j) & 1u) && l[j] == m) a = j;
                } else {
                    const float t = D1_MUL(sample_uniform((uint32_t)(first_env + row), seed, step), total);
                    float run = 0.f;
#pragma unroll
                    for (int j = 0; j < NACT; j++) {
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
                for (int j = 1; j < NACT; j++)
                    if (a == j) la = l[j];
                action[row] = a;
                if (logp) logp[row] = (la - m) - logf(total);
            }
        }
    }
}

}  // namespace head
}  // namespace d1

extern "C" int d1_policy_head_sample(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                     const uint16_t *legal, uint64_t seed, uint64_t step, int first_env,
                                     int64_t *action, float *logp, float *value, float *logits, void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    int blocks = (n + WARPS * 4 - 1) / (WARPS * 4);
    if (blocks > 148 * 8) blocks = 148 * 8;
    head_sample_kernel<<<blocks, WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, seed, step, first_env, action,
        logp, value, logits, 0);
    return (int)cudaGetLastError();
}

extern "C" int d1_policy_head_greedy(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                     const uint16_t *legal, int64_t *action, float *logp, float *value,
                                     void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh || !action) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    int blocks = (n + WARPS * 4 - 1) / (WARPS * 4);
    if (blocks > 148 * 8) blocks = 148 * 8;
    head_sample_kernel<<<blocks, WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, 0, 0, 0, action, logp, value,
        nullptr, 1);
    return (int)cudaGetLastError();
}
