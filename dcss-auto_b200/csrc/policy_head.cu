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
// One warp per row: lane l holds hidden elements 8l..8l+7 (one 16-byte load;
// a row is one coalesced 512-byte read), head weights live in shared memory,
// partial sums are combined with butterfly shuffles.
#include <cuda_bf16.h>

#include "d1_common.cuh"
#include "d1_math.cuh"

namespace d1 {
namespace head {

constexpr int HID = 256, NOUT = 13, NACT = 12, WARPS = 8;

__device__ __forceinline__ uint4 philox(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    }
    return c;
}

// Uniform in [0, 1) with 24 random bits: word 0 of
// Philox(ctr = {lo(step), hi(step), hi(seed), 1}, key = {env, lo(seed)}).
__device__ __forceinline__ float sample_uniform(uint32_t env, uint64_t seed, uint64_t step) {
    const uint4 o = philox(make_uint4((uint32_t)step, (uint32_t)(step >> 32), (uint32_t)(seed >> 32), 1u), env,
                           (uint32_t)seed);
    return (float)(o.x >> 8) * (1.0f / 16777216.0f);
}

__global__ void __launch_bounds__(WARPS * 32)
    head_sample_kernel(const __nv_bfloat16 *__restrict__ h, int n, const __nv_bfloat16 *__restrict__ wh,
                       const float *__restrict__ bh, const uint16_t *__restrict__ legal, uint64_t seed, uint64_t step,
                       int first_env, int64_t *__restrict__ action, float *__restrict__ logp,
                       float *__restrict__ value, float *__restrict__ logits_out) {
    __shared__ float w_s[NOUT][HID];
    for (int i = threadIdx.x; i < NOUT * HID; i += blockDim.x) w_s[i / HID][i % HID] = __bfloat162float(wh[i]);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int warps_total = gridDim.x * WARPS;
    for (int row = blockIdx.x * WARPS + (threadIdx.x >> 5); row < n; row += warps_total) {
        const uint4 raw = reinterpret_cast<const uint4 *>(h + (size_t)row * HID)[lane];
        float x[8];
        {
            const __nv_bfloat162 *p2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 f = __bfloat1622float2(p2[i]);
                x[2 * i] = f.x;
                x[2 * i + 1] = f.y;
            }
        }
        float acc[NOUT];
#pragma unroll
        for (int j = 0; j < NOUT; j++) {
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++) s += x[i] * w_s[j][lane * 8 + i];
            acc[j] = s;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int j = 0; j < NOUT; j++) acc[j] += __shfl_xor_sync(FULL, acc[j], o);
        float l[NACT];
#pragma unroll
        for (int j = 0; j < NACT; j++) l[j] = acc[j] + bh[j];
        const float v = acc[NACT] + bh[NACT];
        if (logits_out && lane < NACT) {
            float mine = l[0];
#pragma unroll
            for (int j = 1; j < NACT; j++)
                if (lane == j) mine = l[j];
            logits_out[(size_t)row * NACT + lane] = mine;
        }
        if (lane == 0) {
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
                const float t = D1_MUL(sample_uniform((uint32_t)(first_env + row), seed, step), total);
                int a = -1, last = 0;
                float run = 0.f;
#pragma unroll
                for (int j = 0; j < NACT; j++) {
                    if (!((bits >> j) & 1u)) continue;
                    last = j;
                    run = D1_ADD(run, z[j]);
                    if (a < 0 && t < run) a = j;
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
    int blocks = (n + WARPS - 1) / WARPS;
    if (blocks > 148 * 16) blocks = 148 * 16;
    head_sample_kernel<<<blocks, WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, seed, step, first_env, action,
        logp, value, logits);
    return (int)cudaGetLastError();
}
