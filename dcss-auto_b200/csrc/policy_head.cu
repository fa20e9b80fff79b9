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
// One thread per row; the head weights live in shared memory (fp32, read as
// broadcast float4s).
#include <cuda_bf16.h>

#include "d1_common.cuh"
#include "d1_math.cuh"
#include "d1_philox.cuh"
#include "d1_sampler.cuh"

namespace d1 {
namespace head {

constexpr int HID = 256, NOUT = 13, NACT = 12;


// One thread per row. The head weights sit in shared memory as fp32, so a
// warp's 32 threads read the same float4 (a broadcast) for 4 FMAs each; a row
// is read as 32 x 16-byte loads (8 hidden units each), 104 FMAs per load.
// Blocks of 128 threads keep ~48 warps per SM resident to hide the loads.
constexpr int ROWS_PER_BLOCK = 128;
__global__ void __launch_bounds__(ROWS_PER_BLOCK)
    head_sample_kernel(const __nv_bfloat16 *__restrict__ h, int n, const __nv_bfloat16 *__restrict__ wh,
                       const float *__restrict__ bh, const uint16_t *__restrict__ legal, uint64_t seed, uint64_t step,
                       int first_env, int64_t *__restrict__ action, float *__restrict__ logp,
                       float *__restrict__ value, float *__restrict__ logits_out, int greedy,
                       const int64_t *__restrict__ step_dev) {
    if (step_dev) step += (uint64_t)*step_dev;
    __shared__ float4 w4[NOUT][HID / 4];
    __shared__ float b_s[NOUT];
    for (int i = threadIdx.x; i < NOUT * HID / 4; i += blockDim.x) {
        const int j = i / (HID / 4), k = (i % (HID / 4)) * 4;
        const __nv_bfloat16 *src = wh + j * HID + k;
        w4[j][k / 4] = make_float4(__bfloat162float(src[0]), __bfloat162float(src[1]), __bfloat162float(src[2]),
                                   __bfloat162float(src[3]));
    }
    if (threadIdx.x < NOUT) b_s[threadIdx.x] = bh[threadIdx.x];
    __syncthreads();
    for (int row = blockIdx.x * blockDim.x + threadIdx.x; row < n; row += gridDim.x * blockDim.x) {
        float acc[NOUT];
#pragma unroll
        for (int j = 0; j < NOUT; j++) acc[j] = 0.f;
        const uint4 *src = reinterpret_cast<const uint4 *>(h + (size_t)row * HID);
#pragma unroll 4
        for (int c = 0; c < HID / 8; c++) {
            const uint4 raw = __ldg(src + c);
            const __nv_bfloat162 *p2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
            const float2 x01 = __bfloat1622float2(p2[0]), x23 = __bfloat1622float2(p2[1]);
            const float2 x45 = __bfloat1622float2(p2[2]), x67 = __bfloat1622float2(p2[3]);
#pragma unroll
            for (int j = 0; j < NOUT; j++) {
                const float4 wa = w4[j][2 * c], wb = w4[j][2 * c + 1];
                float a = acc[j];
                a = fmaf(x01.x, wa.x, a);
                a = fmaf(x01.y, wa.y, a);
                a = fmaf(x23.x, wa.z, a);
                a = fmaf(x23.y, wa.w, a);
                a = fmaf(x45.x, wb.x, a);
                a = fmaf(x45.y, wb.y, a);
                a = fmaf(x67.x, wb.z, a);
                a = fmaf(x67.y, wb.w, a);
                acc[j] = a;
            }
        }
        float l[NACT];
#pragma unroll
        for (int j = 0; j < NACT; j++) l[j] = acc[j] + b_s[j];
        if (value) value[row] = acc[NACT] + b_s[NACT];
        if (logits_out) {
#pragma unroll
            for (int j = 0; j < NACT; j++) logits_out[(size_t)row * NACT + j] = l[j];
        }
        if (action) {
            const uint32_t bits = legal ? legal[row] : 0xfffu;
            int a;
            float lp;
            sample_masked(l, bits, (uint32_t)(first_env + row), seed, step, greedy != 0, a, lp);
            action[row] = a;
            if (logp) logp[row] = lp;
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
    const int blocks = (n + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;
    head_sample_kernel<<<blocks, ROWS_PER_BLOCK, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, seed, step, first_env, action,
        logp, value, logits, 0, nullptr);
    return (int)cudaGetLastError();
}

extern "C" int d1_policy_head_sample_dev(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                         const uint16_t *legal, uint64_t seed, const int64_t *step_dev,
                                         int first_env, int64_t *action, float *logp, float *value, float *logits,
                                         void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh || !step_dev) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    const int blocks = (n + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;
    head_sample_kernel<<<blocks, ROWS_PER_BLOCK, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, seed, 0, first_env, action,
        logp, value, logits, 0, step_dev);
    return (int)cudaGetLastError();
}

extern "C" int d1_policy_head_greedy(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                     const uint16_t *legal, int64_t *action, float *logp, float *value,
                                     void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh || !action) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    const int blocks = (n + ROWS_PER_BLOCK - 1) / ROWS_PER_BLOCK;
    head_sample_kernel<<<blocks, ROWS_PER_BLOCK, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, 0, 0, 0, action, logp, value,
        nullptr, 1, nullptr);
    return (int)cudaGetLastError();
}
