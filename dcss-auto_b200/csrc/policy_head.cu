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
// The 13 dot products run on the tensor cores (mma.sync, see head_sample_kernel);
// the draw runs one thread per row.
#include <cuda_bf16.h>

#include "d1_common.cuh"
#include "d1_math.cuh"
#include "d1_philox.cuh"
#include "d1_sampler.cuh"

namespace d1 {
namespace head {

constexpr int HID = 256, NOUT = 13, NACT = 12;


// Tensor-core head: a warp takes 32 rows as two 16-row tiles and computes
// their 16 outputs (13 used) with mma.sync.m16n8k16 (bf16 in, fp32 accumulate),
// 16 K steps x 2 N tiles per tile. The dot product does not depend on the order
// of K, so K is permuted to make every fragment a contiguous load: for the
// K-step pair p, lane (g = lane / 4, q = lane % 4) takes hidden units
// 32p + 8q .. 32p + 8q + 7 of a row in one 16-byte load -- units +0,+1 / +2,+3
// are the A (or B) fragment halves of K step 2p, units +4..+7 those of step
// 2p + 1 -- so a warp's load covers 8 rows x 64 contiguous bytes. The head
// weights, permuted the same way, stay in 64 registers per lane. The logits go
// through shared memory so that each lane then owns one row for the masked
// draw (the same sampler as before: the draw from given logits is unchanged).
constexpr int WARPS_PER_BLOCK = 4, ROWS_PER_WARP = 32, PITCH = NOUT + 1;

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__global__ void __launch_bounds__(WARPS_PER_BLOCK * 32)
    head_sample_kernel(const __nv_bfloat16 *__restrict__ h, int n, const __nv_bfloat16 *__restrict__ wh,
                       const float *__restrict__ bh, const uint16_t *__restrict__ legal, uint64_t seed, uint64_t step,
                       int first_env, int64_t *__restrict__ action, float *__restrict__ logp,
                       float *__restrict__ value, float *__restrict__ logits_out, int greedy,
                       const int64_t *__restrict__ step_dev) {
    __shared__ float lg[WARPS_PER_BLOCK][ROWS_PER_WARP * PITCH];
    if (step_dev) step += (uint64_t)*step_dev;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, q = lane & 3;
    // B fragments: output n = 8t + g, K-step pair p
    uint4 bw[2][8];
#pragma unroll
    for (int t = 0; t < 2; t++) {
        const int nrow = 8 * t + g;
#pragma unroll
        for (int p = 0; p < 8; p++)
            bw[t][p] = nrow < NOUT ? __ldg(reinterpret_cast<const uint4 *>(wh + nrow * HID + 32 * p + 8 * q))
                                   : make_uint4(0u, 0u, 0u, 0u);
    }
    float bias[4];
#pragma unroll
    for (int t = 0; t < 2; t++)
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int col = 8 * t + 2 * q + j;
            bias[2 * t + j] = col < NOUT ? bh[col] : 0.f;
        }
    float *L = lg[warp];
    const int warps = gridDim.x * WARPS_PER_BLOCK;
    for (int base = (blockIdx.x * WARPS_PER_BLOCK + warp) * ROWS_PER_WARP; base < n; base += warps * ROWS_PER_WARP) {
#pragma unroll
        for (int tile = 0; tile < 2; tile++) {
            const int r0 = base + 16 * tile + g, r1 = r0 + 8;
            const uint4 *p0 = reinterpret_cast<const uint4 *>(h + (size_t)r0 * HID + 8 * q);
            const uint4 *p1 = reinterpret_cast<const uint4 *>(h + (size_t)r1 * HID + 8 * q);
            float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int p = 0; p < 8; p++) {
                const uint4 x0 = r0 < n ? __ldg(p0 + 4 * p) : make_uint4(0u, 0u, 0u, 0u);
                const uint4 x1 = r1 < n ? __ldg(p1 + 4 * p) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
                for (int t = 0; t < 2; t++) {
                    mma16816(c[t], x0.x, x1.x, x0.y, x1.y, bw[t][p].x, bw[t][p].y);
                    mma16816(c[t], x0.z, x1.z, x0.w, x1.w, bw[t][p].z, bw[t][p].w);
                }
            }
#pragma unroll
            for (int t = 0; t < 2; t++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    const int col = 8 * t + 2 * q + j;
                    if (col < NOUT) {
                        L[(16 * tile + g) * PITCH + col] = c[t][j] + bias[2 * t + j];
                        L[(16 * tile + g + 8) * PITCH + col] = c[t][2 + j] + bias[2 * t + j];
                    }
                }
        }
        __syncwarp();
        const int row = base + lane;
        if (row < n) {
            float l[NACT];
#pragma unroll
            for (int j = 0; j < NACT; j++) l[j] = L[lane * PITCH + j];
            if (value) value[row] = L[lane * PITCH + NACT];
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
        __syncwarp();
    }
}

static int head_launch(const void *h_bf16, int n, const void *wh_bf16, const float *bh, const uint16_t *legal,
                       uint64_t seed, uint64_t step, int first_env, int64_t *action, float *logp, float *value,
                       float *logits, int greedy, const int64_t *step_dev, void *stream) {
    if ((reinterpret_cast<uintptr_t>(h_bf16) | reinterpret_cast<uintptr_t>(wh_bf16)) & 15) return D1_ERR_BAD_ARGUMENT;
    const int rows_per_block = WARPS_PER_BLOCK * ROWS_PER_WARP;
    int blocks = (n + rows_per_block - 1) / rows_per_block;
    if (blocks > 148 * 16) blocks = 148 * 16;
    head_sample_kernel<<<blocks, WARPS_PER_BLOCK * 32, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)h_bf16, n, (const __nv_bfloat16 *)wh_bf16, bh, legal, seed, step, first_env, action,
        logp, value, logits, greedy, step_dev);
    return (int)cudaGetLastError();
}
}  // namespace head
}  // namespace d1

extern "C" int d1_policy_head_sample(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                     const uint16_t *legal, uint64_t seed, uint64_t step, int first_env,
                                     int64_t *action, float *logp, float *value, float *logits, void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    return head_launch(h_bf16, n, wh_bf16, bh, legal, seed, step, first_env, action, logp, value, logits, 0, nullptr,
                       stream);
}

extern "C" int d1_policy_head_sample_dev(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                         const uint16_t *legal, uint64_t seed, const int64_t *step_dev,
                                         int first_env, int64_t *action, float *logp, float *value, float *logits,
                                         void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh || !step_dev) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    return head_launch(h_bf16, n, wh_bf16, bh, legal, seed, 0, first_env, action, logp, value, logits, 0, step_dev,
                       stream);
}

extern "C" int d1_policy_head_greedy(const void *h_bf16, int n, int hidden, const void *wh_bf16, const float *bh,
                                     const uint16_t *legal, int64_t *action, float *logp, float *value,
                                     void *stream) {
    using namespace d1::head;
    if (n < 0 || hidden != HID || !h_bf16 || !wh_bf16 || !bh || !action) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    return head_launch(h_bf16, n, wh_bf16, bh, legal, 0, 0, 0, action, logp, value, nullptr, 1, nullptr, stream);
}
