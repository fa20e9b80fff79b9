// Rollout-side and update-side kernels of PPO (sm_100a): GAE, minibatch
// gather, fused head/loss/backward-to-hidden, split-K reduction with bias
// column sums, gradient norm and Adam. The tensor-core GEMMs in between are
// d1_gemm (gemm_tc.cu).
//
// Reference update: gpu-d1/scripts/run_ring_ablations.py:354-372.
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "d1_common.cuh"
#include "d1_pdl.cuh"

namespace d1 {
namespace ppo {

// ------------------------------------------------------------------ GAE
// A_t = delta_t + gamma*lambda*(1 - done_t) * A_{t+1},
// delta_t = r_t + gamma * V_{t+1} * (1 - done_t) - V_t, returns = A + V.
// rewards/dones are read with element strides (they live in the env's
// outcome rows: reward at out[t, b, 0], done at out[t, b, 1]).
// Deterministic cross-block sums. Each block reduces its values in a fixed
// order, writes one partial, and the last block to finish (an integer ticket,
// whose outcome does not depend on timing) adds the partials in block order.
// Floating-point atomics would make the sums -- and everything downstream of the
// advantage normalisation and the gradient-norm clip -- vary from run to run.
// The partial arrays are fixed in the library: calls on one device are
// serialised by the caller (one stream per training process).
constexpr int RED_MAX_BLOCKS = 65536;
__device__ double g_gae_part[RED_MAX_BLOCKS][2];
__device__ unsigned g_gae_ticket;

// Block-wide ordered sum of (a, b): warp butterflies, then thread 0 over the
// warps in order. Result valid in thread 0.
template <int WARPS_>
__device__ __forceinline__ void block_sum2(double &a, double &b, double (*ws)[2]) {
    for (int o = 16; o > 0; o >>= 1) {
        a += __shfl_xor_sync(FULL, a, o);
        b += __shfl_xor_sync(FULL, b, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        ws[warp][0] = a;
        ws[warp][1] = b;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        a = 0.0;
        b = 0.0;
        for (int w = 0; w < WARPS_; w++) {
            a += ws[w][0];
            b += ws[w][1];
        }
    }
}
// Thread 0 of every block passes its partial; the last block adds all partials
// to out[0] (and out[1] when `two`) and resets the ticket. The last block's
// threads each add the partials i = thread, thread + blockDim, ... (loads issued
// together through L2, not one dependent round trip per partial), then the
// block adds the threads' sums in a fixed order, so the result does not depend
// on timing.
__device__ __forceinline__ void finish_sum2(double a, double b, double (*part)[2], unsigned *ticket, double *out,
                                            bool two) {
    __shared__ bool last;
    __shared__ double fin[32][2];
    const int nparts = gridDim.x;
    if (threadIdx.x == 0) {
        part[blockIdx.x][0] = a;
        part[blockIdx.x][1] = b;
        __threadfence();
        last = atomicAdd(ticket, 1u) == (unsigned)nparts - 1u;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    double s1 = 0.0, s2 = 0.0;
#pragma unroll 8
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) {
        s1 += __ldcg(&part[i][0]);
        s2 += __ldcg(&part[i][1]);
    }
    for (int o = 16; o > 0; o >>= 1) {
        s1 += __shfl_xor_sync(FULL, s1, o);
        s2 += __shfl_xor_sync(FULL, s2, o);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = (blockDim.x + 31) >> 5;
    if (lane == 0) {
        fin[warp][0] = s1;
        fin[warp][1] = s2;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        s1 = 0.0;
        s2 = 0.0;
        for (int w = 0; w < warps; w++) {
            s1 += fin[w][0];
            s2 += fin[w][1];
        }
        out[0] += s1;
        if (two) out[1] += s2;
        *ticket = 0u;
    }
}

struct GaeArgs {
    const float *reward, *done, *value;  // value: [T+1, B]
    int64_t r_step, r_env;               // element strides of reward (and done)
    float *adv, *ret;                    // [T, B]
    double *stats;                       // [3]: sum adv, sum adv^2 (accumulated), unused
    int T, B;
    float gamma, gamma_lambda;
};

// Exact replay of the reference's per-step tensor ops, each separately rounded
// (torch evaluates r + g*v*live - V and delta + gl*live*A one op at a time).
__global__ void gae_sequential_kernel(GaeArgs a) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    double s1 = 0.0, s2 = 0.0;
    if (b < a.B) {
        float nextv = a.value[(size_t)a.T * a.B + b], gae = 0.f;
        for (int t = a.T - 1; t >= 0; t--) {
            const size_t o = (size_t)t * a.r_step + (size_t)b * a.r_env;
            const float live = __fsub_rn(1.f, a.done[o]);
            const float v = a.value[(size_t)t * a.B + b];
            const float delta = __fsub_rn(__fadd_rn(a.reward[o], __fmul_rn(__fmul_rn(a.gamma, nextv), live)), v);
            gae = __fadd_rn(delta, __fmul_rn(__fmul_rn(a.gamma_lambda, live), gae));
            a.adv[(size_t)t * a.B + b] = gae;
            a.ret[(size_t)t * a.B + b] = __fadd_rn(gae, v);
            s1 += gae;
            s2 += (double)gae * gae;
            nextv = v;
        }
    }
    if (a.stats) {
        __shared__ double ws[8][2];
        block_sum2<8>(s1, s2, ws);
        finish_sum2(s1, s2, g_gae_part, &g_gae_ticket, a.stats, true);
    }
}

// Segmented scan over time. The recurrence is an affine map
// A_t = d_t + c_t * A_{t+1} (d_t = r_t + gamma * v_{t+1} * live_t - v_t,
// c_t = gamma * lambda * live_t), and maps compose associatively:
// (D1, C1) o (D2, C2) = (D1 + C1 * D2, C1 * C2). An env group is 32 * EPT envs
// (lane l holds envs EPT*l .. EPT*l + EPT-1, so every row of the group is one
// coalesced 128- or 256-byte access) and warp w the contiguous rows
// [w * R, (w + 1) * R), R = ceil(T / 8):
//   1. each thread composes its run front to back in registers (2 ops a step);
//   2. the 8 runs of an env are combined across the warps through shared
//      memory: the value entering warp w's run is runs w+1..7 applied to
//      A_T = 0;
//   3. each thread walks its run back to front from that value and writes the
//      advantages and returns.
// Runs go in chunks of SCAN_CHUNK rows; the last chunk of a run stays in
// registers from step 1 to step 3, the others are re-read (from L2). Blocks
// are persistent (SCAN_BLOCKS_PER_SM per SM) and loop over the env groups, so
// the statistics' ordered block sum runs once per block, not once per group.
// Rounding differs from the sequential order (tolerance 1e-5 relative).
// Measured at 65,536 envs x 128 steps: 0.043 ms with EPT = 2 (float2 rows),
// against 0.050 with EPT = 1 and 0.085 for the earlier form that transposed
// each group through shared memory (lane = time run; instruction-bound).
constexpr int SCAN_WARPS = 8, SCAN_CHUNK = 8, SCAN_BLOCKS_PER_SM = 3;
template <int EPT>
struct GaeVec;
template <>
struct GaeVec<1> {
    static __device__ __forceinline__ void load(const float *p, float (&x)[1][SCAN_CHUNK], int i, bool ld, float fill) {
        x[0][i] = ld ? __ldg(p) : fill;
    }
    static __device__ __forceinline__ void load1(const float *p, float (&x)[1][SCAN_CHUNK + 1], int i, bool ld) {
        x[0][i] = ld ? __ldg(p) : 0.f;
    }
    static __device__ __forceinline__ void store(float *p, const float (&x)[1]) { *p = x[0]; }
};
template <>
struct GaeVec<2> {
    static __device__ __forceinline__ void load(const float *p, float (&x)[2][SCAN_CHUNK], int i, bool ld, float fill) {
        const float2 v = ld ? __ldg(reinterpret_cast<const float2 *>(p)) : make_float2(fill, fill);
        x[0][i] = v.x;
        x[1][i] = v.y;
    }
    static __device__ __forceinline__ void load1(const float *p, float (&x)[2][SCAN_CHUNK + 1], int i, bool ld) {
        const float2 v = ld ? __ldg(reinterpret_cast<const float2 *>(p)) : make_float2(0.f, 0.f);
        x[0][i] = v.x;
        x[1][i] = v.y;
    }
    static __device__ __forceinline__ void store(float *p, const float (&x)[2]) {
        *reinterpret_cast<float2 *>(p) = make_float2(x[0], x[1]);
    }
};
// Rows [c0, c0 + SCAN_CHUNK) below r1 of this thread's envs: d_t in d[e][],
// v_t in v[e][], live_t as bit i of live[e] (rows past r1 read nothing).
template <int EPT>
__device__ __forceinline__ void gae_load_chunk(const GaeArgs &a, const float *rw, const float *dn, const float *vl,
                                               bool in, int c0, int r1, float (&d)[EPT][SCAN_CHUNK],
                                               float (&v)[EPT][SCAN_CHUNK], unsigned (&live)[EPT]) {
    const int64_t rs = a.r_step, vs = a.B;
    float rv[EPT][SCAN_CHUNK], dv[EPT][SCAN_CHUNK], vn[EPT][SCAN_CHUNK + 1];
    rw += c0 * rs;
    dn += c0 * rs;
    vl += c0 * vs;
#pragma unroll
    for (int i = 0; i < SCAN_CHUNK; i++) {
        const bool ld = in && c0 + i < r1;
        GaeVec<EPT>::load(rw + i * rs, rv, i, ld, 0.f);
        GaeVec<EPT>::load(dn + i * rs, dv, i, ld, 1.f);
    }
#pragma unroll
    for (int i = 0; i <= SCAN_CHUNK; i++)  // value has T + 1 rows and r1 <= T
        GaeVec<EPT>::load1(vl + i * vs, vn, i, in && c0 + i <= r1);
#pragma unroll
    for (int e = 0; e < EPT; e++) {
        live[e] = 0u;
#pragma unroll
        for (int i = 0; i < SCAN_CHUNK; i++) {
            const float l = 1.f - dv[e][i];
            d[e][i] = rv[e][i] + a.gamma * vn[e][i + 1] * l - vn[e][i];
            v[e][i] = vn[e][i];
            live[e] |= (l != 0.f ? 1u : 0u) << i;
        }
    }
}
// EPT = 2 needs r_env == 1, B even and 8-byte aligned rows (the launcher checks).
template <int EPT>
__global__ void __launch_bounds__(SCAN_WARPS * 32, SCAN_BLOCKS_PER_SM) gae_scan_kernel(GaeArgs a) {
    constexpr int ENVS = 32 * EPT;
    __shared__ float run_d[SCAN_WARPS][ENVS], run_c[SCAN_WARPS][ENVS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int R = (a.T + SCAN_WARPS - 1) / SCAN_WARPS;
    const int r0 = min(a.T, warp * R), r1 = min(a.T, r0 + R);
    const float gl = a.gamma_lambda;
    const int64_t vs = a.B;
    const int groups = (a.B + ENVS - 1) / ENVS;
    double s1 = 0.0, s2 = 0.0;
    for (int g = blockIdx.x; g < groups; g += gridDim.x) {
        const int b = g * ENVS + lane * EPT;
        const bool in = b < a.B;  // with EPT = 2, B is even: both envs or neither
        const size_t bo = in ? (size_t)b : 0;
        const float *rw = a.reward + bo * a.r_env, *dn = a.done + bo * a.r_env, *vl = a.value + bo;
        float d[EPT][SCAN_CHUNK], v[EPT][SCAN_CHUNK], D[EPT], C[EPT];
        unsigned live[EPT];
#pragma unroll
        for (int e = 0; e < EPT; e++) {
            D[e] = 0.f;
            C[e] = 1.f;
        }
        // 1. compose the run front to back: (D, C) <- (D + C * d_t, C * c_t)
        int last = r0;  // first row of the chunk held in registers
        for (int c0 = r0; c0 < r1; c0 += SCAN_CHUNK) {
            gae_load_chunk<EPT>(a, rw, dn, vl, in, c0, r1, d, v, live);
            last = c0;
#pragma unroll
            for (int i = 0; i < SCAN_CHUNK; i++) {
                if (c0 + i < r1) {
#pragma unroll
                    for (int e = 0; e < EPT; e++) {
                        D[e] = D[e] + C[e] * d[e][i];
                        C[e] = C[e] * (((live[e] >> i) & 1u) ? gl : 0.f);
                    }
                }
            }
        }
        // 2. the value entering this run: the later warps' runs applied to A_T = 0
        __syncthreads();  // the previous group's reads of run_d / run_c are done
#pragma unroll
        for (int e = 0; e < EPT; e++) {
            run_d[warp][lane * EPT + e] = D[e];
            run_c[warp][lane * EPT + e] = C[e];
        }
        __syncthreads();
        float A[EPT];
#pragma unroll
        for (int e = 0; e < EPT; e++) {
            A[e] = 0.f;
            for (int k = SCAN_WARPS - 1; k > warp; k--) A[e] = run_d[k][lane * EPT + e] + run_c[k][lane * EPT + e] * A[e];
        }
        // 3. back to front: A_t = d_t + c_t * A_{t+1}
        for (int c0 = last; c0 >= r0; c0 -= SCAN_CHUNK) {
            if (c0 != last) gae_load_chunk<EPT>(a, rw, dn, vl, in, c0, r1, d, v, live);
            float *ad = a.adv + bo + c0 * vs, *rt = a.ret + bo + c0 * vs;
            float f1 = 0.f, f2 = 0.f;  // this chunk's sums, added to the double totals below
#pragma unroll
            for (int i = SCAN_CHUNK - 1; i >= 0; i--) {
                if (c0 + i < r1) {
                    float q[EPT];
#pragma unroll
                    for (int e = 0; e < EPT; e++) {
                        A[e] = d[e][i] + (((live[e] >> i) & 1u) ? gl : 0.f) * A[e];
                        q[e] = A[e] + v[e][i];
                        f1 += A[e];
                        f2 += A[e] * A[e];
                    }
                    if (in) {
                        GaeVec<EPT>::store(ad + i * vs, A);
                        GaeVec<EPT>::store(rt + i * vs, q);
                    }
                }
            }
            if (in) {
                s1 += f1;
                s2 += f2;
            }
        }
    }
    if (a.stats) {
        __shared__ double ws[SCAN_WARPS][2];
        block_sum2<SCAN_WARPS>(s1, s2, ws);
        finish_sum2(s1, s2, g_gae_part, &g_gae_ticket, a.stats, true);
    }
}


// ------------------------------------------------------------------ minibatch gather
// X[i] = obs[idx[i]] (bf16 rows of F features) and X^T (feature-major, the
// B operand of the first-layer weight-gradient GEMM). Block (x, y) owns 64
// samples and G_GROUP 64-feature chunks of their rows, which it walks through a
// G_STAGES-deep cp.async ring in shared memory: five chunks (40 KB) are in
// flight while the sixth is written out. Row writes are 128-byte sample
// segments, transposed writes 128-byte feature segments. Splitting the features
// over blockIdx.y gives ~7 blocks per SM at minibatch 16,384, so the samples
// spread evenly over the 148 SMs. F must be a multiple of 8.
constexpr int G_SAMPLES = 64, G_FEAT = 64, G_STAGES = 6, G_PITCH = G_FEAT, G_GROUP = 8;
// A stage holds 64 sample rows of 128 B. The 16-byte unit u of row r sits at
// unit u ^ ((r >> 3) & 7), so the transposed reads (8 threads on rows 8 apart,
// same feature) land in 8 different banks instead of one.
__device__ __forceinline__ int g_swz(int row, int unit) { return row * G_PITCH + ((unit ^ ((row >> 3) & 7)) << 3); }
constexpr int G_SMEM = G_STAGES * G_SAMPLES * G_PITCH * 2;

__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(256) gather_kernel(const __nv_bfloat16 *__restrict__ obs, int F,
                                                     const int64_t *__restrict__ idx, int n, __nv_bfloat16 *x,
                                                     int ldx, int ones) {
    extern __shared__ __align__(16) __nv_bfloat16 gbuf[];  // [G_STAGES][G_SAMPLES][G_PITCH]
    const int s0 = blockIdx.x * G_SAMPLES;
    const int t = threadIdx.x, part = t & 7;
    const int c_begin = blockIdx.y * G_GROUP;
    const int nchunks = min((F + G_FEAT - 1) / G_FEAT - c_begin, G_GROUP);
    const __nv_bfloat16 *src[2];
    bool live[2];
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int gs = s0 + (t >> 3) + 32 * h;
        live[h] = gs < n;
        src[h] = obs + (live[h] ? (size_t)idx[gs] * F : 0);
    }
    auto issue = [&](int c) {
        if (c < nchunks) {
            __nv_bfloat16 *buf = gbuf + (c % G_STAGES) * (G_SAMPLES * G_PITCH);
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int ls = (t >> 3) + 32 * h, f = (c_begin + c) * G_FEAT + part * 8;
                const bool ok = live[h] && f < F;
                cp_async16(buf + g_swz(ls, part), ok ? src[h] + f : obs, ok ? 16 : 0);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int c = 0; c < G_STAGES - 1; c++) issue(c);
    for (int c = 0; c < nchunks; c++) {
        issue(c + G_STAGES - 1);
        cp_async_wait<G_STAGES - 1>();
        __syncthreads();
        const __nv_bfloat16 *buf = gbuf + (c % G_STAGES) * (G_SAMPLES * G_PITCH);
        const int f0 = (c_begin + c) * G_FEAT;
        if (x) {
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int ls = (t >> 3) + 32 * h, f = f0 + part * 8;
                if (live[h] && f < F)
                    *reinterpret_cast<uint4 *>(x + (size_t)(s0 + ls) * ldx + f) =
                        *reinterpret_cast<const uint4 *>(buf + g_swz(ls, part));
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();
    // columns F..F+7 = (1, 0, ..., 0): the product dh^T X then carries the
    // column sums of dh (the bias gradient) in its column F
    if (x && ones && blockIdx.y == 0 && t < G_SAMPLES && s0 + t < n)
        *reinterpret_cast<uint4 *>(x + (size_t)(s0 + t) * ldx + F) = make_uint4(0x3f80u, 0u, 0u, 0u);
}

// ------------------------------------------------------------------ compact-observation gather
// X[i] = one-hot expansion of the compact observation row cobs[idx[i]] (320 B:
// the channel 0-7 of each of the 225 window cells as a byte, then the 32
// scalars as bf16 at byte 256) into the 1832-feature bf16 layout the policy
// reads (cell c, channel k at element 8c + k; scalars at 1800), plus the ones
// column (1, 0, ..., 0) at 1832 when asked for. One warp per sample: the row is
// staged in shared memory, then each lane writes 16-byte units (one cell's 8
// channels, or 8 scalars) from a table of the 8 one-hot patterns.
constexpr int CG_WARPS = 8, COBS_BYTES = 320, COBS_CELLS = 225, COBS_SCALARS = 256;
__global__ void __launch_bounds__(CG_WARPS * 32)
    gather_cobs_kernel(const uint8_t *__restrict__ cobs, const int64_t *__restrict__ idx, int n, uint4 *x, int ldx16,
                       int ones) {
    __shared__ uint4 rows[CG_WARPS][COBS_BYTES / 16];
    __shared__ uint4 onehot[8];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 8) {
        const uint32_t one = 0x3f80u << (16 * (threadIdx.x & 1));
        const int k = threadIdx.x >> 1;
        onehot[threadIdx.x] = make_uint4(k == 0 ? one : 0u, k == 1 ? one : 0u, k == 2 ? one : 0u, k == 3 ? one : 0u);
    }
    __syncthreads();
    for (int i = blockIdx.x * CG_WARPS + w; i < n; i += gridDim.x * CG_WARPS) {
        const uint4 *src = reinterpret_cast<const uint4 *>(cobs + (size_t)idx[i] * COBS_BYTES);
        if (lane < COBS_BYTES / 16) rows[w][lane] = __ldg(src + lane);
        __syncwarp();
        const uint8_t *codes = reinterpret_cast<const uint8_t *>(rows[w]);
        uint4 *dst = x + (size_t)i * ldx16;
        for (int u = lane; u < COBS_CELLS + 5; u += 32) {
            uint4 v;
            if (u < COBS_CELLS) v = onehot[codes[u] & 7];
            else if (u < COBS_CELLS + 4) v = rows[w][COBS_SCALARS / 16 + (u - COBS_CELLS)];
            else if (ones) v = make_uint4(0x3f80u, 0u, 0u, 0u);
            else break;
            dst[u] = v;
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------ fused head + loss + backward to h2
// Per minibatch row (sample index idx[row] into the rollout arrays):
//   logits, value = h2 . Wh^T + bh; masked log-softmax over the legal bits;
//   ratio = exp(logp(a) - old_logp); adv normalised with the batch mean/std;
//   pg = -min(ratio*adv, clamp(ratio, 1-clip, 1+clip)*adv)
//   vf = max((v-ret)^2, (v_old + clamp(v-v_old, -vclip, vclip) - ret)^2)   (vclip > 0)
//      = (v-ret)^2                                                           (vclip <= 0)
//   loss = mean(pg) + vf_coef*mean(vf) - ent_coef*mean(entropy)
// and its gradient with respect to logits/value, then dh2 = dhead . Wh masked by
// ReLU'(h2) (bf16, row-major and transposed). Block partials of dWh, dbh, db2
// and of the loss terms go to `part` for a deterministic reduction.
struct LossArgs {
    const __nv_bfloat16 *h2;   // [n, 256]
    const __nv_bfloat16 *wh;   // [13, 256]
    const float *bh;           // [13]
    const int64_t *idx;        // [n] rollout sample ids
    const uint16_t *legal;     // [total]
    const int64_t *action;     // [total]
    const float *old_logp, *adv, *ret, *old_value;  // [total]
    const double *adv_stats;   // [2]: sum, sum of squares over adv_count samples
    double adv_count;
    int n;
    float clip, vclip, vf_coef, ent_coef;
    __nv_bfloat16 *dh2, *dh2t; // [n, 256], [256, ldt]
    int ldt;
    float *part;               // per block: dWh[13*256], dbh[13], db2[256], terms[8]
};
constexpr int L_HID = 256, L_NOUT = 13, L_NACT = 12;
constexpr int L_PART = L_NOUT * L_HID + L_NOUT + L_HID + 8;

// ------------------------------------------------------------------ loss on warp-level tensor-core MMAs
// Its three small products run on mma.sync.m16n8k16 (bf16 in, fp32 accumulate):
//   logits [16 rows x 16]   = h2 [16 x 256] . Wh^T          (per warp, 16 k-steps)
//   dWh    [16 x 256]      += dhead^T [16 x 64 rows] . h2    (warp w: columns 64w..)
//   dh2    [16 rows x 256]  = dhead [16 x 16] . Wh           (per warp, 32 n-tiles)
// The head gradient dhead (fp32) enters the MMAs as two bf16 parts, hi + lo,
// so its ~16-bit precision survives. The softmax, loss and dhead are computed
// on the accumulator layout: lane (g, q) holds rows g and g + 8, columns
// 2q, 2q+1, 2q+8, 2q+9; row statistics are quad shuffles. A block (4 warps)
// takes 64 rows per pass; dh2 overwrites the staged h2 tile in place (masked by
// h2 > 0) and leaves as row-major and transposed 16-byte stores.
constexpr int M_ROWS = 64, M_WARPS = 4, M_PITCH = L_HID + 8, D_PITCH = 24;
struct MmaSmem {
    __nv_bfloat16 h2[M_ROWS][M_PITCH];     // h2 tile, then dh2
    __nv_bfloat16 wh[16][M_PITCH];         // head weights, rows 13-15 zero
    __nv_bfloat16 dhi[M_ROWS][D_PITCH];    // dhead, bf16 high part
    __nv_bfloat16 dlo[M_ROWS][D_PITCH];    // dhead, bf16 remainder
    float dhf[M_ROWS][16];                 // dhead fp32 (for dbh)
    float r_olp[M_ROWS], r_adv[M_ROWS], r_ret[M_ROWS], r_vold[M_ROWS];
    int r_bits[M_ROWS], r_act[M_ROWS];
    float terms[M_WARPS][8];
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void mma16816(float *c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float quad_max(float v) {
    v = fmaxf(v, __shfl_xor_sync(FULL, v, 1));
    return fmaxf(v, __shfl_xor_sync(FULL, v, 2));
}
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(FULL, v, 1);
    return v + __shfl_xor_sync(FULL, v, 2);
}
__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__global__ void __launch_bounds__(M_WARPS * 32) loss_mma_kernel(LossArgs a) {
    extern __shared__ __align__(16) uint8_t mma_raw[];
    MmaSmem &S = *reinterpret_cast<MmaSmem *>(mma_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, q = lane & 3;
    for (int i = tid; i < 16 * (L_HID / 8); i += blockDim.x) {
        const int j = i / (L_HID / 8), c = (i % (L_HID / 8)) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (j < L_NOUT) v = *reinterpret_cast<const uint4 *>(a.wh + j * L_HID + c);
        *reinterpret_cast<uint4 *>(&S.wh[j][c]) = v;
    }
    const double mean = a.adv_stats[0] / a.adv_count;
    const double var = (a.adv_stats[1] - a.adv_stats[0] * mean) / (a.adv_count - 1.0);
    const float amean = (float)mean, astd = (float)sqrt(var > 0 ? var : 0.0);
    const float inv_n = 1.f / (float)a.n;
    // this lane's four head columns and their biases
    int col[4];
    float bias[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        col[e] = (e < 2 ? 0 : 8) + 2 * q + (e & 1);
        bias[e] = col[e] < L_NOUT ? a.bh[col[e]] : 0.f;
    }
    float acc_w[8][4];  // dWh for columns 64*warp + 8*nt .. (rows j = g, g + 8)
#pragma unroll
    for (int nt = 0; nt < 8; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc_w[nt][e] = 0.f;
    float acc_b2[2] = {0.f, 0.f}, acc_bh = 0.f;
    float t_pg = 0.f, t_vf = 0.f, t_ent = 0.f, t_clip = 0.f, t_kl = 0.f;
    const int nb = (a.n + M_ROWS - 1) / M_ROWS;
    for (int blk = blockIdx.x; blk < nb; blk += gridDim.x) {
        const int r0 = blk * M_ROWS;
        __syncthreads();  // the previous pass's readers are done
        if (tid < M_ROWS && r0 + tid < a.n) {
            const int64_t sidx = a.idx[r0 + tid];
            S.r_bits[tid] = a.legal[sidx];
            S.r_act[tid] = (int)a.action[sidx];
            S.r_olp[tid] = a.old_logp[sidx];
            S.r_adv[tid] = a.adv[sidx];
            S.r_ret[tid] = a.ret[sidx];
            S.r_vold[tid] = a.old_value[sidx];
        }
        for (int i = tid; i < M_ROWS * (L_HID / 8); i += blockDim.x) {
            const int r = i / (L_HID / 8), c = (i % (L_HID / 8)) * 8;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r0 + r < a.n) v = *reinterpret_cast<const uint4 *>(a.h2 + (size_t)(r0 + r) * L_HID + c);
            *reinterpret_cast<uint4 *>(&S.h2[r][c]) = v;
        }
        __syncthreads();
        // ---- logits: rows 16*warp .. +15
        const int wr = warp * 16;
        float lg[2][4];  // n-tile 0 (cols 0-7), n-tile 1 (cols 8-15); c0..c3
#pragma unroll
        for (int t = 0; t < 2; t++)
#pragma unroll
            for (int e = 0; e < 4; e++) lg[t][e] = 0.f;
        {
            // A: matrix m = lane / 8: rows wr + (m & 1) * 8 + lane % 8, cols k + (m >> 1) * 8
            const int am = lane >> 3;
            const uint32_t a_base = smem_addr(&S.h2[wr + (am & 1) * 8 + (lane & 7)][(am >> 1) * 8]);
            // B (Wh as [n = j][k]): matrix m: rows j = (m >> 1) * 8 + lane % 8, cols k + (m & 1) * 8
            const uint32_t b_base = smem_addr(&S.wh[(am >> 1) * 8 + (lane & 7)][(am & 1) * 8]);
#pragma unroll 4
            for (int ks = 0; ks < L_HID / 16; ks++) {
                uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
                ldsm_x4(a_base + ks * 32, a0, a1, a2, a3);
                ldsm_x4(b_base + ks * 32, b0, b1, b2, b3);
                mma16816(lg[0], a0, a1, a2, a3, b0, b1);
                mma16816(lg[1], a0, a1, a2, a3, b2, b3);
            }
        }
        // ---- per-row loss and dhead on the accumulator layout (rows g, g + 8)
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int lr = wr + g + 8 * h, row = r0 + lr;
            const bool live = row < a.n;
            const uint32_t bits = live ? (uint32_t)S.r_bits[lr] : 0u;
            const int act = live ? S.r_act[lr] : 0;
            float l[4];
            bool ok[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                l[e] = lg[e >> 1][(e & 1) + 2 * h] + bias[e];
                ok[e] = col[e] < L_NACT && ((bits >> col[e]) & 1u);
            }
            float m = -3.402823466e38f;
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (ok[e]) m = fmaxf(m, l[e]);
            m = quad_max(m);
            float z = 0.f;
#pragma unroll
            for (int e = 0; e < 4; e++)
                if (ok[e]) z += expf(l[e] - m);
            z = quad_sum(z);
            const float lz = logf(z);
            float lp[4], p[4], ent = 0.f, la = 0.f, value = 0.f;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                lp[e] = l[e] - m - lz;
                p[e] = ok[e] ? expf(lp[e]) : 0.f;
                if (ok[e]) ent -= p[e] * lp[e];
                if (col[e] == act) la = lp[e];
                if (col[e] == L_NACT) value = l[e];
            }
            ent = quad_sum(ent);
            la = quad_sum(la);
            value = quad_sum(value);
            float dl[4] = {0.f, 0.f, 0.f, 0.f};
            if (live) {
                const float adv = (S.r_adv[lr] - amean) / (astd + 1e-8f);
                const float olp = S.r_olp[lr];
                const float ratio = expf(la - olp);
                const float s1 = ratio * adv, rc = fminf(fmaxf(ratio, 1.f - a.clip), 1.f + a.clip), s2 = rc * adv;
                const float pg = -fminf(s1, s2);
                float dpg_dr = 0.f;
                if (s1 <= s2) dpg_dr = -adv;
                else if (ratio > 1.f - a.clip && ratio < 1.f + a.clip) dpg_dr = -adv;
                const float dlogp = dpg_dr * ratio * inv_n;
                const float R = S.r_ret[lr], vold = S.r_vold[lr];
                float vf, dvf;
                const float e1 = value - R;
                if (a.vclip > 0.f) {
                    const float dvc = fminf(fmaxf(value - vold, -a.vclip), a.vclip);
                    const float e2 = vold + dvc - R;
                    if (e1 * e1 >= e2 * e2) {
                        vf = e1 * e1;
                        dvf = 2.f * e1;
                    } else {
                        vf = e2 * e2;
                        dvf = (value - vold > -a.vclip && value - vold < a.vclip) ? 2.f * e2 : 0.f;
                    }
                } else {
                    vf = e1 * e1;
                    dvf = 2.f * e1;
                }
                const float dv = a.vf_coef * dvf * inv_n;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    if (ok[e])
                        dl[e] = dlogp * ((col[e] == act ? 1.f : 0.f) - p[e]) + a.ent_coef * inv_n * p[e] * (lp[e] + ent);
                    else if (col[e] == L_NACT)
                        dl[e] = dv;
                }
                if (q == 0) {
                    t_pg += pg;
                    t_vf += vf;
                    t_ent += ent;
                    t_clip += fabsf(ratio - 1.f) > a.clip ? 1.f : 0.f;
                    t_kl += olp - la;
                }
            }
#pragma unroll
            for (int e = 0; e < 4; e += 2) {
                const __nv_bfloat162 hi = __floats2bfloat162_rn(dl[e], dl[e + 1]);
                const float2 hf = __bfloat1622float2(hi);
                const __nv_bfloat162 lo = __floats2bfloat162_rn(dl[e] - hf.x, dl[e + 1] - hf.y);
                *reinterpret_cast<__nv_bfloat162 *>(&S.dhi[lr][col[e]]) = hi;
                *reinterpret_cast<__nv_bfloat162 *>(&S.dlo[lr][col[e]]) = lo;
                S.dhf[lr][col[e]] = dl[e];
                S.dhf[lr][col[e] + 1] = dl[e + 1];
            }
        }
        __syncthreads();
        // ---- dWh[j][c] += sum_r dhead[r][j] h2[r][c], warp w: columns 64w .. 64w+63
        {
            const int am = lane >> 3;
#pragma unroll
            for (int ks = 0; ks < M_ROWS / 16; ks++) {
                // A = dhead^T (m = j, k = r) from dhead stored [r][j]: transposed loads,
                // matrix m: rows r = ks*16 + (m >> 1) * 8 + lane % 8, cols j = (m & 1) * 8
                uint32_t ah[4], al[4];
                ldsm_x4_t(smem_addr(&S.dhi[ks * 16 + (am >> 1) * 8 + (lane & 7)][(am & 1) * 8]), ah[0], ah[1], ah[2],
                          ah[3]);
                ldsm_x4_t(smem_addr(&S.dlo[ks * 16 + (am >> 1) * 8 + (lane & 7)][(am & 1) * 8]), al[0], al[1], al[2],
                          al[3]);
#pragma unroll
                for (int np = 0; np < 4; np++) {
                    // B = h2 (k = r, n = c) from h2 stored [r][c]: transposed loads,
                    // matrix m: rows r = ks*16 + (m & 1) * 8 + lane % 8, cols c = base + (m >> 1) * 8
                    const int c0 = warp * 64 + np * 16;
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(smem_addr(&S.h2[ks * 16 + (am & 1) * 8 + (lane & 7)][c0 + (am >> 1) * 8]), b0, b1, b2,
                              b3);
                    mma16816(acc_w[2 * np], ah[0], ah[1], ah[2], ah[3], b0, b1);
                    mma16816(acc_w[2 * np], al[0], al[1], al[2], al[3], b0, b1);
                    mma16816(acc_w[2 * np + 1], ah[0], ah[1], ah[2], ah[3], b2, b3);
                    mma16816(acc_w[2 * np + 1], al[0], al[1], al[2], al[3], b2, b3);
                }
            }
        }
        __syncthreads();  // every warp has read h2 for dWh: it may now become dh2
        // ---- dh2 = (dhead . Wh) masked by ReLU'(h2), rows 16*warp .. +15, in place
        {
            const int am = lane >> 3;
            uint32_t ah[4], al[4];
            ldsm_x4(smem_addr(&S.dhi[wr + (am & 1) * 8 + (lane & 7)][(am >> 1) * 8]), ah[0], ah[1], ah[2], ah[3]);
            ldsm_x4(smem_addr(&S.dlo[wr + (am & 1) * 8 + (lane & 7)][(am >> 1) * 8]), al[0], al[1], al[2], al[3]);
#pragma unroll 4
            for (int np = 0; np < L_HID / 16; np++) {
                // B = Wh (k = j, n = c) from Wh stored [j][c]: transposed loads,
                // matrix m: rows j = (m & 1) * 8 + lane % 8, cols c = 16 np + (m >> 1) * 8
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(smem_addr(&S.wh[(am & 1) * 8 + (lane & 7)][np * 16 + (am >> 1) * 8]), b0, b1, b2, b3);
                float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};
                mma16816(d0, ah[0], ah[1], ah[2], ah[3], b0, b1);
                mma16816(d0, al[0], al[1], al[2], al[3], b0, b1);
                mma16816(d1, ah[0], ah[1], ah[2], ah[3], b2, b3);
                mma16816(d1, al[0], al[1], al[2], al[3], b2, b3);
#pragma unroll
                for (int t = 0; t < 2; t++) {
                    const float *d = t ? d1 : d0;
                    const int c = np * 16 + t * 8 + 2 * q;
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        __nv_bfloat162 *cell = reinterpret_cast<__nv_bfloat162 *>(&S.h2[wr + g + 8 * h][c]);
                        const float2 hv = __bfloat1622float2(*cell);
                        const float x = hv.x > 0.f ? d[2 * h] : 0.f, y = hv.y > 0.f ? d[2 * h + 1] : 0.f;
                        *cell = __floats2bfloat162_rn(x, y);
                    }
                }
            }
        }
        __syncthreads();
        // ---- dbh (threads 0-12), db2 (two columns per thread), dh2 and dh2^T out
        if (tid < L_NOUT)
            for (int r = 0; r < M_ROWS; r++) acc_bh += S.dhf[r][tid];
        if (a.dh2) {
            for (int i = tid; i < M_ROWS * (L_HID / 8); i += blockDim.x) {
                const int r = i / (L_HID / 8), c = (i % (L_HID / 8)) * 8;
                if (r0 + r < a.n)
                    *reinterpret_cast<uint4 *>(a.dh2 + (size_t)(r0 + r) * L_HID + c) =
                        *reinterpret_cast<const uint4 *>(&S.h2[r][c]);
            }
        }
        {
            // thread t owns columns 2t, 2t+1: sums them (db2) and writes their
            // transposed rows in 8-sample chunks
#pragma unroll 1
            for (int ch = 0; ch < M_ROWS / 8; ch++) {
                __align__(16) __nv_bfloat16 o0[8], o1[8];
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162 *>(&S.h2[ch * 8 + j][2 * tid]);
                    o0[j] = v.x;
                    o1[j] = v.y;
                    const float2 f = __bfloat1622float2(v);
                    acc_b2[0] += f.x;
                    acc_b2[1] += f.y;
                }
                const int rb = r0 + ch * 8;
                if (a.dh2t && rb < a.n) {
                    if (rb + 8 <= a.n) {
                        *reinterpret_cast<uint4 *>(a.dh2t + (size_t)(2 * tid) * a.ldt + rb) = *reinterpret_cast<uint4 *>(o0);
                        *reinterpret_cast<uint4 *>(a.dh2t + (size_t)(2 * tid + 1) * a.ldt + rb) =
                            *reinterpret_cast<uint4 *>(o1);
                    } else {
                        for (int j = 0; j < 8 && rb + j < a.n; j++) {
                            a.dh2t[(size_t)(2 * tid) * a.ldt + rb + j] = o0[j];
                            a.dh2t[(size_t)(2 * tid + 1) * a.ldt + rb + j] = o1[j];
                        }
                    }
                }
            }
        }
    }
    // ---- block partials: dWh [13][256], dbh [13], db2 [256], terms [8]
    float *out = a.part + (size_t)blockIdx.x * L_PART;
#pragma unroll
    for (int nt = 0; nt < 8; nt++) {
        const int c = warp * 64 + nt * 8 + 2 * q;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int j = g + 8 * h;
            if (j < L_NOUT) {
                out[j * L_HID + c] = acc_w[nt][2 * h];
                out[j * L_HID + c + 1] = acc_w[nt][2 * h + 1];
            }
        }
    }
    if (tid < L_NOUT) out[L_NOUT * L_HID + tid] = acc_bh;
    out[L_NOUT * L_HID + L_NOUT + 2 * tid] = acc_b2[0];
    out[L_NOUT * L_HID + L_NOUT + 2 * tid + 1] = acc_b2[1];
    // loss terms: q == 0 lanes hold them; warp sums, then warps in order
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        t_pg += __shfl_xor_sync(FULL, t_pg, o);
        t_vf += __shfl_xor_sync(FULL, t_vf, o);
        t_ent += __shfl_xor_sync(FULL, t_ent, o);
        t_clip += __shfl_xor_sync(FULL, t_clip, o);
        t_kl += __shfl_xor_sync(FULL, t_kl, o);
    }
    if (lane == 0) {
        S.terms[warp][0] = t_pg;
        S.terms[warp][1] = t_vf;
        S.terms[warp][2] = t_ent;
        S.terms[warp][3] = t_clip;
        S.terms[warp][4] = t_kl;
    }
    __syncthreads();
    if (tid < 8) {
        float v = 0.f;
        if (tid < 5)
            for (int w = 0; w < M_WARPS; w++) v += S.terms[w][tid];
        out[L_NOUT * L_HID + L_NOUT + L_HID + tid] = v;
    }
}

// out[i] = sum over splits of slabs[s][i] (split-K partial products), i < count.
// A block owns 64 float4 columns and G = blockDim.x / 64 groups of threads
// (G grows with the number of slabs, up to 4); group y adds slabs y, y+G, ...
// of its column, and the group sums are added in group order, so the result
// does not depend on scheduling.
constexpr int RS_COLS = 64, RS_GROUPS = 4;
__global__ void __launch_bounds__(RS_COLS * RS_GROUPS) reduce_slabs_kernel(const float *__restrict__ slabs, int splits,
                                                                          int64_t count, float *out) {
    __shared__ float4 part[RS_GROUPS][RS_COLS];
    const int cx = threadIdx.x % RS_COLS, gy = threadIdx.x / RS_COLS, groups = blockDim.x / RS_COLS;
    const int64_t i4 = (int64_t)blockIdx.x * RS_COLS + cx;
    const bool vec = (count & 3) == 0;
    const int64_t n4 = vec ? count / 4 : count;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i4 < n4) {
        for (int k = gy; k < splits; k += groups) {
            if (vec) {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(slabs + (size_t)k * count) + i4);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            } else {
                acc.x += slabs[(size_t)k * count + i4];
            }
        }
    }
    part[gy][cx] = acc;
    __syncthreads();
    if (gy == 0 && i4 < n4) {
        float4 t = part[0][cx];
        for (int g = 1; g < groups; g++) {
            t.x += part[g][cx].x;
            t.y += part[g][cx].y;
            t.z += part[g][cx].z;
            t.w += part[g][cx].w;
        }
        if (vec) reinterpret_cast<float4 *>(out)[i4] = t;
        else out[i4] = t.x;
    }
}

// ------------------------------------------------------------------ optimizer
// Adam (torch.optim.Adam semantics) on fp32 masters with the gradient scaled by
// min(1, max_norm / (||g|| + 1e-6)) (torch.nn.utils.clip_grad_norm_). Segments
// that feed the GEMMs are also written as bf16 copies: seg_bf16[i] (same
// layout) and, when seg_t is given, transposed [cols, rows] for W2^T.
struct AdamSeg {
    int64_t offset, count;
    int rows, cols;
    __nv_bfloat16 *bf16, *bf16_t;
};
struct AdamArgs {
    float *param, *grad, *m, *v;
    float lr, beta1, beta2, eps, max_norm;
    AdamSeg seg[8];
    int nseg;
    int64_t total;
};
// Four elements per thread (float4 loads and stores of the four fp32 arrays);
// the bf16 compute copies are written element by element.
__device__ __forceinline__ float adam_one(const AdamArgs &a, float g, float &m, float &v, float p, float scale,
                                          float bc1, float bc2_sqrt) {
    g *= scale;
    m = a.beta1 * m + (1.f - a.beta1) * g;
    v = a.beta2 * v + (1.f - a.beta2) * g * g;
    const float denom = sqrtf(v) / bc2_sqrt + a.eps;
    return p - (a.lr / bc1) * m / denom;
}
__device__ __forceinline__ void adam_copies(const AdamArgs &a, int64_t i, float p) {
    for (int s = 0; s < a.nseg; s++) {
        const AdamSeg &g2 = a.seg[s];
        if (i >= g2.offset && i < g2.offset + g2.count) {
            const int64_t j = i - g2.offset;
            const __nv_bfloat16 pb = __float2bfloat16_rn(p);
            if (g2.bf16) g2.bf16[j] = pb;
            if (g2.bf16_t) {
                const int r = (int)(j / g2.cols), c = (int)(j % g2.cols);
                g2.bf16_t[(size_t)c * g2.rows + r] = pb;
            }
        }
    }
}
__global__ void counter_add_kernel(int64_t *c, int64_t delta) { *c += delta; }

// ------------------------------------------------------------------ epoch permutation
// perm[i] = P(i) for a keyed bijection P of [0, n): an alternating Feistel
// network over the m-bit words, 2^m the smallest power of two >= n (a high half
// of floor(m/2) bits and a low half of ceil(m/2) bits, at most 20 each; each
// round XORs one half with a hash of the other half and a round key, so every
// round and their composition are bijections), walked until it lands in
// [0, n). The walk follows i's cycle of the bijection of [0, 2^m), which
// returns to i < n, so it ends; 2^m < 2n makes the expected walk under two
// applications. Round hash: the murmur3 32-bit finaliser (Appleby) of
// (round key ^ half); round keys: the splitmix64 finaliser (Steele, Lea and
// Flood, 2014) of the key plus the round number. The key mixes the caller's
// seed with an epoch count read on the device, so a captured epoch draws a
// fresh permutation on every replay (the caller advances the count with
// d1_counter_add).
constexpr int PERM_ROUNDS = 6;
__device__ __forceinline__ uint64_t perm_hash64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint32_t perm_hash32(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    return h ^ (h >> 16);
}
__global__ void permute_kernel(int64_t *perm, int64_t n, int m, uint64_t seed, const int64_t *epoch) {
    const uint64_t key = perm_hash64(seed ^ perm_hash64((uint64_t)*epoch + 0x9e3779b97f4a7c15ull));
    uint32_t rk[PERM_ROUNDS];
#pragma unroll
    for (int r = 0; r < PERM_ROUNDS; r++) rk[r] = (uint32_t)perm_hash64(key + (uint64_t)r);
    const int hb = m / 2, lb = m - hb;
    const uint32_t hmask = (uint32_t)((1ull << hb) - 1ull), lmask = (uint32_t)((1ull << lb) - 1ull);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t x = (uint64_t)i;
        do {
            uint32_t hi = (uint32_t)(x >> lb), lo = (uint32_t)x & lmask;
#pragma unroll
            for (int r = 0; r < PERM_ROUNDS; r += 2) {
                hi ^= perm_hash32(rk[r] ^ lo) & hmask;
                lo ^= perm_hash32(rk[r + 1] ^ hi) & lmask;
            }
            x = ((uint64_t)hi << lb) | lo;
        } while (x >= (uint64_t)n);
        perm[i] = (int64_t)x;
    }
}

// ------------------------------------------------------------------ fused optimizer step
// One launch for the end of a minibatch: (1) reduce the gradient's partial
// products into the flat gradient, (2) its global sum of squares, (3) grid
// barrier, (4) clip + Adam + bf16 copies, with the step counter advanced on the
// device. Job j: element e < rows * cols_in of every partial p < nsrc sits at
// src[p * stride + e]; element (r, c) goes to dst[r * cols_out + c] when
// c < cols_out, to dst_extra[r] when c == cols_out (a bias carried as an extra
// product column), else nowhere. A block owns 32 consecutive elements of a
// job at a time; its 8 warps sum the partials p = warp, warp + 8, ... and the
// warp sums are added in warp order, so the result does not depend on
// scheduling. Without jobs (the multi-GPU path, after the gradient
// all-reduce) step (1) is skipped and (2) reads the gradient.
constexpr int STEP_BLOCKS_PER_SM = 4, STEP_MAX_JOBS = 4, STEP_MAX_BLOCKS = 2048;
struct StepJob {
    const float *src;
    int64_t stride;
    int nsrc, rows, cols_in, cols_out, in_norm;
    float *dst, *dst_extra;
    int64_t chunk_begin;
    int vec;  // 4: float4 loads (a chunk is 128 elements), 1: scalar (32)
};
constexpr int PEER_MAX = 8;
struct StepArgs {
    StepJob job[STEP_MAX_JOBS];
    int njobs;
    int64_t chunks, wide_chunks;  // chunks of all jobs; of the leading jobs with > 16 partials
    const float *grad;  // without jobs: the gradient whose sum of squares is taken
    int64_t total;
    int norm;           // write this block's sum of squares to g_step_part[block]
    // Peer exchange (multi-GPU): job writes that fall in the flat gradient
    // [remap_from, remap_from + remap_len) go to half (epoch & 1) of this rank's
    // exchange buffer instead, and the last block to finish tells every peer
    // (flag[rank] = epoch in the peer's flag array, a system-scope release).
    const float *remap_from;
    int64_t remap_len, xstride;
    float *xbuf;
    const int64_t *epoch_src;  // epoch = *epoch_src + 1 (the optimizer's step count)
    unsigned long long *peer_flags[PEER_MAX];
    int world, rank;
    // two-phase exchange: element e of the flat gradient goes to slot
    // [half][rank][e - j * slice] of rank j = e / slice's inbox (a peer store)
    float *inbox[PEER_MAX];
    int64_t slice;
    int two_phase;
};
__device__ double g_step_part[STEP_MAX_BLOCKS];
__device__ unsigned g_step_ticket, g_peer_ticket;
// g_peer_error: sticky, read and cleared by the host (d1_peer_error).
// g_peer_abort: this step's verdict, cleared by the step's reduction launch,
// set by any all-reduce block that gave up waiting; the Adam launch then
// leaves the parameters, moments and step count untouched.
__device__ int g_peer_error, g_peer_abort;

struct Remap {
    const float *from;
    float *to;
    int64_t len;
    // two-phase: the owners' inboxes, the slice length, this rank's slot offset
    float *const *inbox;
    int64_t slice, slot;
};
__device__ __forceinline__ float *remap(const Remap &m, float *p) {
    if (!(m.to && p >= m.from && p < m.from + m.len)) return p;
    const int64_t off = p - m.from;
    if (!m.inbox) return m.to + off;
    const int64_t j = off / m.slice;
    return m.inbox[j] + m.slot + (off - j * m.slice);
}
// Sum of partials p = first, first + step, ... of the chunk's elements (vec of
// them per lane); returns the lane's first element index.
__device__ __forceinline__ int64_t chunk_partial(const StepJob &jb, int64_t ch, int lane, int first, int step,
                                                 float4 &sum) {
    const int vw = jb.vec;
    const int64_t e = ((ch - jb.chunk_begin) * 32 + lane) * vw, n_el = (int64_t)jb.rows * jb.cols_in;
    sum = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e < n_el) {
        if (vw == 4) {
#pragma unroll 8
            for (int pp = first; pp < jb.nsrc; pp += step) {
                const float4 q = __ldg(reinterpret_cast<const float4 *>(jb.src + (size_t)pp * jb.stride + e));
                sum.x += q.x;
                sum.y += q.y;
                sum.z += q.z;
                sum.w += q.w;
            }
        } else {
            // scalar rows (the loss partials: 256 of them, 32 per warp): one
            // batch of loads in flight instead of four
#pragma unroll 32
            for (int pp = first; pp < jb.nsrc; pp += step) sum.x += __ldg(jb.src + (size_t)pp * jb.stride + e);
        }
    }
    return e;
}
// Writes the lane's summed elements where the job sends them; returns their
// sum of squares when the job counts toward the gradient norm.
__device__ __forceinline__ double chunk_store(const StepJob &jb, int64_t e, float4 t4, const Remap &rm) {
    const int64_t n_el = (int64_t)jb.rows * jb.cols_in;
    const float t[4] = {t4.x, t4.y, t4.z, t4.w};
    double sq = 0.0;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        if (k >= jb.vec || e + k >= n_el) break;
        const int64_t ek = e + k;
        const int r = (int)(ek / jb.cols_in), c = (int)(ek - (int64_t)r * jb.cols_in);
        bool kept = false;
        if (c < jb.cols_out) {
            *remap(rm, jb.dst + (size_t)r * jb.cols_out + c) = t[k];
            kept = true;
        } else if (c == jb.cols_out && jb.dst_extra) {
            *remap(rm, jb.dst_extra + r) = t[k];
            kept = true;
        }
        if (kept && jb.in_norm) sq += (double)t[k] * t[k];
    }
    return sq;
}

__global__ void __launch_bounds__(256) grad_reduce_kernel(const __grid_constant__ StepArgs a) {
    pdl_wait();  // before any global access: the slabs come from the previous kernels
    __shared__ float4 ps[8][32];
    __shared__ double ws[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t epoch = a.xbuf ? (uint64_t)(*a.epoch_src + 1) : 0;
    const Remap rm{a.remap_from, a.xbuf ? a.xbuf + (epoch & 1) * a.xstride : nullptr, a.remap_len,
                   a.two_phase ? a.inbox : nullptr, a.slice,
                   ((int64_t)(epoch & 1) * a.world + a.rank) * a.slice};
    if (a.xbuf && blockIdx.x == 0 && threadIdx.x == 0) g_peer_abort = 0;
    double sq = 0.0;
    if (a.njobs > 0) {
        // jobs with many partials: a block per chunk, its 8 warps splitting the partials
        for (int64_t ch = blockIdx.x; ch < a.wide_chunks; ch += gridDim.x) {
            int j = 0;
            while (j + 1 < a.njobs && ch >= a.job[j + 1].chunk_begin) j++;
            const StepJob &jb = a.job[j];
            float4 sum;
            const int64_t e = chunk_partial(jb, ch, lane, warp, 8, sum);
            ps[warp][lane] = sum;
            __syncthreads();
            if (warp == 0) {
                float4 t = ps[0][lane];
#pragma unroll
                for (int w = 1; w < 8; w++) {
                    const float4 q = ps[w][lane];
                    t.x += q.x;
                    t.y += q.y;
                    t.z += q.z;
                    t.w += q.w;
                }
                sq += chunk_store(jb, e, t, rm);
            }
            __syncthreads();
        }
        // jobs with few partials: a warp per chunk, no block synchronisation
        const int64_t warps = (int64_t)gridDim.x * 8;
        for (int64_t ch = a.wide_chunks + (int64_t)blockIdx.x * 8 + warp; ch < a.chunks; ch += warps) {
            int j = 0;
            while (j + 1 < a.njobs && ch >= a.job[j + 1].chunk_begin) j++;
            const StepJob &jb = a.job[j];
            float4 t;
            const int64_t e = chunk_partial(jb, ch, lane, 0, 1, t);
            sq += chunk_store(jb, e, t, rm);
        }
    } else {
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.total; i += (int64_t)gridDim.x * blockDim.x) {
            const float g = a.grad[i];
            sq += (double)g * g;
        }
    }
    if (a.xbuf) {
        // the last block to finish publishes this rank's gradient to the peers
        __shared__ unsigned last;
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence_system();
            last = atomicAdd(&g_peer_ticket, 1u) == gridDim.x - 1;
        }
        __syncthreads();
        if (last && threadIdx.x < 32) {
            // one system-scope fence, then lane p raises peer p's flag (a fence
            // followed by relaxed stores is a release of everything before it)
            if (threadIdx.x == 0) g_peer_ticket = 0;
            __threadfence_system();
#pragma unroll
            for (int p = 0; p < PEER_MAX; p++)  // static indices: the flag pointers stay in the parameter space
                if (p == (int)threadIdx.x && p < a.world && p != a.rank)
                    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a.peer_flags[p] + a.rank), "l"(epoch)
                                 : "memory");
        }
    }
    if (!a.norm) return;
    // block partial of the sum of squares (fixed shuffle tree, then warp order)
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(FULL, sq, o);
    if (lane == 0) ws[warp] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; w++) t += ws[w];
        g_step_part[blockIdx.x] = t;
    }
}

// Cross-rank mean of the gradient through peer memory (one shot): every block
// first waits (bounded) until each peer has flagged this epoch, then sums a
// contiguous range of all ranks' exchange buffers in rank order, divides by the
// world size, writes the flat gradient and its block partial of the sum of
// squares. A wait that gives up (after wait_limit polls) sets g_peer_error
// (d1_peer_error) and g_peer_abort, and leaves the block's range as it was;
// the Adam launch that follows then changes nothing.
struct PeerArgs {
    const float *xbuf[PEER_MAX];  // each rank's exchange buffer (this rank's is local)
    // NVLS: the exchange buffers' multicast address; when set, each block reads
    // the sum over the ranks with multimem.ld_reduce (the switch adds) instead
    // of reading every peer's buffer
    const float *mc;
    int64_t xstride;
    const unsigned long long *flags;  // this rank's flag array, written by the peers
    const int64_t *epoch_src;
    float *grad;
    int64_t total;
    int world, rank;
    uint32_t wait_limit;
};
constexpr uint32_t PEER_WAIT_LIMIT = 1u << 24;  // default: ~1 s of 64 ns polls
__global__ void __launch_bounds__(256) peer_allreduce_kernel(const __grid_constant__ PeerArgs a) {
    pdl_wait();  // before any global access: this rank's reduced gradient comes from the previous kernel
    __shared__ int ok;
    __shared__ double ws[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t epoch = (uint64_t)(*a.epoch_src + 1);
    if (threadIdx.x == 0) {
        int good = 1;
        for (int p = 0; p < a.world && good; p++) {
            if (p == a.rank) continue;
            for (uint32_t it = 0;; it++) {
                unsigned long long v;
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(a.flags + p) : "memory");
                if (v >= epoch) break;
                if (it >= a.wait_limit) {
                    good = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        if (!good) {
            atomicExch(&g_peer_error, 1);
            atomicExch(&g_peer_abort, 1);
        }
        ok = good;
    }
    __syncthreads();
    double sq = 0.0;
    if (ok) {
        const int64_t half = (int64_t)(epoch & 1) * a.xstride;
        const int64_t n4 = (a.total + 3) / 4, per = (n4 + gridDim.x - 1) / gridDim.x;
        const int64_t q0 = (int64_t)blockIdx.x * per, q1 = q0 + per < n4 ? q0 + per : n4;
        const float inv = (float)a.world;
        for (int64_t q = q0 + threadIdx.x; q < q1; q += blockDim.x) {
            float4 t;
            if (a.mc) {
                asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                             : "=f"(t.x), "=f"(t.y), "=f"(t.z), "=f"(t.w)
                             : "l"(reinterpret_cast<const float4 *>(a.mc + half) + q)
                             : "memory");
            } else {
                // every rank's value is loaded before the first add (one NVLink
                // round trip, not one per rank); the adds keep rank order
                float4 v[PEER_MAX];
#pragma unroll
                for (int r = 0; r < PEER_MAX; r++)
                    if (r < a.world) v[r] = __ldcv(reinterpret_cast<const float4 *>(a.xbuf[r] + half) + q);
                t = v[0];
#pragma unroll
                for (int r = 1; r < PEER_MAX; r++)
                    if (r < a.world) {
                        t.x += v[r].x;
                        t.y += v[r].y;
                        t.z += v[r].z;
                        t.w += v[r].w;
                    }
            }
            const float f[4] = {__fdiv_rn(t.x, inv), __fdiv_rn(t.y, inv), __fdiv_rn(t.z, inv), __fdiv_rn(t.w, inv)};
#pragma unroll
            for (int k = 0; k < 4; k++)
                if (4 * q + k < a.total) {
                    a.grad[4 * q + k] = f[k];
                    sq += (double)f[k] * f[k];
                }
        }
    }
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(FULL, sq, o);
    if (lane == 0) ws[warp] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; w++) t += ws[w];
        g_step_part[blockIdx.x] = t;
    }
}

// Two-phase exchange, for more ranks: each rank owns a slice of the flat
// gradient. The reduction launch stores every rank's part of slice j straight
// into rank j's inbox (peer stores) and flags it; then each rank sums its own
// slice's inbox in rank order, divides by the world size and stores the result
// into every rank's gather area (peer stores) and flags that; then each rank
// copies the gathered slices into its flat gradient. Each rank moves 2 (world -
// 1) / world of the gradient over NVLink instead of reading (world - 1) copies.
// Buffer of rank p: inbox [2 halves][world][slice] floats, then gather
// [2][world][slice]; flags: u64 [8] for the first phase, [8] for the second.
struct Peer2Args {
    float *xbuf[PEER_MAX];                 // each rank's buffer (this rank's is local)
    unsigned long long *xflags[PEER_MAX];  // each rank's flag area
    const int64_t *epoch_src;
    float *grad;
    int64_t total, slice;
    int world, rank;
    uint32_t wait_limit;
};
__device__ unsigned g_peer2_ticket;
// Bounded wait by thread 0 for flag[p] >= epoch of every other rank; on a
// timeout records the error and this step's abort. Returns 1 when all arrived.
__device__ __forceinline__ int wait_peers(const unsigned long long *flag, int world, int rank, uint64_t epoch,
                                          uint32_t limit) {
    int good = 1;
    for (int p = 0; p < world && good; p++) {
        if (p == rank) continue;
        for (uint32_t it = 0;; it++) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag + p) : "memory");
            if (v >= epoch) break;
            if (it >= limit) {
                good = 0;
                break;
            }
            __nanosleep(64);
        }
    }
    if (!good) {
        atomicExch(&g_peer_error, 1);
        atomicExch(&g_peer_abort, 1);
    }
    return good;
}
// Every block counts itself in; the last one to finish raises flag[index] =
// epoch in every other rank's flag area (system-scope release after a system
// fence), unless a block of this step gave up waiting.
__device__ __forceinline__ void publish(unsigned long long *const *xflags, int index, int world, int rank,
                                        uint64_t epoch) {
    __shared__ unsigned last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        last = atomicAdd(&g_peer2_ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        g_peer2_ticket = 0;
        __threadfence_system();
        if (!*(volatile int *)&g_peer_abort)
            for (int p = 0; p < world; p++)
                if (p != rank)
                    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(xflags[p] + index), "l"(epoch)
                                 : "memory");
    }
}
__global__ void __launch_bounds__(256) peer_reduce2_kernel(const __grid_constant__ Peer2Args a) {
    pdl_wait();  // before any global access: this rank's reduced gradient comes from the previous kernel
    __shared__ int ok;
    const uint64_t epoch = (uint64_t)(*a.epoch_src + 1);
    const int64_t half = (int64_t)(epoch & 1);
    if (threadIdx.x == 0) ok = wait_peers(a.xflags[a.rank], a.world, a.rank, epoch, a.wait_limit);
    __syncthreads();
    // after a timeout nothing is published, so the peers' gathers run out too
    const float *inbox = a.xbuf[a.rank] + half * a.world * a.slice;
    const int64_t gather_slot = (2 + half) * a.world * a.slice + (int64_t)a.rank * a.slice;
    const int64_t n4 = a.slice / 4;
    const float inv = (float)a.world;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; ok && q < n4;
         q += (int64_t)gridDim.x * blockDim.x) {
        float4 t = __ldcv(reinterpret_cast<const float4 *>(inbox) + q);
        for (int r = 1; r < a.world; r++) {
            const float4 v = __ldcv(reinterpret_cast<const float4 *>(inbox + (int64_t)r * a.slice) + q);
            t.x += v.x;
            t.y += v.y;
            t.z += v.z;
            t.w += v.w;
        }
        const float4 f = make_float4(__fdiv_rn(t.x, inv), __fdiv_rn(t.y, inv), __fdiv_rn(t.z, inv),
                                     __fdiv_rn(t.w, inv));
        for (int j = 0; j < a.world; j++) reinterpret_cast<float4 *>(a.xbuf[j] + gather_slot)[q] = f;
    }
    publish(a.xflags, 8 + a.rank, a.world, a.rank, epoch);
}
__global__ void __launch_bounds__(256) peer_gather2_kernel(const __grid_constant__ Peer2Args a) {
    pdl_wait();  // before any global access: this rank's reduced gradient comes from the previous kernel
    __shared__ int ok;
    __shared__ double ws[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t epoch = (uint64_t)(*a.epoch_src + 1);
    const int64_t half = (int64_t)(epoch & 1);
    if (threadIdx.x == 0) ok = wait_peers(a.xflags[a.rank] + 8, a.world, a.rank, epoch, a.wait_limit);
    __syncthreads();
    double sq = 0.0;
    if (ok) {
        const float *gather = a.xbuf[a.rank] + (2 + half) * a.world * a.slice;
        const int64_t per = (a.total + gridDim.x - 1) / gridDim.x;
        const int64_t e0 = (int64_t)blockIdx.x * per, e1 = e0 + per < a.total ? e0 + per : a.total;
        for (int64_t e = e0 + threadIdx.x; e < e1; e += blockDim.x) {
            const int64_t j = e / a.slice;
            const float g = __ldcv(gather + j * a.slice + (e - j * a.slice));
            a.grad[e] = g;
            sq += (double)g * g;
        }
    }
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(FULL, sq, o);
    if (lane == 0) ws[warp] = sq;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; w++) t += ws[w];
        g_step_part[blockIdx.x] = t;
    }
}

// Adam after grad_reduce_kernel: the global sum of squares is the sum of that
// launch's block partials, added in block order by every block (so the clip
// coefficient is the same everywhere), and *step advances on the device. After
// a peer all-reduce (check_abort) that gave up waiting, nothing is updated.
__global__ void __launch_bounds__(256) adam_update_kernel(AdamArgs d, int nparts, int64_t *step, int check_abort) {
    pdl_wait();  // before any global access: the gradient and its norm partials come from the previous kernel
    __shared__ float sc[3];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (check_abort && *(volatile int *)&g_peer_abort) return;
    const int64_t step0 = *step;
    // warp 0: the norm from the block partials (unrolled, so the loads are in
    // flight together; the adds keep their fixed order); warp 1, meanwhile:
    // the bias corrections
    if (warp == 0) {
        double t = 0.0;
#pragma unroll 16
        for (int b = lane; b < nparts; b += 32) t += __ldcg(&g_step_part[b]);
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(FULL, t, o);
        if (lane == 0) {
            float scale = 1.f;
            if (d.max_norm > 0.f) {
                const float coef = d.max_norm / ((float)sqrt(t) + 1e-6f);
                if (coef < 1.f) scale = coef;
            }
            sc[2] = scale;
        }
    } else if (warp == 1 && lane == 0) {
        const double tstep = (double)(step0 + 1);
        sc[0] = (float)(1.0 - pow((double)d.beta1, tstep));
        sc[1] = (float)sqrt(1.0 - pow((double)d.beta2, tstep));
    }
    __syncthreads();
    const float bc1 = sc[0], bc2_sqrt = sc[1], scale = sc[2];
    const int64_t n4 = d.total / 4, stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4; q += stride) {
        const float4 g4 = reinterpret_cast<const float4 *>(d.grad)[q];
        float4 m4 = reinterpret_cast<const float4 *>(d.m)[q], v4 = reinterpret_cast<const float4 *>(d.v)[q];
        float4 p4 = reinterpret_cast<const float4 *>(d.param)[q];
        p4.x = adam_one(d, g4.x, m4.x, v4.x, p4.x, scale, bc1, bc2_sqrt);
        p4.y = adam_one(d, g4.y, m4.y, v4.y, p4.y, scale, bc1, bc2_sqrt);
        p4.z = adam_one(d, g4.z, m4.z, v4.z, p4.z, scale, bc1, bc2_sqrt);
        p4.w = adam_one(d, g4.w, m4.w, v4.w, p4.w, scale, bc1, bc2_sqrt);
        reinterpret_cast<float4 *>(d.m)[q] = m4;
        reinterpret_cast<float4 *>(d.v)[q] = v4;
        reinterpret_cast<float4 *>(d.param)[q] = p4;
        adam_copies(d, 4 * q, p4.x);
        adam_copies(d, 4 * q + 1, p4.y);
        adam_copies(d, 4 * q + 2, p4.z);
        adam_copies(d, 4 * q + 3, p4.w);
    }
    if (blockIdx.x == 0)
        for (int64_t i = 4 * n4 + threadIdx.x; i < d.total; i += blockDim.x) {
            float m = d.m[i], v = d.v[i];
            const float p = adam_one(d, d.grad[i], m, v, d.param[i], scale, bc1, bc2_sqrt);
            d.m[i] = m;
            d.v[i] = v;
            d.param[i] = p;
            adam_copies(d, i, p);
        }
    // every block has read *step above; the last block to finish advances it
    __shared__ unsigned last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(&g_step_ticket, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        *step = step0 + 1;
        g_step_ticket = 0;
    }
}

// Dynamic shared memory above 48 KB is opted into once per kernel and device;
// `ready` is that kernel's bitmask of devices already set up.
static int opt_in_smem(const void *fn, int bytes, uint64_t *ready) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 64 && (*ready >> dev) & 1) return 0;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess) return (int)e;
    if (dev < 64) *ready |= 1ull << dev;
    return 0;
}

}  // namespace ppo
}  // namespace d1

using namespace d1;


extern "C" {

int d1_ppo_gather_x(const void *obs, int F, const int64_t *idx, int n, void *x, int ldx, int ones_col,
                    void *stream) {
    if (!obs || !idx || !x || n <= 0 || F <= 0 || F % 8 || ldx % 8 || ldx < F + (ones_col ? 8 : 0) ||
        (reinterpret_cast<uintptr_t>(x) & 15))
        return D1_ERR_BAD_ARGUMENT;
    static uint64_t ready = 0;
    const int err = ppo::opt_in_smem((const void *)ppo::gather_kernel, ppo::G_SMEM, &ready);
    if (err) return err;
    const int groups = ((F + ppo::G_FEAT - 1) / ppo::G_FEAT + ppo::G_GROUP - 1) / ppo::G_GROUP;
    const dim3 grid((n + ppo::G_SAMPLES - 1) / ppo::G_SAMPLES, groups);
    ppo::gather_kernel<<<grid, 256, ppo::G_SMEM, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)obs, F, idx, n, (__nv_bfloat16 *)x, ldx, ones_col != 0);
    return (int)cudaGetLastError();
}

int d1_ppo_gather_cobs(const void *cobs, const int64_t *idx, int n, void *x, int ldx, int ones_col, void *stream) {
    if (!cobs || !idx || !x || n <= 0 || ldx % 8 || ldx < 1832 + (ones_col ? 8 : 0) ||
        ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(cobs)) & 15))
        return D1_ERR_BAD_ARGUMENT;
    int blocks = (n + ppo::CG_WARPS - 1) / ppo::CG_WARPS;
    if (blocks > 148 * 16) blocks = 148 * 16;
    ppo::gather_cobs_kernel<<<blocks, ppo::CG_WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)cobs, idx, n, (uint4 *)x, ldx / 8, ones_col != 0);
    return (int)cudaGetLastError();
}

int d1_ppo_loss_part_len(void) { return ppo::L_PART; }

int d1_ppo_loss(const void *h2, const void *wh, const float *bh, const int64_t *idx, const uint16_t *legal,
                const int64_t *action, const float *old_logp, const float *adv, const float *ret,
                const float *old_value, const double *adv_stats, double adv_count, int n, float clip, float vclip,
                float vf_coef, float ent_coef, void *dh2, void *dh2t, int ldt, float *part, int blocks,
                void *stream) {
    if (n <= 0 || blocks <= 0 || !h2 || !wh || !bh || !idx || !legal || !action || !old_logp || !adv || !ret ||
        !old_value || !adv_stats || !part || adv_count < 2 || (dh2t && ldt < n))
        return D1_ERR_BAD_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(h2) | reinterpret_cast<uintptr_t>(wh)) & 15) return D1_ERR_BAD_ARGUMENT;
    if (dh2t && (ldt % 8 || reinterpret_cast<uintptr_t>(dh2t) & 15)) return D1_ERR_BAD_ARGUMENT;
    static uint64_t ready = 0;
    const int err = ppo::opt_in_smem((const void *)ppo::loss_mma_kernel, (int)sizeof(ppo::MmaSmem), &ready);
    if (err) return err;
    ppo::LossArgs a{(const __nv_bfloat16 *)h2, (const __nv_bfloat16 *)wh, bh, idx, legal, action, old_logp, adv,
                    ret, old_value, adv_stats, adv_count, n, clip, vclip, vf_coef, ent_coef,
                    (__nv_bfloat16 *)dh2, (__nv_bfloat16 *)dh2t, ldt, part};
    ppo::loss_mma_kernel<<<blocks, ppo::M_WARPS * 32, sizeof(ppo::MmaSmem), (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}

int d1_reduce_slabs(const float *slabs, int splits, int64_t count, float *out, void *stream) {
    if (!slabs || !out || splits <= 0 || count <= 0) return D1_ERR_BAD_ARGUMENT;
    const int64_t n = (count & 3) == 0 ? count / 4 : count;
    const int groups = splits >= 32 ? ppo::RS_GROUPS : splits >= 16 ? 2 : 1;
    ppo::reduce_slabs_kernel<<<(unsigned)((n + ppo::RS_COLS - 1) / ppo::RS_COLS), ppo::RS_COLS * groups, 0,
                               (cudaStream_t)stream>>>(slabs, splits, count, out);
    return (int)cudaGetLastError();
}

struct PeerSetup {
    void *const *xbufs;
    void *const *flags;
    int64_t xstride;  // one-shot: half length; two-phase: slice length
    int world, rank;
    int two_phase;
    const void *mc;   // one-shot over NVLS: the exchange buffers' multicast address
};

static int step_launch(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                       float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                       const D1AdamSegment *segs, int nseg, int do_adam, void *stream, const PeerSetup *peer = nullptr,
                       uint32_t wait_limit = 0) {
    using namespace ppo;
    if (njobs < 0 || njobs > STEP_MAX_JOBS || (njobs > 0 && !jobs) || (!do_adam && njobs == 0)) return D1_ERR_BAD_ARGUMENT;
    if (peer && (njobs == 0 || !do_adam || peer->world < 2 || peer->world > PEER_MAX || peer->rank < 0 ||
                 peer->rank >= peer->world || !peer->xbufs || !peer->flags || peer->xstride % 4 || !step ||
                 (peer->two_phase ? peer->xstride * peer->world < total : peer->xstride < total)))
        return D1_ERR_BAD_ARGUMENT;
    StepArgs a;
    memset(&a, 0, sizeof(a));
    int64_t chunks = 0;
    int order[STEP_MAX_JOBS], n_ord = 0;
    for (int j = 0; j < njobs; j++)
        if (jobs[j].nsrc > 16) order[n_ord++] = j;
    const int n_wide = n_ord;
    for (int j = 0; j < njobs; j++)
        if (jobs[j].nsrc <= 16) order[n_ord++] = j;
    for (int jj = 0; jj < njobs; jj++) {
        const D1GradJob &q = jobs[order[jj]];
        if (!q.src || !q.dst || q.nsrc <= 0 || q.rows <= 0 || q.cols_in <= 0 || q.cols_out <= 0 ||
            q.cols_out > q.cols_in || q.stride < (int64_t)q.rows * q.cols_in)
            return D1_ERR_BAD_ARGUMENT;
        const int vec = ((q.cols_in | q.cols_out) % 4 == 0 && q.stride % 4 == 0 &&
                         (reinterpret_cast<uintptr_t>(q.src) & 15) == 0) ? 4 : 1;
        a.job[jj] = StepJob{q.src, q.stride, q.nsrc, q.rows, q.cols_in, q.cols_out, q.in_norm, q.dst, q.dst_extra,
                            chunks, vec};
        chunks += ((int64_t)q.rows * q.cols_in + 32 * vec - 1) / (32 * vec);
        if (jj + 1 == n_wide) a.wide_chunks = chunks;
    }
    a.njobs = njobs;
    a.chunks = chunks;
    a.norm = do_adam && !peer;
    PeerArgs pa;
    memset(&pa, 0, sizeof(pa));
    Peer2Args p2;
    memset(&p2, 0, sizeof(p2));
    if (peer) {
        a.remap_from = grad;
        a.remap_len = total;
        a.xstride = peer->xstride;
        a.xbuf = (float *)peer->xbufs[peer->rank];
        a.epoch_src = step;
        a.world = peer->world;
        a.rank = peer->rank;
        for (int i = 0; i < peer->world; i++) {
            if (!peer->xbufs[i] || !peer->flags[i] || (reinterpret_cast<uintptr_t>(peer->xbufs[i]) & 15))
                return D1_ERR_BAD_ARGUMENT;
            a.peer_flags[i] = (unsigned long long *)peer->flags[i];
            pa.xbuf[i] = (const float *)peer->xbufs[i];
        }
        pa.xstride = peer->xstride;
        pa.mc = (const float *)peer->mc;
        pa.flags = (const unsigned long long *)peer->flags[peer->rank];
        pa.epoch_src = step;
        pa.grad = grad;
        pa.total = total;
        pa.world = peer->world;
        pa.rank = peer->rank;
        pa.wait_limit = wait_limit ? wait_limit : PEER_WAIT_LIMIT;
        if (peer->two_phase) {
            a.two_phase = 1;
            a.slice = peer->xstride;
            for (int i = 0; i < peer->world; i++) {
                a.inbox[i] = (float *)peer->xbufs[i];
                p2.xbuf[i] = (float *)peer->xbufs[i];
                p2.xflags[i] = (unsigned long long *)peer->flags[i];
            }
            p2.epoch_src = step;
            p2.grad = grad;
            p2.total = total;
            p2.slice = peer->xstride;
            p2.world = peer->world;
            p2.rank = peer->rank;
            p2.wait_limit = pa.wait_limit;
        }
    }
    AdamArgs d;
    if (do_adam) {
        if (!param || !grad || !m || !v || !step || total <= 0 || nseg < 0 || nseg > 8) return D1_ERR_BAD_ARGUMENT;
        if ((reinterpret_cast<uintptr_t>(param) | reinterpret_cast<uintptr_t>(grad) | reinterpret_cast<uintptr_t>(m) |
             reinterpret_cast<uintptr_t>(v)) & 15)
            return D1_ERR_BAD_ARGUMENT;
        a.grad = grad;
        a.total = total;
        d.param = param;
        d.grad = grad;
        d.m = m;
        d.v = v;
        d.lr = lr;
        d.beta1 = beta1;
        d.beta2 = beta2;
        d.eps = eps;
        d.max_norm = max_norm;
        d.nseg = nseg;
        d.total = total;
        for (int i = 0; i < nseg; i++)
            d.seg[i] = AdamSeg{segs[i].offset, segs[i].count, segs[i].rows, segs[i].cols,
                               (__nv_bfloat16 *)segs[i].bf16, (__nv_bfloat16 *)segs[i].bf16_t};
    }
    int dev = 0, sms = 0;
    if (cudaError_t e = cudaGetDevice(&dev)) return (int)e;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    int blocks = sms * STEP_BLOCKS_PER_SM;
    if (blocks > STEP_MAX_BLOCKS) blocks = STEP_MAX_BLOCKS;
    // the reduction, the peer exchange and Adam launch with programmatic
    // overlap of the previous kernel's end (each pdl_wait first)
    cudaLaunchAttribute attr;
    const cudaLaunchConfig_t cfg = pdl_config(dim3(blocks), dim3(256), 0, (cudaStream_t)stream, &attr);
    if (cudaError_t e = cudaLaunchKernelEx(&cfg, grad_reduce_kernel, a)) return (int)e;
    if (peer && peer->two_phase) {
        if (cudaError_t e = cudaLaunchKernelEx(&cfg, peer_reduce2_kernel, p2)) return (int)e;
        if (cudaError_t e = cudaLaunchKernelEx(&cfg, peer_gather2_kernel, p2)) return (int)e;
    } else if (peer) {
        if (cudaError_t e = cudaLaunchKernelEx(&cfg, peer_allreduce_kernel, pa)) return (int)e;
    }
    if (do_adam) {
        const int abort_check = peer ? 1 : 0;
        if (cudaError_t e = cudaLaunchKernelEx(&cfg, adam_update_kernel, d, blocks, step, abort_check)) return (int)e;
    }
    return (int)cudaGetLastError();
}

int d1_ppo_step(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step, const D1AdamSegment *segs,
                int nseg, void *stream) {
    return step_launch(jobs, njobs, param, grad, m, v, total, lr, beta1, beta2, eps, max_norm, step, segs, nseg, 1,
                       stream);
}

int d1_ppo_step_peer(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                     float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                     const D1AdamSegment *segs, int nseg, void *const *xbufs, void *const *flags, int64_t xstride,
                     int world, int rank, unsigned wait_limit, void *stream) {
    const PeerSetup peer{xbufs, flags, xstride, world, rank, 0};
    return step_launch(jobs, njobs, param, grad, m, v, total, lr, beta1, beta2, eps, max_norm, step, segs, nseg, 1,
                       stream, &peer, wait_limit);
}

int d1_ppo_step_nvls(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                     float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                     const D1AdamSegment *segs, int nseg, void *const *xbufs, void *const *flags, int64_t xstride,
                     const void *mc, int world, int rank, unsigned wait_limit, void *stream) {
    if (!mc || (reinterpret_cast<uintptr_t>(mc) & 15)) return D1_ERR_BAD_ARGUMENT;
    const PeerSetup peer{xbufs, flags, xstride, world, rank, 0, mc};
    return step_launch(jobs, njobs, param, grad, m, v, total, lr, beta1, beta2, eps, max_norm, step, segs, nseg, 1,
                       stream, &peer, wait_limit);
}

int d1_ppo_step_peer2(const D1GradJob *jobs, int njobs, float *param, float *grad, float *m, float *v, int64_t total,
                      float lr, float beta1, float beta2, float eps, float max_norm, int64_t *step,
                      const D1AdamSegment *segs, int nseg, void *const *xbufs, void *const *flags, int64_t slice,
                      int world, int rank, unsigned wait_limit, void *stream) {
    const PeerSetup peer{xbufs, flags, slice, world, rank, 1};
    return step_launch(jobs, njobs, param, grad, m, v, total, lr, beta1, beta2, eps, max_norm, step, segs, nseg, 1,
                       stream, &peer, wait_limit);
}

// Exchange buffers: plain device allocations shared with the other ranks'
// processes through CUDA IPC handles (set-up time only, not the hot path).
int d1_peer_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int d1_peer_alloc(int64_t bytes, void **ptr, void *handle) {
    if (bytes <= 0 || !ptr || !handle) return D1_ERR_BAD_ARGUMENT;
    cudaError_t e = cudaMalloc(ptr, (size_t)bytes);
    if (e == cudaSuccess) e = cudaMemset(*ptr, 0, (size_t)bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle((cudaIpcMemHandle_t *)handle, *ptr);
    return (int)e;
}

int d1_peer_open(const void *handle, void **ptr) {
    if (!handle || !ptr) return D1_ERR_BAD_ARGUMENT;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

int d1_peer_close(void *ptr) { return ptr ? (int)cudaIpcCloseMemHandle(ptr) : D1_ERR_BAD_ARGUMENT; }

int d1_peer_free(void *ptr) { return ptr ? (int)cudaFree(ptr) : D1_ERR_BAD_ARGUMENT; }

// Nonzero when a peer all-reduce gave up waiting for a peer; reading clears it.
int d1_peer_error(void) {
    int h = 0, z = 0;
    if (cudaMemcpyFromSymbol(&h, ppo::g_peer_error, sizeof(int)) != cudaSuccess) return -1;
    if (h) cudaMemcpyToSymbol(ppo::g_peer_error, &z, sizeof(int));
    return h;
}

int d1_grad_reduce(const D1GradJob *jobs, int njobs, void *stream) {
    return step_launch(jobs, njobs, nullptr, nullptr, nullptr, nullptr, 0, 0.f, 0.f, 0.f, 0.f, 0.f, nullptr, nullptr, 0,
                       0, stream);
}

int d1_counter_add(int64_t *counter, int64_t delta, void *stream) {
    if (!counter) return D1_ERR_BAD_ARGUMENT;
    ppo::counter_add_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(counter, delta);
    return (int)cudaGetLastError();
}

int d1_ppo_permute(int64_t *perm, int64_t n, uint64_t seed, const int64_t *epoch, void *stream) {
    if (!perm || !epoch || n <= 0 || n > ((int64_t)1 << 40)) return D1_ERR_BAD_ARGUMENT;
    int m = 0;
    while (((int64_t)1 << m) < n) m++;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t want = (n + 255) / 256, cap = (int64_t)sms * 8;
    ppo::permute_kernel<<<(int)(want < cap ? want : cap), 256, 0, (cudaStream_t)stream>>>(perm, n, m, seed, epoch);
    return (int)cudaGetLastError();
}

int d1_gae(const float *reward, const float *done, int64_t r_step, int64_t r_env, const float *value, int T, int B,
           float gamma, float lambda, float *adv, float *ret, double *stats, int mode, void *stream) {
    if (T <= 0 || B <= 0 || !reward || !done || !value || !adv || !ret) return D1_ERR_BAD_ARGUMENT;
    ppo::GaeArgs a{reward, done, value, r_step, r_env, adv, ret, stats, T, B, gamma, (float)((double)gamma * lambda)};
    if (mode == 0 && stats && (B + 255) / 256 > ppo::RED_MAX_BLOCKS) return D1_ERR_TOO_LARGE;
    if (mode == 0) {
        ppo::gae_sequential_kernel<<<(B + 255) / 256, 256, 0, (cudaStream_t)stream>>>(a);
    } else {
        const bool pairs = r_env == 1 && B % 2 == 0 && r_step % 2 == 0 &&
                           ((uintptr_t)reward | (uintptr_t)done | (uintptr_t)value | (uintptr_t)adv |
                            (uintptr_t)ret) % 8 == 0;
        int sms = 148, dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int64_t groups = (B + 32 * (pairs ? 2 : 1) - 1) / (32 * (pairs ? 2 : 1));
        const int64_t cap = (int64_t)sms * ppo::SCAN_BLOCKS_PER_SM;
        const int blocks = (int)(groups < cap ? groups : cap);
        if (pairs)
            ppo::gae_scan_kernel<2><<<blocks, ppo::SCAN_WARPS * 32, 0, (cudaStream_t)stream>>>(a);
        else
            ppo::gae_scan_kernel<1><<<blocks, ppo::SCAN_WARPS * 32, 0, (cudaStream_t)stream>>>(a);
    }
    return (int)cudaGetLastError();
}

}  // extern "C"
