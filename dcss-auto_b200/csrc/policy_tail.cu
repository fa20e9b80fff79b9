// The rollout policy after layer 1 in one persistent launch on the
// 5th-generation tensor cores (sm_100a tcgen05 + TMA): layer 2, the
// policy/value head and the masked categorical draw for 128 rows per tile.
// It replaces the layer-2 GEMM and the head + sampler kernel of the unfused
// act() (two launches and an h2 round trip through memory).
//
//   h2     = relu(h1 W2^T + b2)            MMA M128 N256, K 256  (TMEM cols 0-255)
//   head   = h2 Wh^T + bh (12 logits, v)   MMA M128 N16, K 256   (cols 256-271)
//   draw   d1_sampler.cuh's sample_masked, one epilogue thread per row, so an
//          action equals the oracle's draw given the logits written here
//
// One CTA per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ... W2
// (128 KB) is loaded once per CTA and stays in shared memory beside one
// 128 x 256 bf16 tile, which holds h1 (TMA) and then h2 (written by the
// epilogue in the same 128-byte-swizzled layout the tensor cores read). As
// soon as the head MMA has read h2 the tile is handed back to TMA, so the next
// tile's h1 load overlaps the draw of this one.
//
// Warp roles (320 threads): warp 0 issues the TMA loads; warp 1 owns the TMEM
// allocation and one lane issues the MMAs; warps 2-9 are the epilogue, warp w
// reading TMEM lanes 32 (w % 4) .. +31 (tile rows) and column half (w - 2) / 4;
// the draw runs on the half-0 warps. Every mbarrier wait is bounded: on expiry
// the kernel records an error (read by d1_policy_tail_error), leaves its loop
// and still frees TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/d1.h"
#include "d1_pdl.cuh"
#include "d1_sampler.cuh"
#include "tc_ptx.cuh"

namespace d1 {
namespace ptail {
using namespace tcx;

__device__ int g_ptail_error;  // read and cleared by d1_policy_tail_error

constexpr int ROWS = 128, HID = 256, NOUT = 13, NACT = 12;
constexpr int EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t WAIT_LIMIT = 1u << 22;
// Shared memory, offsets from a 1024-byte aligned base.
constexpr int OFF_W2 = 0;       // W2 [kb 4][out 256][128 B], 128-byte swizzle
constexpr int OFF_X = 131072;   // activation tile [kb 4][row 128][128 B], 128-byte swizzle
constexpr int OFF_HB = 196608;  // Wh as the head's B [c/8 32][j 16][8 c] (no swizzle)
constexpr int OFF_B2 = 204800;  // b2 [256] f32
constexpr int OFF_BH = 205824;  // bh [16] f32
constexpr int OFF_BAR = 205888;  // 8 barriers, abort flag, TMEM slot
constexpr int SMEM = OFF_BAR + 128 + 1024;
constexpr uint32_t TMEM_ALLOC = 512, D_MAIN = 0, D_HEAD = 256;
constexpr uint32_t ID_L2 = idesc_bf16(128, 256, false, false), ID_HEAD = idesc_bf16(128, 16, false, false);

struct Args {
    const __nv_bfloat16 *wh;  // [13, 256]
    const float *b2, *bh;
    const uint16_t *legal;    // [n] (null: all 12 legal)
    uint64_t seed, step;
    const int64_t *step_dev;  // the step from device memory when not null
    int first_env, n, tiles;
    int64_t *action;               // null: no draw (value and logits only)
    float *logp, *value, *logits;  // logp, logits [n, 12] may be null
};

__device__ __forceinline__ uint32_t x_off(int row, int col) {
    return (uint32_t)(OFF_X + (col >> 6) * 16384 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__global__ void __launch_bounds__(THREADS, 1)
    policy_tail_kernel(const __grid_constant__ CUtensorMap map_h1, const __grid_constant__ CUtensorMap map_w2, Args a) {
    d1::pdl_wait();  // before any global access: h1 comes from the previous kernel
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(sm);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    // W2 landed; h1 tile landed; layer-2 accumulator ready; h2 written (and the
    // accumulator read); head accumulator ready; head results read; tile free
    const uint32_t bar_w2 = smem_u32(bars), bar_h1 = smem_u32(bars + 1), bar_acc = smem_u32(bars + 2),
                   bar_h2 = smem_u32(bars + 3), bar_head = smem_u32(bars + 4), bar_hfree = smem_u32(bars + 5),
                   bar_xfree = smem_u32(bars + 6);
    volatile int *abort_s = reinterpret_cast<volatile int *>(bars + 7);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 8);
    float *b2_s = reinterpret_cast<float *>(sm + OFF_B2), *bh_s = reinterpret_cast<float *>(sm + OFF_BH);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0 && lane == 0) {
        mbar_init(bar_w2, 1);
        mbar_init(bar_h1, 1);
        mbar_init(bar_acc, 1);
        mbar_init(bar_h2, EPI_WARPS);
        mbar_init(bar_head, 1);
        mbar_init(bar_hfree, EPI_WARPS);
        mbar_init(bar_xfree, 1);
        *abort_s = 0;
        mbar_init_fence();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TMEM_ALLOC)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA: W2 once, then each tile's h1 when the tile buffer is free
        if (lane == 0) {
            mbar_expect_tx(bar_w2, 131072);
            for (int kb = 0; kb < 4; kb++) tma_load_2d(base + OFF_W2 + kb * 32768, &map_w2, bar_w2, kb * 64, 0);
            int i = 0;
            for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, i++) {
                if (i > 0 && (!mbar_wait(bar_xfree, (uint32_t)(i - 1) & 1u, WAIT_LIMIT) || *abort_s)) {
                    atomicExch(&g_ptail_error, 1);
                    *abort_s = 1;
                    break;
                }
                mbar_expect_tx(bar_h1, 65536);
                for (int kb = 0; kb < 4; kb++)
                    tma_load_2d(base + OFF_X + kb * 16384, &map_h1, bar_h1, kb * 64, t * ROWS);
            }
            // every TMA write has landed before teardown (the last tile's, on the abort path)
            mbar_wait(bar_w2, 0, WAIT_LIMIT);
            if (i > 0) mbar_wait(bar_h1, (uint32_t)(i - 1) & 1u, WAIT_LIMIT);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer
            bool ok = mbar_wait(bar_w2, 0, WAIT_LIMIT);
            int i = 0, committed = 0, acc_commits = 0;
            for (int t = blockIdx.x; t < a.tiles && ok; t += gridDim.x, i++) {
                const uint32_t par = (uint32_t)i & 1u;
                ok = mbar_wait(bar_h1, par, WAIT_LIMIT) && !*abort_s;
                if (!ok) break;
                tc_fence_after();
                for (int kb = 0; kb < 4; kb++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16(tmem + D_MAIN, desc_sw128_k(base + OFF_X + kb * 16384 + kk * 32),
                                 desc_sw128_k(base + OFF_W2 + kb * 32768 + kk * 32), ID_L2, (kb | kk) ? 1u : 0u);
                mma_commit(bar_acc);
                acc_commits = i + 1;
                // h2 written by the epilogue, and the previous tile's head results read
                ok = mbar_wait(bar_h2, par, WAIT_LIMIT) && (i == 0 || mbar_wait(bar_hfree, par ^ 1u, WAIT_LIMIT)) &&
                     !*abort_s;
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 16; ks++)
                    mma_bf16(tmem + D_HEAD, desc_sw128_k(base + OFF_X + (ks >> 2) * 16384 + (ks & 3) * 32),
                             desc_plain_k(base + OFF_HB + ks * 512, 256), ID_HEAD, ks ? 1u : 0u);
                mma_commit(bar_head);
                mma_commit(bar_xfree);
                committed = i + 1;
            }
            if (!ok) {
                atomicExch(&g_ptail_error, 2);
                *abort_s = 1;
            }
            // the tensor cores are done with TMEM and shared memory before teardown
            // (MMAs complete in order: the latest commit of each barrier covers them)
            if (acc_commits > 0) mbar_wait(bar_acc, (uint32_t)(acc_commits - 1) & 1u, WAIT_LIMIT);
            if (committed > 0) mbar_wait(bar_xfree, (uint32_t)(committed - 1) & 1u, WAIT_LIMIT);
        }
    } else {
        // ---- epilogue
        const int q = warp & 3, half = (warp - 2) >> 2, te = threadIdx.x - 64;
        const int row = q * 32 + lane;
        b2_s[te] = __ldg(a.b2 + te);
        if (te < 16) bh_s[te] = te < NOUT ? __ldg(a.bh + te) : 0.f;
        {
            const int c = te;  // Wh as the head's B, thread per hidden column
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const __nv_bfloat16 v = j < NOUT ? a.wh[j * HID + c] : __float2bfloat16_rn(0.f);
                *reinterpret_cast<__nv_bfloat16 *>(sm + OFF_HB + (c >> 3) * 256 + j * 16 + (c & 7) * 2) = v;
            }
        }
        fence_proxy_async();
        const uint64_t step = a.step_dev ? (uint64_t)*a.step_dev : a.step;
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");  // b2_s, bh_s written
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        bool ok = true;
        int i = 0;
        for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, i++) {
            const uint32_t par = (uint32_t)i & 1u;
            const int grow = t * ROWS + row;
            // this row's legal mask, loaded now so its latency hides behind layer 2
            const uint32_t bits = (half == 0 && grow < a.n && a.legal) ? (uint32_t)a.legal[grow] : 0xfffu;
            // h2 = relu(acc + b2) as bf16 into the tile
            ok = mbar_wait(bar_acc, par, WAIT_LIMIT) && !*abort_s;
            if (ok) {
                tc_fence_after();
#pragma unroll 1
                for (int cc = 0; cc < 4; cc++) {
                    const int c0 = half * 128 + cc * 32;
                    uint32_t v[32];
                    D1X_TMEM_LD32(tmem + lanes + D_MAIN + (uint32_t)c0, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        float f[8];
#pragma unroll
                        for (int k = 0; k < 8; k++)
                            f[k] = fmaxf(__uint_as_float(v[8 * u + k]) + b2_s[c0 + 8 * u + k], 0.f);
                        *reinterpret_cast<uint4 *>(sm + x_off(row, c0 + 8 * u)) =
                            make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                    }
                }
            }
            fence_proxy_async();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_h2);
            if (!ok) break;
            // head outputs -> value, logits, the draw (column half 0: one thread per row)
            ok = mbar_wait(bar_head, par, WAIT_LIMIT) && !*abort_s;
            if (ok && half == 0) {
                tc_fence_after();
                uint32_t v[16];
                D1X_TMEM_LD16(tmem + lanes + D_HEAD, v);
                tmem_wait_ld();
                if (grow < a.n) {
                    float l[NOUT];
#pragma unroll
                    for (int j = 0; j < NOUT; j++) l[j] = __uint_as_float(v[j]) + bh_s[j];
                    a.value[grow] = l[NACT];
                    if (a.logits) {
#pragma unroll
                        for (int j = 0; j < NACT; j++) a.logits[(size_t)grow * NACT + j] = l[j];
                    }
                    if (a.action) {
                        int act;
                        float lp;
                        sample_masked(l, bits, (uint32_t)(a.first_env + grow), a.seed, step, false, act, lp);
                        a.action[grow] = act;
                        if (a.logp) a.logp[grow] = lp;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_hfree);
            if (!ok) break;
        }
        if (!ok) {
            atomicExch(&g_ptail_error, 3);
            *abort_s = 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_ALLOC) : "memory");
    }
}

typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static bool map_bf16(CUtensorMap *m, const void *ptr, int rows, int cols, int ld, int box_rows) {
    static EncodeTiled enc = nullptr;
    if (!enc) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult qr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) != cudaSuccess ||
            qr != cudaDriverEntryPointSuccess)
            return false;
        enc = reinterpret_cast<EncodeTiled>(p);
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace ptail
}  // namespace d1

extern "C" {

int d1_policy_tail_sample(const void *h1, int n, int ldh, const void *w2, const float *b2, const void *wh,
                          const float *bh, const uint16_t *legal, uint64_t seed, uint64_t step,
                          const int64_t *step_dev, int first_env, int64_t *action, float *logp, float *value,
                          float *logits, void *stream) {
    using namespace d1::ptail;
    if (!h1 || !w2 || !b2 || !wh || !bh || !value || n <= 0 || ldh < HID || (ldh & 7))
        return D1_ERR_BAD_ARGUMENT;
    if (((uintptr_t)h1 | (uintptr_t)w2) & 15) return D1_ERR_BAD_ARGUMENT;
    CUtensorMap mh, mw;
    if (!map_bf16(&mh, h1, n, HID, ldh, ROWS) || !map_bf16(&mw, w2, HID, HID, HID, HID)) return D1_ERR_BAD_ARGUMENT;
    static uint64_t ready = 0;
    int dev = 0, sms = 0;
    if (cudaError_t e = cudaGetDevice(&dev)) return (int)e;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
    if (dev >= 64 || !((ready >> dev) & 1)) {
        cudaError_t e = cudaFuncSetAttribute(policy_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return (int)e;
        if (dev < 64) ready |= 1ull << dev;
    }
    const int tiles = (n + ROWS - 1) / ROWS;
    Args a{(const __nv_bfloat16 *)wh, b2, bh, legal, seed, step, step_dev, first_env, n, tiles, action, logp, value,
           logits};
    cudaLaunchAttribute attr;
    const cudaLaunchConfig_t cfg =
        d1::pdl_config(dim3(tiles < sms ? tiles : sms), dim3(THREADS), SMEM, (cudaStream_t)stream, &attr);
    return (int)cudaLaunchKernelEx(&cfg, policy_tail_kernel, mh, mw, a);
}

int d1_policy_tail_error(void) {
    int h = 0, z = 0;
    if (cudaMemcpyFromSymbol(&h, d1::ptail::g_ptail_error, sizeof(int)) != cudaSuccess) return -1;
    if (h) cudaMemcpyToSymbol(d1::ptail::g_ptail_error, &z, sizeof(int));
    return h;
}

}  // extern "C"
