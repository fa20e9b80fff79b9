// Dense layers on the 5th-generation tensor cores (sm_100a tcgen05 + TMA).
//
//   C[M, N] = act(A[M, K] . B[N, K]^T + bias[N])      (bf16 operands, fp32 accumulate)
//
// Both operands are K-major (row-major with K contiguous), as the policy's
// activations and nn.Linear-style weights are. One CTA computes a 128 x 256
// tile; K advances in 64-element blocks through a 4-stage ring of shared-memory
// buffers filled by TMA (128-byte swizzle, zero fill past the tensor edges).
//
// Warp roles (320 threads): warp 0 lane 0 issues TMA loads; warp 1 owns the
// tensor-memory allocation and one lane issues tcgen05.mma (M=128, N=256, K=16
// per instruction, accumulators in 2 x 256 TMEM columns); warps 2-9 are the
// epilogue, warp w reading TMEM lanes 32*(w%4).. (= 32 tile rows) of one
// 128-column half with tcgen05.ld.
//
// Outputs (any subset): bf16 C (row-major), bf16 C^T (feature-major, for the
// weight-gradient GEMMs of the backward pass), and fp32 C (row-major, one slab
// per K split for deterministic split-K reduction).
//
// Every wait on an mbarrier is bounded: on expiry the kernel records an error
// code in d1_gemm_error and runs its teardown (TMEM is always freed).
#include <atomic>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/d1.h"
#include "d1_pdl.cuh"
#include "d1_sampler.cuh"


namespace d1 {
namespace tc {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int BIAS_BYTES = EPI_WARPS * (BN / 2) * 4;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + BIAS_BYTES;
// Fused policy head (N = 256 in one tile): head weights fp32 [13][256] and the
// per-row partial dot products of the two column halves [2][128][13].
constexpr int HEAD_OUT = 13, HEAD_W_BYTES = HEAD_OUT * BN * 4, HEAD_PART_BYTES = 2 * BM * HEAD_OUT * 4;
constexpr int SMEM_HEAD_BYTES = SMEM_BYTES + HEAD_W_BYTES + HEAD_PART_BYTES + 16;  // + abort flag
constexpr int SM_COUNT = 148;
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t WAIT_LIMIT = 1u << 22;

__device__ int g_error;

struct Params {
    int M, N, K;
    int k_tiles_per_split, k_tiles_total;
    const float *bias;   // may be null
    int relu;
    int a_mn;            // A stored [K, M] (M contiguous) instead of [M, K]
    const int64_t *a_rows;  // A row m = row a_rows[m] of a [rows, K] table (K-major A; null: plain)
    const int64_t *b_rows;  // B K-row k = row b_rows[k] of a [rows, N] table (MN-major B; null: plain)
    int b_mn;            // B stored [K, N] (N contiguous) instead of [N, K]
    // operand expanded from compact observation rows (pair kernel, XM != 0):
    // row r of the expanded matrix = the 1832 one-hot features of compact row
    // cidx[r] (or r), then the ones column at 1832, zeros after
    const uint8_t *cobs;
    const int64_t *cidx;
    const __nv_bfloat16 *mask;  // row-major [M, ldm]: zero where mask <= 0 (may be null)
    int ldm;
    __nv_bfloat16 *c;    // row-major [M, ldc] (may be null)
    int ldc;
    __nv_bfloat16 *ct;   // feature-major [N, ldct] (may be null)
    int ldct;
    float *cf;           // fp32 row-major [splits][M, ldcf] (may be null)
    int ldcf;
    // fused head + sampler (head != 0): logits/value = bf16(C) . Wh^T + bh, then
    // the masked draw of d1_sampler.cuh
    int head;
    const __nv_bfloat16 *head_w;  // [13, 256]
    const float *head_b;          // [13]
    const uint16_t *legal;        // [M] (null: all 12 legal)
    uint64_t seed, step;
    int first_env;
    int64_t *action;              // [M] (null: value only)
    float *logp, *value, *logits; // [M], [M], [M, 12] (each may be null)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bounded parity wait: true when the phase completed, false after WAIT_LIMIT polls.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t it = 0; it < WAIT_LIMIT; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
    }
    return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// tile::gather4: four rows r[0..3] of a tensor map whose box is one row of 64
// elements, landing as four consecutive 128-byte rows at dst (swizzled by the map).
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, const int *r) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(bar)
        : "memory");
}
__device__ __forceinline__ bool full_cols_m(int col0, int n) { return col0 + 32 <= n; }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major tile stored with the 128-byte
// swizzle (rows of 128 B, 8-row groups 1024 B apart): start address >> 4,
// stride byte offset 1024 >> 4, fixed version bits 46-48 = 0b001, swizzle mode 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(16u >> 4) << 16;      // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024u >> 4) << 32;    // stride byte offset
    d |= (uint64_t)1 << 46;               // version
    d |= (uint64_t)2 << 61;               // 128-byte swizzle
    return d;
}
// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
// A given MN-major (stored [K, M]): "transpose A" bit 15; B given MN-major
// (stored [K, N], N contiguous): "transpose B" bit 16.
constexpr uint32_t IDESC_AMN = 1u << 15, IDESC_BMN_BIT = 1u << 16;

__device__ __forceinline__ void mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t accumulate,
                                    uint32_t idesc = IDESC) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// MN-major operand with the 128-byte swizzle: each K row of a 64-element MN
// atom is one 128-byte line, 8 K rows form a 1024-byte swizzle atom (stride
// byte offset 1024), and the 64-element MN atoms are 8 KB apart (leading byte
// offset 8192: one TMA box of 64 K rows x 64 MN elements each).
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(8192u >> 4) << 16;    // leading byte offset: next 64 MN elements
    d |= (uint64_t)(1024u >> 4) << 32;    // stride byte offset: next 8 K rows
    d |= (uint64_t)1 << 46;               // version
    d |= (uint64_t)2 << 61;               // 128-byte swizzle
    return d;
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

#define D1_TMEM_LD32(taddr, v)                                                                                      \
    asm volatile(                                                                                                   \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                             \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),          \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),    \
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),  \
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])   \
        : "r"(taddr))

// Persistent: one CTA per SM walks tiles t = blockIdx.x, blockIdx.x + gridDim.x,
// ... (tile -> (m block, n block, K split)). The TMA ring runs continuously
// across tile boundaries and the accumulator is double-buffered in TMEM
// (2 x 256 columns), so the epilogue of one tile overlaps the MMAs of the next.
template <bool HEAD>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Params p,
                int tiles_m, int tiles_n, int tiles_total) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STAGES * STAGE_BYTES);
    // bars: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2]; then the TMEM slot
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STAGES + 4);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
    const uint32_t accf0 = smem_u32(bars + 2 * STAGES), acce0 = smem_u32(bars + 2 * STAGES + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(accf0 + 8 * b, 1);
            mbar_init(acce0 + 8 * b, EPI_WARPS);  // one arrival per epilogue warp
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer warp: k blocks of every tile of this CTA, one ring.
        // Lane 0 owns the barriers and the plain tile loads; with gathered rows
        // (a_rows / b_rows) every lane issues tile::gather4 loads of 4 rows.
        int it = 0, inflight_lo = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles_total && ok; t += gridDim.x) {
            const int mt = t % tiles_m, nt = (t / tiles_m) % tiles_n, split = t / (tiles_m * tiles_n);
            const int kt0 = split * p.k_tiles_per_split;
            const int kt1 = min(p.k_tiles_total, kt0 + p.k_tiles_per_split);
            // A rows of this tile for gathered A: lane l owns rows 4l .. 4l+3
            int ar[4] = {0, 0, 0, 0};
            if (p.a_rows) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int m = mt * BM + 4 * lane + i;
                    ar[i] = m < p.M ? (int)p.a_rows[m] : (int)p.a_rows[0];
                }
            }
            for (int kt = kt0; kt < kt1; kt++, it++) {
                const int s = it % STAGES;
                int good = 1;
                if (lane == 0 && it >= STAGES && !mbar_wait(empty0 + 8 * s, ((uint32_t)(it / STAGES) & 1u) ^ 1u))
                    good = 0;
                if (!__shfl_sync(0xffffffffu, good, 0)) {
                    ok = false;
                    break;
                }
                if (it >= STAGES) inflight_lo = it - STAGES + 1;
                const uint32_t a_dst = smem_u32(smem + s * STAGE_BYTES), b_dst = a_dst + A_BYTES;
                if (lane == 0) mbar_expect_tx(full0 + 8 * s, STAGE_BYTES);
                __syncwarp();
                if (p.a_rows) {
                    tma_gather4(a_dst + lane * 512, &map_a, full0 + 8 * s, kt * BK, ar);
                } else if (lane == 0) {
                    if (p.a_mn) {
#pragma unroll
                        for (int j = 0; j < BM / 64; j++)
                            tma_load_2d(a_dst + j * 8192, &map_a, full0 + 8 * s, mt * BM + 64 * j, kt * BK);
                    } else {
                        tma_load_2d(a_dst, &map_a, full0 + 8 * s, kt * BK, mt * BM);
                    }
                }
                if (p.b_rows) {
                    // MN-major B from gathered K rows: lanes 0-15 load N chunks 0 and 2,
                    // lanes 16-31 chunks 1 and 3; lane l % 16 owns K rows 4(l%16) .. +3
                    const int q = lane & 15, c0 = lane >> 4;
                    int br[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int k = kt * BK + 4 * q + i;
                        br[i] = k < p.K ? (int)p.b_rows[k] : (int)p.b_rows[0];
                    }
#pragma unroll
                    for (int cc = 0; cc < 2; cc++) {
                        const int j = c0 + 2 * cc;
                        tma_gather4(b_dst + j * 8192 + q * 512, &map_b, full0 + 8 * s, nt * BN + 64 * j, br);
                    }
                } else if (lane == 0) {
                    if (p.b_mn) {
#pragma unroll
                        for (int j = 0; j < BN / 64; j++)
                            tma_load_2d(b_dst + j * 8192, &map_b, full0 + 8 * s, nt * BN + 64 * j, kt * BK);
                    } else {
                        tma_load_2d(b_dst, &map_b, full0 + 8 * s, kt * BK, nt * BN);
                    }
                }
            }
        }
        if (!ok && lane == 0) {
            atomicExch(&g_error, 1);
            for (int i = inflight_lo; i < it; i++) mbar_wait(full0 + 8 * (i % STAGES), (uint32_t)(i / STAGES) & 1u);
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer
        int it = 0, local = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles_total && ok; t += gridDim.x, local++) {
            const int split = t / (tiles_m * tiles_n);
            const int kt0 = split * p.k_tiles_per_split;
            const int kt1 = min(p.k_tiles_total, kt0 + p.k_tiles_per_split);
            const int b = local & 1;
            const uint32_t acc = tmem + (uint32_t)(b * TMEM_COLS);
            if (local >= 2 && !mbar_wait(acce0 + 8 * b, ((uint32_t)(local >> 1) & 1u) ^ 1u)) {
                atomicExch(&g_error, 4);
                ok = false;
                break;
            }
            fence_after();
            for (int kt = kt0; kt < kt1; kt++, it++) {
                const int s = it % STAGES;
                if (!mbar_wait(full0 + 8 * s, (uint32_t)(it / STAGES) & 1u)) {
                    atomicExch(&g_error, 2);
                    ok = false;
                    break;
                }
                fence_after();
                const uint32_t a_base = smem_u32(smem + s * STAGE_BYTES), b_base = a_base + A_BYTES;
#pragma unroll
                for (int kk = 0; kk < BK / 16; kk++)
                    mma(acc, p.a_mn ? sw128_mn_desc(a_base + kk * 2048) : sw128_desc(a_base + kk * 32),
                        p.b_mn ? sw128_mn_desc(b_base + kk * 2048) : sw128_desc(b_base + kk * 32),
                        (kt > kt0 || kk > 0) ? 1u : 0u,
                        IDESC | (p.a_mn ? IDESC_AMN : 0u) | (p.b_mn ? IDESC_BMN_BIT : 0u));
                mma_commit(empty0 + 8 * s);
            }
            mma_commit(accf0 + 8 * b);
        }
    } else if (warp >= 2) {
        // ---- epilogue: warp w reads TMEM lanes 32*(w % 4) .. +31 (= tile rows)
        // and column half (w - 2) / 4 of the accumulator.
        const int q = warp & 3, half = (warp - 2) >> 2;
        float *bias_s = reinterpret_cast<float *>(smem + STAGES * STAGE_BYTES + 256) + (warp - 2) * (BN / 2);
        float *head_w = reinterpret_cast<float *>(smem + SMEM_BYTES - 1024);  // [13][256] (head mode)
        float *head_part = head_w + HEAD_OUT * BN;                             // [2][128][13]
        volatile int *head_abort = reinterpret_cast<volatile int *>(head_part + 2 * BM * HEAD_OUT);
        if constexpr (HEAD) {
            for (int i = threadIdx.x - 64; i < HEAD_OUT * BN; i += EPI_WARPS * 32)
                head_w[i] = __bfloat162float(p.head_w[i]);
            if (threadIdx.x == 64) *head_abort = 0;
            asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
        }
        int local = 0;
        for (int t = blockIdx.x; t < tiles_total; t += gridDim.x, local++) {
            const int mt = t % tiles_m, nt = (t / tiles_m) % tiles_n, split = t / (tiles_m * tiles_n);
            const int b = local & 1;
            const int row = mt * BM + q * 32 + lane;
            const int c0 = nt * BN + half * (BN / 2);
            // this warp's 128 bias values (zero past N or without bias)
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int col = c0 + lane * 4 + j;
                bias_s[lane * 4 + j] = (p.bias && col < p.N) ? __ldg(p.bias + col) : 0.f;
            }
            __syncwarp();
            const bool waited = mbar_wait(accf0 + 8 * b, (uint32_t)(local >> 1) & 1u);
            if (!waited) {
                atomicExch(&g_error, 3);
                if constexpr (!HEAD) break;
                *head_abort = 1;  // every epilogue warp leaves after this tile's barriers
            }
            fence_after();
            float hacc[HEAD ? HEAD_OUT : 1];
#pragma unroll
            for (int j = 0; j < (HEAD ? HEAD_OUT : 1); j++) hacc[j] = 0.f;
#pragma unroll 1
            for (int cc = 0; cc < BN / 64 && waited; cc++) {
                uint32_t v[32];
                const uint32_t taddr = tmem + (uint32_t)(b * TMEM_COLS) + ((uint32_t)(q * 32) << 16) +
                                       (uint32_t)(half * (BN / 2) + cc * 32);
                __syncwarp();  // tcgen05.ld is .sync.aligned: reconverge after the row/column guards
                D1_TMEM_LD32(taddr, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int col0 = c0 + cc * 32;
                if (row >= p.M || col0 >= p.N) continue;
                float f[32];
                const float4 *bs = reinterpret_cast<const float4 *>(bias_s + cc * 32);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 bb = bs[j / 4];
                    f[j] = __uint_as_float(v[j]) + bb.x;
                    f[j + 1] = __uint_as_float(v[j + 1]) + bb.y;
                    f[j + 2] = __uint_as_float(v[j + 2]) + bb.z;
                    f[j + 3] = __uint_as_float(v[j + 3]) + bb.w;
                }
                if (p.relu) {
#pragma unroll
                    for (int j = 0; j < 32; j++) f[j] = fmaxf(f[j], 0.f);
                }
                if constexpr (HEAD) {
                    // the head sees the activation as stored (bf16), like the unfused path
                    const float *wcol = head_w + col0;
#pragma unroll 4
                    for (int i = 0; i < 32; i++) {
                        const float x = __bfloat162float(__float2bfloat16_rn(f[i]));
#pragma unroll
                        for (int j = 0; j < HEAD_OUT; j++) hacc[j] = fmaf(x, wcol[j * BN + i], hacc[j]);
                    }
                }
                if (p.mask) {
                    const __nv_bfloat16 *mk = p.mask + (size_t)row * p.ldm + col0;
                    if (full_cols_m(col0, p.N)) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            const uint4 raw = *reinterpret_cast<const uint4 *>(mk + j);
                            const __nv_bfloat16 *h = reinterpret_cast<const __nv_bfloat16 *>(&raw);
#pragma unroll
                            for (int i = 0; i < 8; i++)
                                if (!(__bfloat162float(h[i]) > 0.f)) f[j + i] = 0.f;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j >= p.N || !(__bfloat162float(mk[j]) > 0.f)) f[j] = 0.f;
                    }
                }
                const bool full_cols = col0 + 32 <= p.N;
                if (p.cf) {
                    float *dst = p.cf + (size_t)split * p.M * p.ldcf + (size_t)row * p.ldcf + col0;
                    if (full_cols) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j < p.N) dst[j] = f[j];
                    }
                }
                if (p.c) {
                    __nv_bfloat16 *dst = p.c + (size_t)row * p.ldc + col0;
                    if (full_cols) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint4 w;
                            __nv_bfloat162 h0 = __floats2bfloat162_rn(f[j], f[j + 1]);
                            __nv_bfloat162 h1 = __floats2bfloat162_rn(f[j + 2], f[j + 3]);
                            __nv_bfloat162 h2 = __floats2bfloat162_rn(f[j + 4], f[j + 5]);
                            __nv_bfloat162 h3 = __floats2bfloat162_rn(f[j + 6], f[j + 7]);
                            w.x = *reinterpret_cast<uint32_t *>(&h0);
                            w.y = *reinterpret_cast<uint32_t *>(&h1);
                            w.z = *reinterpret_cast<uint32_t *>(&h2);
                            w.w = *reinterpret_cast<uint32_t *>(&h3);
                            *reinterpret_cast<uint4 *>(dst + j) = w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j < p.N) dst[j] = __float2bfloat16_rn(f[j]);
                    }
                }
                if (p.ct) {
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (col0 + j < p.N) p.ct[(size_t)(col0 + j) * p.ldct + row] = __float2bfloat16_rn(f[j]);
                }
            }
            // Release this accumulator buffer to the MMA issuer.
            fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(acce0 + 8 * b) : "memory");
            if constexpr (HEAD) {
                // combine the two column halves, then one thread per row draws
                const int r = q * 32 + lane;
#pragma unroll
                for (int j = 0; j < HEAD_OUT; j++) head_part[(half * BM + r) * HEAD_OUT + j] = hacc[j];
                asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
                const bool abort = *head_abort != 0;
                const int grow = mt * BM + r;
                if (half == 0 && !abort && grow < p.M) {
                    float l[HEAD_OUT];
#pragma unroll
                    for (int j = 0; j < HEAD_OUT; j++)
                        l[j] = head_part[r * HEAD_OUT + j] + head_part[(BM + r) * HEAD_OUT + j] + __ldg(p.head_b + j);
                    if (p.value) p.value[grow] = l[12];
                    if (p.logits) {
#pragma unroll
                        for (int j = 0; j < 12; j++) p.logits[(size_t)grow * 12 + j] = l[j];
                    }
                    if (p.action) {
                        int a;
                        float lp;
                        sample_masked(l, p.legal ? (uint32_t)p.legal[grow] : 0xfffu, (uint32_t)(p.first_env + grow),
                                      p.seed, p.step, false, a, lp);
                        p.action[grow] = a;
                        if (p.logp) p.logp[grow] = lp;
                    }
                }
                asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
                if (abort) break;
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------- 2-SM pair kernel
// A cluster of two CTAs computes one 256 x 256 tile with tcgen05.mma.cta_group::2
// (M = 256): CTA rank r holds A rows m0 + 128r .. +127 and B rows (N)
// n0 + 128r .. +127 of every K block in its own shared memory, so each SM
// streams 32 KB per K block instead of 48 KB (A 16 KB + all of B's 32 KB) --
// the B re-reads that bound the one-CTA kernel. Both CTAs' TMA loads complete
// on the leader's (rank 0) full barrier; the leader's one thread issues the
// MMAs and commits to the empty and accumulator barriers of both CTAs; each CTA
// drains its own 128 TMEM lanes (its 128 rows of the tile) and arrives on the
// leader's accumulator-empty barrier. Six 32 KB stages; accumulators
// double-buffered (2 x 256 columns). Epilogue: bias, ReLU, ReLU-mask, bf16 and
// split-K fp32 slabs (no transposed output, no fused head).
constexpr int P_STAGES = 6, P_B_BYTES = 128 * BK * 2, P_STAGE_BYTES = A_BYTES + P_B_BYTES;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/ + BIAS_BYTES;
constexpr int P2_SMEM_BYTES = 4 * (2 * A_BYTES + P_B_BYTES) + 1024 + 256 + BIAS_BYTES;
// compact observation rows (d1_spec_step_ex): a channel byte per window cell,
// zeros to byte 255, then 32 bf16 scalars
constexpr int X_ROW = 320, X_CELLS = 225, X_SCALARS = 256, X_K = 1832, X_EXPANDERS = 4;
// compact-operand kernels: channel codes (and sample indices) are copied
// X_DEPTH K blocks ahead into shared-memory rings; scalar units are staged in
// shared memory too (XM = 1: 64 bytes per A row of a tile; XM = 2: 64 bytes per
// sample of X_DEPTH K blocks)
constexpr int X_DEPTH = 4, X_SCAL_BYTES = 256 * 64, X_SMEM_BYTES = X_SCAL_BYTES + 8192 /*code and index rings*/;
constexpr uint32_t P_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t mapa(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory that completes on the pair leader's barrier.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, uint32_t bar_cluster, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
        "%3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void commit_pair(uint32_t bar_cluster) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
                 : "memory");
}
// Arrival on a barrier of either CTA of the pair (default release semantics:
// measured, a cluster-scope release here serialised every pipeline stage and
// doubled the kernel's time).
__device__ __forceinline__ void arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// bar.red.or over the expander warps: true on every thread if any passed true.
__device__ __forceinline__ bool expanders_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 2, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(32 * X_EXPANDERS)
        : "memory");
    return r != 0;
}
// One-hot unit of channel code c (0..7): bf16 1.0 at feature c of the 8.
__device__ __forceinline__ uint4 onehot_unit(uint32_t c) {
    const uint32_t v = 0x3f80u << ((c & 1u) << 4), w = c >> 1;
    return make_uint4(w == 0 ? v : 0u, w == 1 ? v : 0u, w == 2 ? v : 0u, w == 3 ? v : 0u);
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// The 32 bf16 scalars (64 bytes at byte 256) of compact row `row` copied to
// shared memory at `dst`.
__device__ __forceinline__ void x_stage_scalars(uint8_t *dst, const uint8_t *__restrict__ cobs, int64_t row) {
#pragma unroll
    for (int q = 0; q < 4; q++) cp_async16(smem_u32(dst + 16 * q), cobs + row * X_ROW + X_SCALARS + 16 * q);
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
// Channel codes of cells c .. c + 7 of compact row `row` (c a multiple of 8;
// from cell 224 on, the last cell's code and the zero bytes after it) copied to
// shared memory at `dst`. The copies are asynchronous: a bar.sync waits for a
// thread's outstanding loads into registers but not for cp.async groups, so the
// ring stays in flight across the per-stage barriers.
__device__ __forceinline__ void x_stage_codes(uint8_t *dst, const uint8_t *__restrict__ cobs, int64_t row, int c) {
    cp_async8(smem_u32(dst), cobs + row * X_ROW + min(c, X_CELLS - 1));
}
// The eight 16-byte units of features 8c .. 8c + 63 into one 128-byte row of a
// 128-byte-swizzled tile (unit u at u ^ sw): the one-hot channels of cells
// c .. c + 7, or for the last block cell 224, the four scalar units `scal`, the
// ones unit (feature 1832) and zeros; all zeros where `live` is false.
__device__ __forceinline__ void x_write_row(uint8_t *dst, int sw, int c, uint2 codes, const uint4 *scal,
                                            bool live) {
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    if (live && c + 8 <= X_CELLS) {
#pragma unroll
        for (int u = 0; u < 8; u++)
            *reinterpret_cast<uint4 *>(dst + ((u ^ sw) << 4)) =
                onehot_unit(((u < 4 ? codes.x : codes.y) >> (8 * (u & 3))) & 7u);
    } else if (live && c == X_CELLS - 1) {
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const uint4 v = u == 0   ? onehot_unit(codes.x & 7u)
                            : u < 5  ? scal[u - 1]
                            : u == 5 ? make_uint4(0x3f80u, 0u, 0u, 0u)
                                     : zero;
            *reinterpret_cast<uint4 *>(dst + ((u ^ sw) << 4)) = v;
        }
    } else {
#pragma unroll
        for (int u = 0; u < 8; u++) *reinterpret_cast<uint4 *>(dst + ((u ^ sw) << 4)) = zero;
    }
}

// SUB = 2: each CTA holds two 128-row blocks of A per K block (a 512-row pair
// tile) and issues two MMAs against the same B half, so B is streamed half as
// often; the two accumulators fill the 512 TMEM columns, so the accumulator is
// single-buffered (the next tile's loads still run during the epilogue).
// XM = 1: A (K-major, K = 1832) is expanded from compact observation rows and
// XM = 2: B (MN-major, [K = samples, N = features + ones column]) is, by four
// extra warps that write the operand tile into the 128-byte-swizzled layout the
// TMA would have produced (16-byte unit u of a 128-byte row r at u ^ (r % 8)),
// fence it for the async proxy and arrive on the leader's full barrier, which
// then expects the TMA bytes of the other operand plus the two CTAs' expander
// arrivals. Reading 8 bytes of channel codes instead of 128 bytes of one-hot
// features per 64-deep K block cuts the operand's L2 and HBM traffic 16-fold.
template <int SUB, int XM>
__global__ void __launch_bounds__(THREADS + (XM ? 32 * X_EXPANDERS : 0), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Params p,
                     int tiles_m, int tiles_n, int tiles_total) {
    constexpr int STG = SUB == 1 ? P_STAGES : 4, STG_BYTES = SUB * A_BYTES + P_B_BYTES, NBUF = SUB == 1 ? 2 : 1;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + STG * STG_BYTES);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * STG + 4);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STG);
    const uint32_t accf0 = smem_u32(bars + 2 * STG), acce0 = smem_u32(bars + 2 * STG + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;

    if (warp == 0 && lane == 0) {
        for (int s = 0; s < STG; s++) {
            mbar_init(full0 + 8 * s, XM ? 3 : 1);  // + one arrival per CTA's expanders
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(accf0 + 8 * b, 1);
            mbar_init(acce0 + 8 * b, 2 * EPI_WARPS);  // the epilogue warps of both CTAs
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers exist before any cross-CTA signal
    fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // the previous kernel's outputs (operands, the weights) are complete from here on

    if (warp == 0 && lane == 0) {
        // ---- producer (both CTAs): this CTA's A rows and B half, signalling the leader
        int it = 0, inflight_lo = 0;
        bool ok = true;
        for (int t = cluster; t < tiles_total && ok; t += clusters) {
            const int mt = t % tiles_m, nt = (t / tiles_m) % tiles_n, split = t / (tiles_m * tiles_n);
            const int kt0 = split * p.k_tiles_per_split;
            const int kt1 = min(p.k_tiles_total, kt0 + p.k_tiles_per_split);
            const int m0 = mt * 256 * SUB + 128 * (int)rank, n0 = nt * BN + 128 * (int)rank;
            for (int kt = kt0; kt < kt1; kt++, it++) {
                const int s = it % STG;
                if (it >= STG && !mbar_wait(empty0 + 8 * s, ((uint32_t)(it / STG) & 1u) ^ 1u)) {
                    ok = false;
                    break;
                }
                if (it >= STG) inflight_lo = it - STG + 1;
                const uint32_t a_dst = smem_u32(smem + s * STG_BYTES), b_dst = a_dst + SUB * A_BYTES;
                const uint32_t leader_full = mapa(full0 + 8 * s, 0);
                if (rank == 0)
                    mbar_expect_tx(full0 + 8 * s, XM == 1 ? 2 * P_B_BYTES : XM == 2 ? 2 * SUB * A_BYTES : 2 * STG_BYTES);
#pragma unroll
                for (int sb = 0; sb < SUB; sb++) {
                    if (XM == 1) break;
                    if (p.a_mn) {
#pragma unroll
                        for (int j = 0; j < 2; j++)
                            tma_load_2d_pair(a_dst + sb * A_BYTES + j * 8192, &map_a, leader_full, m0 + 256 * sb + 64 * j,
                                             kt * BK);
                    } else {
                        tma_load_2d_pair(a_dst + sb * A_BYTES, &map_a, leader_full, kt * BK, m0 + 256 * sb);
                    }
                }
                if (XM == 2) {
                } else if (p.b_mn) {
#pragma unroll
                    for (int j = 0; j < 2; j++) tma_load_2d_pair(b_dst + j * 8192, &map_b, leader_full, n0 + 64 * j, kt * BK);
                } else {
                    tma_load_2d_pair(b_dst, &map_b, leader_full, kt * BK, n0);
                }
            }
        }
        if (!ok) {
            atomicExch(&g_error, 5);
            if (rank == 0)
                for (int i = inflight_lo; i < it; i++) mbar_wait(full0 + 8 * (i % STG), (uint32_t)(i / STG) & 1u);
        } else {
            // the leader's last commits to this CTA's empty barriers land before it exits
            for (int i = it > STG ? it - STG : 0; i < it; i++)
                mbar_wait(empty0 + 8 * (i % STG), (uint32_t)(i / STG) & 1u);
        }
    } else if (warp == 1 && lane == 0 && rank == 0) {
        // ---- MMA issuer (leader only)
        int it = 0, local = 0;
        bool ok = true;
        const uint32_t idesc = P_IDESC | (p.a_mn ? (1u << 15) : 0u) | (p.b_mn ? (1u << 16) : 0u);
        for (int t = cluster; t < tiles_total && ok; t += clusters, local++) {
            const int split = t / (tiles_m * tiles_n);
            const int kt0 = split * p.k_tiles_per_split;
            const int kt1 = min(p.k_tiles_total, kt0 + p.k_tiles_per_split);
            const int b = local % NBUF;
            const uint32_t acc = tmem + (uint32_t)(b * SUB * TMEM_COLS);
            if (local >= NBUF && !mbar_wait(acce0 + 8 * b, ((uint32_t)(local / NBUF) & 1u) ^ 1u)) {
                atomicExch(&g_error, 6);
                ok = false;
                break;
            }
            fence_after();
            for (int kt = kt0; kt < kt1; kt++, it++) {
                const int s = it % STG;
                if (!mbar_wait(full0 + 8 * s, (uint32_t)(it / STG) & 1u)) {
                    atomicExch(&g_error, 7);
                    ok = false;
                    break;
                }
                fence_after();
                const uint32_t a_base = smem_u32(smem + s * STG_BYTES), b_base = a_base + SUB * A_BYTES;
#pragma unroll
                for (int sb = 0; sb < SUB; sb++)
#pragma unroll
                    for (int kk = 0; kk < BK / 16; kk++)
                        mma_pair(acc + (uint32_t)(sb * TMEM_COLS),
                                 p.a_mn ? sw128_mn_desc(a_base + sb * A_BYTES + kk * 2048)
                                        : sw128_desc(a_base + sb * A_BYTES + kk * 32),
                                 p.b_mn ? sw128_mn_desc(b_base + kk * 2048) : sw128_desc(b_base + kk * 32), idesc,
                                 (kt > kt0 || kk > 0) ? 1u : 0u);
                commit_pair(empty0 + 8 * s);
                commit_pair(mapa(empty0 + 8 * s, 1));
            }
            if (!ok) break;
            commit_pair(accf0 + 8 * b);
            commit_pair(mapa(accf0 + 8 * b, 1));
        }
    } else if (XM && warp >= 2 + EPI_WARPS) {
        // ---- expanders (both CTAs): the expanded operand's tile of every stage.
        // Channel codes, sample indices and scalar units arrive by cp.async
        // X_DEPTH K blocks ahead of use, so no global load latency sits between a
        // stage's empty barrier and its arrival. Every expander thread waits for
        // the empty stage itself; one bar.red after the writes both orders them
        // before the arrival and agrees on a timed-out wait.
        const int tx = threadIdx.x - 32 * (2 + EPI_WARPS);
        uint8_t *xs = smem + STG * STG_BYTES + 256 + BIAS_BYTES;
        int it = 0;
        bool ok = true;
        for (int t = cluster; t < tiles_total && ok; t += clusters) {
            const int mt = t % tiles_m, nt = (t / tiles_m) % tiles_n, split = t / (tiles_m * tiles_n);
            const int kt0 = split * p.k_tiles_per_split;
            const int kt1 = min(p.k_tiles_total, kt0 + p.k_tiles_per_split);
            const int m0 = mt * 256 * SUB + 128 * (int)rank, n0 = nt * BN + 128 * (int)rank;
            if (XM == 1) {
                // A rows m0 + 256 sb + tx; K block kt = features 64 kt .. = cells 8 kt ..
                // (rows past M read row M - 1 and are written as zeros). Copy groups:
                // the scalars, then one per K block.
                uint8_t *xc = xs + X_SCAL_BYTES;
                int64_t row[SUB];
#pragma unroll
                for (int sb = 0; sb < SUB; sb++) {
                    const int grow = min(m0 + 256 * sb + tx, p.M - 1);
                    row[sb] = p.cidx ? __ldg(p.cidx + grow) : (int64_t)grow;
                    x_stage_scalars(xs + (sb * 128 + tx) * 64, p.cobs, row[sb]);
                }
                cp_async_commit();
                for (int d = 0; d < X_DEPTH; d++) {
                    if (kt0 + d < kt1)
#pragma unroll
                        for (int sb = 0; sb < SUB; sb++)
                            x_stage_codes(xc + ((d * SUB + sb) * 128 + tx) * 8, p.cobs, row[sb], 8 * (kt0 + d));
                    cp_async_commit();
                }
                for (int kt = kt0; kt < kt1; kt++, it++) {
                    const int s = it % STG, d = (kt - kt0) % X_DEPTH;
                    const bool got = it < STG || mbar_wait(empty0 + 8 * s, ((uint32_t)(it / STG) & 1u) ^ 1u);
                    cp_async_wait<X_DEPTH - 1>();
                    uint8_t *stage = smem + s * STG_BYTES;
                    if (got)
#pragma unroll
                        for (int sb = 0; sb < SUB; sb++)
                            x_write_row(stage + sb * A_BYTES + tx * 128, tx & 7, 8 * kt,
                                        *reinterpret_cast<const uint2 *>(xc + ((d * SUB + sb) * 128 + tx) * 8),
                                        reinterpret_cast<const uint4 *>(xs + (sb * 128 + tx) * 64),
                                        m0 + 256 * sb + tx < p.M);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    if (expanders_any(!got)) {
                        ok = false;
                        break;
                    }
                    if (tx == 0) arrive_cluster(mapa(full0 + 8 * s, 0));
                    if (kt + X_DEPTH < kt1)
#pragma unroll
                        for (int sb = 0; sb < SUB; sb++)
                            x_stage_codes(xc + ((d * SUB + sb) * 128 + tx) * 8, p.cobs, row[sb], 8 * (kt + X_DEPTH));
                    cp_async_commit();
                }
            } else {
                // B K rows (samples) 64 kt + k, N features n0 + 64 j .. + 63 = cells c0 .. c0 + 7
                // (samples past K read sample K - 1 and are written as zeros). Sample
                // indices are copied 2 X_DEPTH K blocks ahead, codes and scalars
                // X_DEPTH ahead; one copy group per K block.
                const int k = tx & 63, j = tx >> 6;
                const int c0 = (n0 + 64 * j) / 8;
                const bool scal = c0 == X_CELLS - 1;
                const int dst0 = SUB * A_BYTES + j * 8192 + (k >> 3) * 1024 + (k & 7) * 128;
                uint8_t *xc = xs + X_SCAL_BYTES, *xi = xc + 4096;
                auto stage_index = [&](int kt, int d) {
                    const int g = min(kt * BK + k, p.K - 1);
                    uint8_t *dst = xi + (d * 128 + tx) * 8;
                    if (p.cidx)
                        cp_async8(smem_u32(dst), p.cidx + g);
                    else
                        *reinterpret_cast<int64_t *>(dst) = g;
                };
                auto stage_sample = [&](int64_t r, int d) {
                    x_stage_codes(xc + (d * 128 + tx) * 8, p.cobs, r, c0);
                    if (scal) x_stage_scalars(xs + (d * 64 + k) * 64, p.cobs, r);
                };
                for (int d = 0; d < X_DEPTH; d++) {
                    if (kt0 + d < kt1) {
                        const int g = min((kt0 + d) * BK + k, p.K - 1);
                        stage_sample(p.cidx ? __ldg(p.cidx + g) : (int64_t)g, d);
                        if (kt0 + X_DEPTH + d < kt1) stage_index(kt0 + X_DEPTH + d, d);
                    }
                    cp_async_commit();
                }
                for (int kt = kt0; kt < kt1; kt++, it++) {
                    const int s = it % STG, d = (kt - kt0) % X_DEPTH;
                    const bool got = it < STG || mbar_wait(empty0 + 8 * s, ((uint32_t)(it / STG) & 1u) ^ 1u);
                    cp_async_wait<X_DEPTH - 1>();
                    if (got)
                        x_write_row(smem + s * STG_BYTES + dst0, k & 7, c0,
                                    *reinterpret_cast<const uint2 *>(xc + (d * 128 + tx) * 8),
                                    reinterpret_cast<const uint4 *>(xs + (d * 64 + k) * 64), kt * BK + k < p.K);
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    if (expanders_any(!got)) {
                        ok = false;
                        break;
                    }
                    if (tx == 0) arrive_cluster(mapa(full0 + 8 * s, 0));
                    if (kt + X_DEPTH < kt1) {
                        stage_sample(*reinterpret_cast<const int64_t *>(xi + (d * 128 + tx) * 8), d);
                        if (kt + 2 * X_DEPTH < kt1) stage_index(kt + 2 * X_DEPTH, d);
                    }
                    cp_async_commit();
                }
            }
        }
        cp_async_wait<0>();
        if (!ok) atomicExch(&g_error, 9);
    } else if (warp >= 2) {
        // ---- epilogue (both CTAs): this CTA's 128 rows of the tile
        const int q = warp & 3, half = (warp - 2) >> 2;
        float *bias_s = reinterpret_cast<float *>(smem + STG * STG_BYTES + 256) + (warp - 2) * (BN / 2);
        int local = 0;
        for (int t = cluster; t < tiles_total; t += clusters, local++) {
            const int mt = t % tiles_m, nt = (t / tiles_m) % tiles_n, split = t / (tiles_m * tiles_n);
            const int b = local % NBUF;
            const int c0 = nt * BN + half * (BN / 2);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int col = c0 + lane * 4 + j;
                bias_s[lane * 4 + j] = (p.bias && col < p.N) ? __ldg(p.bias + col) : 0.f;
            }
            __syncwarp();
            if (!mbar_wait(accf0 + 8 * b, (uint32_t)(local / NBUF) & 1u)) {
                atomicExch(&g_error, 8);
                break;
            }
            fence_after();
#pragma unroll 1
            for (int ci = 0; ci < SUB * (BN / 64); ci++) {
                const int sb = ci / (BN / 64), cc = ci % (BN / 64);
                const int row = mt * 256 * SUB + 256 * sb + 128 * (int)rank + q * 32 + lane;
                uint32_t v[32];
                const uint32_t taddr = tmem + (uint32_t)((b * SUB + sb) * TMEM_COLS) + ((uint32_t)(q * 32) << 16) +
                                       (uint32_t)(half * (BN / 2) + cc * 32);
                __syncwarp();
                D1_TMEM_LD32(taddr, v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int col0 = c0 + cc * 32;
                if (row >= p.M || col0 >= p.N) continue;
                float f[32];
                const float4 *bs = reinterpret_cast<const float4 *>(bias_s + cc * 32);
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 bb = bs[j / 4];
                    f[j] = __uint_as_float(v[j]) + bb.x;
                    f[j + 1] = __uint_as_float(v[j + 1]) + bb.y;
                    f[j + 2] = __uint_as_float(v[j + 2]) + bb.z;
                    f[j + 3] = __uint_as_float(v[j + 3]) + bb.w;
                }
                if (p.relu) {
#pragma unroll
                    for (int j = 0; j < 32; j++) f[j] = fmaxf(f[j], 0.f);
                }
                const bool full_cols = col0 + 32 <= p.N;
                if (p.mask) {
                    const __nv_bfloat16 *mk = p.mask + (size_t)row * p.ldm + col0;
                    if (full_cols) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            const uint4 raw = *reinterpret_cast<const uint4 *>(mk + j);
                            const __nv_bfloat16 *h = reinterpret_cast<const __nv_bfloat16 *>(&raw);
#pragma unroll
                            for (int i = 0; i < 8; i++)
                                if (!(__bfloat162float(h[i]) > 0.f)) f[j + i] = 0.f;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j >= p.N || !(__bfloat162float(mk[j]) > 0.f)) f[j] = 0.f;
                    }
                }
                if (p.cf) {
                    float *dst = p.cf + (size_t)split * p.M * p.ldcf + (size_t)row * p.ldcf + col0;
                    if (full_cols) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(f[j], f[j + 1], f[j + 2], f[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j < p.N) dst[j] = f[j];
                    }
                }
                if (p.c) {
                    __nv_bfloat16 *dst = p.c + (size_t)row * p.ldc + col0;
                    if (full_cols) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint4 w;
                            __nv_bfloat162 h0 = __floats2bfloat162_rn(f[j], f[j + 1]);
                            __nv_bfloat162 h1 = __floats2bfloat162_rn(f[j + 2], f[j + 3]);
                            __nv_bfloat162 h2 = __floats2bfloat162_rn(f[j + 4], f[j + 5]);
                            __nv_bfloat162 h3 = __floats2bfloat162_rn(f[j + 6], f[j + 7]);
                            w.x = *reinterpret_cast<uint32_t *>(&h0);
                            w.y = *reinterpret_cast<uint32_t *>(&h1);
                            w.z = *reinterpret_cast<uint32_t *>(&h2);
                            w.w = *reinterpret_cast<uint32_t *>(&h3);
                            *reinterpret_cast<uint4 *>(dst + j) = w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col0 + j < p.N) dst[j] = __float2bfloat16_rn(f[j]);
                    }
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0) arrive_cluster(mapa(acce0 + 8 * b, 0));
        }
    }
    fence_before();
    __syncthreads();
    cluster_sync();  // no cross-CTA signal is outstanding past this point
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TMEM_COLS)
                     : "memory");
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    }
    return fn;
}

// 2-D bf16 tensor [rows, cols] with row pitch `ld` elements; box BK x box_rows.
static bool make_map(CUtensorMap *m, const void *base, int rows, int cols, int ld, int box_rows) {
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tc
}  // namespace d1

using namespace d1::tc;

// Dynamic shared memory above 48 KB, opted into once per device (the head
// variant's larger figure covers both).
static int gemm_attr() {
    static uint64_t ready = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev < 64 && ((ready >> dev) & 1)) return 0;
    e = cudaFuncSetAttribute(gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_HEAD_BYTES);
    if (e != cudaSuccess) return (int)e;
    if (dev < 64) ready |= 1ull << dev;
    return 0;
}

// The pair kernel wins where each tile's K range is long (B traffic per SM
// dominates): measured 1.2-1.3x on 512+-deep K ranges with N > 128, and no gain
// on 256-deep ones.
static bool pair_pays(int N, int K, int splits, bool ct, bool gathered) {
    if (ct || gathered || N <= 128 || K <= 0 || splits < 1) return false;
    const int kt = (K + BK - 1) / BK;
    if (splits > kt) splits = kt;
    const int per = (kt + splits - 1) / splits;
    return per >= 8;
}

extern "C" {

static int pair_launch(const void *a, int lda, const void *b, int ldb, int M, int N, int K, const float *bias, int relu,
                       const void *mask, int ldm, void *c, int ldc, float *cf, int ldcf, int splits, int a_mn,
                       int b_mn, void *stream, int xm = 0, const uint8_t *cobs = nullptr,
                       const int64_t *cidx = nullptr);

static int gemm_launch(const void *a, int lda, const void *b, int ldb, int M, int N, int K, const float *bias,
                       int relu, const void *mask, int ldm, void *c, int ldc, void *ct, int ldct, float *cf, int ldcf,
                       int splits, int a_mn, int b_mn, void *stream, const int64_t *a_rows = nullptr,
                       int a_table_rows = 0, const int64_t *b_rows = nullptr, int b_table_rows = 0,
                       bool allow_pair = true) {
    if (allow_pair && splits >= 1 && pair_pays(N, K, splits, ct != nullptr, a_rows || b_rows))
        return pair_launch(a, lda, b, ldb, M, N, K, bias, relu, mask, ldm, c, ldc, cf, ldcf, splits, a_mn, b_mn, stream);
    if ((a_rows && (a_mn || a_table_rows <= 0)) || (b_rows && (!b_mn || b_table_rows <= 0)))
        return D1_ERR_BAD_ARGUMENT;
    if (M <= 0 || N <= 0 || K <= 0 || !a || !b || (!c && !ct && !cf) || splits < 1) return D1_ERR_BAD_ARGUMENT;
    // TMA rules: 16-byte aligned bases and row pitches.
    if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15) || (lda * 2) % 16 ||
        (ldb * 2) % 16 || lda < (a_mn ? M : K) || ldb < (b_mn ? N : K))
        return D1_ERR_BAD_ARGUMENT;
    if (c && ((reinterpret_cast<uintptr_t>(c) & 15) || ldc % 8 || ldc < N)) return D1_ERR_BAD_ARGUMENT;
    if (cf && ((reinterpret_cast<uintptr_t>(cf) & 15) || ldcf % 4 || ldcf < N)) return D1_ERR_BAD_ARGUMENT;
    if (ct && ldct < M) return D1_ERR_BAD_ARGUMENT;
    if (mask && ((reinterpret_cast<uintptr_t>(mask) & 15) || ldm % 8 || ldm < N)) return D1_ERR_BAD_ARGUMENT;
    if (splits > 1 && (c || ct)) return D1_ERR_BAD_ARGUMENT;  // split-K writes fp32 partial slabs only
    const int kt = (K + BK - 1) / BK;
    if (splits > kt) splits = kt;
    const int per = (kt + splits - 1) / splits;
    splits = (kt + per - 1) / per;  // every split gets at least one K block
    CUtensorMap ma, mb;
    // A [M, K]: boxes of BM rows x 64 K; A [K, M]: 64 K rows x 64 M; gathered A
    // rows: one-row boxes of the [a_table_rows, K] table (tile::gather4)
    if (!(a_rows  ? make_map(&ma, a, a_table_rows, K, lda, 1)
          : a_mn ? make_map(&ma, a, K, M, lda, 64)
                 : make_map(&ma, a, M, K, lda, BM)))
        return D1_ERR_BAD_ARGUMENT;
    // B [N, K]: boxes of BN rows x 64 K; B [K, N]: boxes of 64 K rows x 64 N
    if (!(b_rows ? make_map(&mb, b, b_table_rows, N, ldb, 1)
          : b_mn ? make_map(&mb, b, K, N, ldb, 64)
                 : make_map(&mb, b, N, K, ldb, BN)))
        return D1_ERR_BAD_ARGUMENT;
    if (int e = gemm_attr()) return e;
    Params p{M, N, K, per, kt, bias, relu, a_mn, a_rows, b_rows, b_mn, nullptr, nullptr, (const __nv_bfloat16 *)mask,
             ldm, (__nv_bfloat16 *)c, ldc, (__nv_bfloat16 *)ct, ldct, cf, ldcf};
    const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n * splits;
    static int sms = 0;
    if (!sms) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = SM_COUNT;
    }
    const int grid = tiles < sms ? tiles : sms;
    gemm_kernel<false><<<grid, THREADS, SMEM_BYTES, (cudaStream_t)stream>>>(ma, mb, p, tiles_m, tiles_n, tiles);
    return (int)cudaGetLastError();
}

int d1_gemm(const void *a, int lda, const void *b, int ldb, int M, int N, int K, const float *bias, int relu,
            const void *mask, int ldm, void *c, int ldc, void *ct, int ldct, float *cf, int ldcf, int splits,
            void *stream) {
    return gemm_launch(a, lda, b, ldb, M, N, K, bias, relu, mask, ldm, c, ldc, ct, ldct, cf, ldcf, splits, 0, 0,
                       stream);
}

int d1_gemm_ex(const void *a, int lda, int a_mn, const void *b, int ldb, int b_mn, int M, int N, int K,
               const float *bias, int relu, const void *mask, int ldm, void *c, int ldc, void *ct, int ldct, float *cf,
               int ldcf, int splits, void *stream) {
    return gemm_launch(a, lda, b, ldb, M, N, K, bias, relu, mask, ldm, c, ldc, ct, ldct, cf, ldcf, splits, a_mn != 0,
                       b_mn != 0, stream);
}

int d1_gemm_single(const void *a, int lda, int a_mn, const void *b, int ldb, int b_mn, int M, int N, int K,
                   const float *bias, int relu, const void *mask, int ldm, void *c, int ldc, void *ct, int ldct,
                   float *cf, int ldcf, int splits, void *stream) {
    return gemm_launch(a, lda, b, ldb, M, N, K, bias, relu, mask, ldm, c, ldc, ct, ldct, cf, ldcf, splits, a_mn != 0,
                       b_mn != 0, stream, nullptr, 0, nullptr, 0, false);
}

int d1_gemm_rows(const void *a, int lda, int a_mn, const int64_t *a_rows, int a_table_rows, const void *b, int ldb,
                 int b_mn, const int64_t *b_rows, int b_table_rows, int M, int N, int K, const float *bias, int relu,
                 const void *mask, int ldm, void *c, int ldc, float *cf, int ldcf, int splits, void *stream) {
    return gemm_launch(a, lda, b, ldb, M, N, K, bias, relu, mask, ldm, c, ldc, nullptr, 0, cf, ldcf, splits,
                       a_mn != 0, b_mn != 0, stream, a_rows, a_table_rows, b_rows, b_table_rows);
}

int d1_gemm_bkn(const void *a, int lda, const void *b_kn, int ldb, int M, int N, int K, const float *bias, int relu,
                void *c, int ldc, float *cf, int ldcf, int splits, void *stream) {
    return gemm_launch(a, lda, b_kn, ldb, M, N, K, bias, relu, nullptr, 0, c, ldc, nullptr, 0, cf, ldcf, splits, 0,
                       1, stream);
}

int d1_gemm_head_sample(const void *a, int lda, const void *b, int ldb, int M, int K, const float *bias,
                        const void *wh_bf16, const float *bh, const uint16_t *legal, uint64_t seed, uint64_t step,
                        int first_env, int64_t *action, float *logp, float *value, float *logits, void *stream) {
    if (M <= 0 || K <= 0 || !a || !b || !wh_bf16 || !bh) return D1_ERR_BAD_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15) || (lda * 2) % 16 ||
        (ldb * 2) % 16 || lda < K || ldb < K)
        return D1_ERR_BAD_ARGUMENT;
    const int kt = (K + BK - 1) / BK;
    CUtensorMap ma, mb;
    if (!make_map(&ma, a, M, K, lda, BM) || !make_map(&mb, b, BN, K, ldb, BN)) return D1_ERR_BAD_ARGUMENT;
    if (int e = gemm_attr()) return e;
    Params p{M, BN, K, kt, kt, bias, 1, 0, nullptr, nullptr, 0, nullptr, nullptr, nullptr, 0, nullptr, 0, nullptr, 0,
             nullptr, 0, 1, (const __nv_bfloat16 *)wh_bf16, bh, legal, seed, step, first_env, action, logp, value,
             logits};
    const int tiles = (M + BM - 1) / BM;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = SM_COUNT;
    const int grid = tiles < sms ? tiles : sms;
    gemm_kernel<true><<<grid, THREADS, SMEM_HEAD_BYTES, (cudaStream_t)stream>>>(ma, mb, p, tiles, 1, tiles);
    return (int)cudaGetLastError();
}

// 2-SM pair kernel: 256 x 256 tiles (see gemm_pair_kernel). Same operands and
// output forms as gemm_launch except the transposed output and row gathers;
// xm = 1 / 2 builds A / B from compact observation rows instead (a / b unused).
static int pair_launch(const void *a, int lda, const void *b, int ldb, int M, int N, int K, const float *bias, int relu,
                       const void *mask, int ldm, void *c, int ldc, float *cf, int ldcf, int splits, int a_mn,
                       int b_mn, void *stream, int xm, const uint8_t *cobs, const int64_t *cidx) {
    if (M <= 0 || N <= 0 || K <= 0 || (!a && xm != 1) || (!b && xm != 2) || (!c && !cf) || splits < 1)
        return D1_ERR_BAD_ARGUMENT;
    if (xm && (!cobs || (reinterpret_cast<uintptr_t>(cobs) & 15))) return D1_ERR_BAD_ARGUMENT;
    if (xm == 1 && (a_mn || K != X_K)) return D1_ERR_BAD_ARGUMENT;
    if (xm == 2 && (!b_mn || N > X_K + 8)) return D1_ERR_BAD_ARGUMENT;
    if ((xm != 1 && ((reinterpret_cast<uintptr_t>(a) & 15) || (lda * 2) % 16 || lda < (a_mn ? M : K))) ||
        (xm != 2 && ((reinterpret_cast<uintptr_t>(b) & 15) || (ldb * 2) % 16 || ldb < (b_mn ? N : K))))
        return D1_ERR_BAD_ARGUMENT;
    if (c && ((reinterpret_cast<uintptr_t>(c) & 15) || ldc % 8 || ldc < N)) return D1_ERR_BAD_ARGUMENT;
    if (cf && ((reinterpret_cast<uintptr_t>(cf) & 15) || ldcf % 4 || ldcf < N)) return D1_ERR_BAD_ARGUMENT;
    if (mask && ((reinterpret_cast<uintptr_t>(mask) & 15) || ldm % 8 || ldm < N)) return D1_ERR_BAD_ARGUMENT;
    if (splits > 1 && c) return D1_ERR_BAD_ARGUMENT;
    const int kt = (K + BK - 1) / BK;
    if (splits > kt) splits = kt;
    const int per = (kt + splits - 1) / splits;
    splits = (kt + per - 1) / per;
    CUtensorMap ma, mb;
    // each CTA loads 128 rows (K-major) or two 64-wide MN atoms (MN-major) of A and of B
    if (xm != 1 && !(a_mn ? make_map(&ma, a, K, M, lda, 64) : make_map(&ma, a, M, K, lda, 128)))
        return D1_ERR_BAD_ARGUMENT;
    if (xm != 2 && !(b_mn ? make_map(&mb, b, K, N, ldb, 64) : make_map(&mb, b, N, K, ldb, 128)))
        return D1_ERR_BAD_ARGUMENT;
    if (xm == 1) ma = mb;  // unused: the expanded operand has no tensor map
    if (xm == 2) mb = ma;
    static uint64_t ready = 0;
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev)) return (int)e;
    if (!(dev < 64 && ((ready >> dev) & 1))) {
        cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<1, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             P_SMEM_BYTES);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_pair_kernel<2, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     P2_SMEM_BYTES);
        for (int xm = 1; xm <= 2 && e == cudaSuccess; xm++) {
            e = cudaFuncSetAttribute(xm == 1 ? gemm_pair_kernel<1, 1> : gemm_pair_kernel<1, 2>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES + X_SMEM_BYTES);
            if (e == cudaSuccess)
                e = cudaFuncSetAttribute(xm == 1 ? gemm_pair_kernel<2, 1> : gemm_pair_kernel<2, 2>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, P2_SMEM_BYTES + X_SMEM_BYTES);
        }
        if (e != cudaSuccess) return (int)e;
        if (dev < 64) ready |= 1ull << dev;
    }
    Params p{M, N, K, per, kt, bias, relu, a_mn, nullptr, nullptr, b_mn, cobs, cidx, (const __nv_bfloat16 *)mask,
             ldm, (__nv_bfloat16 *)c, ldc, nullptr, 0, cf, ldcf};
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = SM_COUNT;
    const int tiles_n = (N + BN - 1) / BN;
    // 512-row pair tiles (B streamed half as often) once M is large enough for
    // them to still give every pair a tile (measured: rollout layer 1, 65,536 x
    // 256 x 1832: 74.7 -> 68.0 us)
    const int sub = (M >= 8192 && ((M + 511) / 512) * tiles_n * splits >= sms / 2) ? 2 : 1;
    const int tiles_m = (M + 256 * sub - 1) / (256 * sub);
    const int tiles = tiles_m * tiles_n * splits;
    const int clusters = tiles < sms / 2 ? tiles : sms / 2;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // launch and prologue may overlap the end of the stream's previous kernel
    // (the kernel's pdl_wait precedes its first global access)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(THREADS + (xm ? 32 * X_EXPANDERS : 0));
    cfg.dynamicSmemBytes = (sub == 2 ? P2_SMEM_BYTES : P_SMEM_BYTES) + (xm ? X_SMEM_BYTES : 0);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    void (*kern)(const CUtensorMap, const CUtensorMap, Params, int, int, int) =
        sub == 2 ? (xm == 1 ? gemm_pair_kernel<2, 1> : xm == 2 ? gemm_pair_kernel<2, 2> : gemm_pair_kernel<2, 0>)
                 : (xm == 1 ? gemm_pair_kernel<1, 1> : xm == 2 ? gemm_pair_kernel<1, 2> : gemm_pair_kernel<1, 0>);
    return (int)cudaLaunchKernelEx(&cfg, kern, ma, mb, p, tiles_m, tiles_n, tiles);
}

int d1_gemm_pair(const void *a, int lda, int a_mn, const void *b, int ldb, int b_mn, int M, int N, int K,
                 const float *bias, int relu, const void *mask, int ldm, void *c, int ldc, float *cf, int ldcf,
                 int splits, void *stream) {
    return pair_launch(a, lda, b, ldb, M, N, K, bias, relu, mask, ldm, c, ldc, cf, ldcf, splits, a_mn != 0, b_mn != 0,
                       stream, 0, nullptr, nullptr);
}

int d1_gemm_cobs_a(const void *cobs, const int64_t *idx, int M, const void *b, int ldb, int N, const float *bias,
                   int relu, void *c, int ldc, void *stream) {
    return pair_launch(nullptr, 0, b, ldb, M, N, X_K, bias, relu, nullptr, 0, c, ldc, nullptr, 0, 1, 0, 0, stream, 1,
                       (const uint8_t *)cobs, idx);
}

int d1_gemm_cobs_b(const void *a, int lda, const void *cobs, const int64_t *idx, int M, int N, int K, float *cf,
                   int ldcf, int splits, void *stream) {
    return pair_launch(a, lda, nullptr, 0, M, N, K, nullptr, 0, nullptr, 0, nullptr, 0, cf, ldcf, splits, 1, 1, stream,
                       2, (const uint8_t *)cobs, idx);
}

// Splits actually used for (K, requested splits): callers size fp32 slabs with it.
int d1_gemm_splits(int K, int splits) {
    if (K <= 0) return D1_ERR_BAD_ARGUMENT;
    const int kt = (K + BK - 1) / BK;
    if (splits < 1) splits = 1;
    if (splits > kt) splits = kt;
    const int per = (kt + splits - 1) / splits;
    return (kt + per - 1) / per;
}

// Last error recorded by a GEMM wait that expired (0 = none); clears it.
int d1_gemm_error(void) {
    int h = 0, z = 0;
    if (cudaMemcpyFromSymbol(&h, g_error, sizeof(int)) != cudaSuccess) return -1;
    if (h) cudaMemcpyToSymbol(g_error, &z, sizeof(int));
    return h;
}

}  // extern "C"

// ---------------------------------------------------------------- no-allocation variant
// Some callers of this library cannot allocate device memory at all: code that
// runs inside another framework's memory arena with no allocator handle, a
// plugin loaded where cudaMalloc is forbidden after start-up, or a process that
// has already handed every byte of HBM to a pool. For them the split-K
// weight-gradient product keeps its partial-product slabs in this file-scope
// device array (16 MiB, reserved on every GPU that loads the library until the
// process exits). Every call shares it and it keeps the last call's contents;
// nothing in it needs to start at zero (each call writes every slab element it
// reads). Calls whose work overlaps on the GPU (different streams, or
// different host threads on one device) race on it and must be serialised by
// the caller.
namespace d1 {
namespace tc {
constexpr int64_t NOALLOC_FLOATS = 4 * 1024 * 1024;
static __device__ __align__(256) float g_noalloc_slabs[NOALLOC_FLOATS];

__global__ void reduce_2d_kernel(const float *__restrict__ slabs, int splits, int M, int N, int ldcf,
                                 float *__restrict__ out, int ldo) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)M * N) return;
    const int r = (int)(i / N), c = (int)(i % N);
    float s = 0.f;
    for (int k = 0; k < splits; k++) s += slabs[(size_t)k * M * ldcf + (size_t)r * ldcf + c];
    out[(size_t)r * ldo + c] = s;
}

// Host-side `g_noalloc_slabs` names a host stand-in, not device memory: the
// device address is looked up with cudaGetSymbolAddress once per device, with
// that device current, on the first call made on it (so that first call should
// come before any stream capture). Concurrent first calls from several host
// threads may each look it up; they find the same address and publish it
// through an atomic. The cached address belongs to the device's primary
// context: after cudaDeviceReset on a device, this entry point must not be
// called again on that device in the same process.
static float *noalloc_scratch(int *err) {
    static std::atomic<float *> ptrs[128];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 128) {
        *err = e != cudaSuccess ? (int)e : D1_ERR_BAD_ARGUMENT;
        return nullptr;
    }
    float *cached = ptrs[dev].load(std::memory_order_acquire);
    if (!cached) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_slabs);
        if (e != cudaSuccess || !p) {
            *err = e != cudaSuccess ? (int)e : D1_ERR_BAD_ARGUMENT;
            return nullptr;
        }
        cached = static_cast<float *>(p);
        ptrs[dev].store(cached, std::memory_order_release);
    }
    return cached;
}
}  // namespace tc
}  // namespace d1

extern "C" int d1_gemm_wgrad_noalloc(const void *a, int lda, const void *b, int ldb, int M, int N, int K, float *out,
                                     int ldo, int splits, void *stream) {
    using namespace d1::tc;
    if (M <= 0 || N <= 0 || K <= 0 || !a || !b || !out || ldo < N || splits < 1) return D1_ERR_BAD_ARGUMENT;
    const int used = d1_gemm_splits(K, splits);
    const int ldcf = (N + 3) / 4 * 4;
    if ((int64_t)used * M * ldcf > NOALLOC_FLOATS) return D1_ERR_TOO_LARGE;
    int err = 0;
    float *slabs = noalloc_scratch(&err);
    if (!slabs) return err;
    int code = d1_gemm(a, lda, b, ldb, M, N, K, nullptr, 0, nullptr, 0, nullptr, 0, nullptr, 0, slabs, ldcf, used,
                       stream);
    if (code) return code;
    const int64_t total = (int64_t)M * N;
    reduce_2d_kernel<<<(unsigned)((total + 255) / 256), 256, 0, (cudaStream_t)stream>>>(slabs, used, M, N, ldcf, out,
                                                                                          ldo);
    return (int)cudaGetLastError();
}
