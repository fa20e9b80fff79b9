// Conv encoder of the centered-map policy on the
// 5th-generation tensor cores:
//
//   crop 63x63x10 --conv 3x3/2, ReLU--> 31x31x32 --conv 3x3/2, ReLU--> 15x15x64
//                 --conv 3x3/2, ReLU--> 7x7x64 (flattened NHWC: 3136 features)
//
// The reference runs this stack as torch Conv2d layers over a recentred map
// built by an encode kernel (gpu-d1/branches/vision15-centered-map-v1/src/
// fast_maps.cu:4-17, scripts/tactical_models.py:11-62).
//
// Implicit GEMM without im2col. A stride-2 3x3 conv reads input pixel
// (2*oy + ky, 2*ox + kx). Each layer's input is stored as four "phase planes"
// P[py][px][y'][x'] = in[2y' + py][2x' + px] with a row pitch PW equal to the
// output row pitch, so for tap (ky, kx) the operand rows of output pixels
// r = oy*PW + ox are rows r + (ky/2)*PW + kx/2 of plane P[ky%2][kx%2]: one
// contiguous run. A tap is therefore a plain shared-memory matrix descriptor
// (canonical K-major layout without swizzle: 8-row core matrices of 16-byte
// rows, channel chunks of 8 one plane apart) at a shifted start address, and
// the conv is 9 taps x (Cin/16) tcgen05.mma (M=128, N=Cout, K=16) accumulating
// in TMEM. Output columns ox >= the valid width and rows past the output are
// computed from neighbouring data and discarded by the epilogue.
//
// Each CTA walks units, several CTAs per SM so one CTA's MMAs overlap the
// others' staging and epilogues: layer 1 (four 128-thread CTAs per SM) = a
// quarter env (8 output rows), expanded from the u16 crop codes into one-hot
// bf16 planes in shared memory, the next quarter's crop rows prefetched into
// registers while the MMAs run; layers 2 and 3 (two 256-thread CTAs per SM) =
// one env, whose planes the previous layer's epilogue
// wrote to global memory in exactly the shared-memory layout, so one bulk copy
// stages them. The epilogue (TMEM -> bias, ReLU -> bf16) scatters every output
// pixel into the next layer's phase planes (or the FC input). Weights stay in
// shared memory for the CTA's lifetime. Every mbarrier wait is bounded; on
// expiry the kernel records an error (d1_conv_error) and frees its TMEM.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/d1.h"

namespace d1 {
namespace conv {

constexpr int CROP_PITCH = 64, CROP_ROWS = 63;
constexpr uint32_t WAIT_LIMIT = 1u << 22;
__device__ int g_error;

template <int L>
struct Geo;
// layer 1: crop codes -> 31x31x32; unit = a quarter env (8 output rows from 9
// phase rows = 18 crop rows); four 128-thread CTAs per SM
template <>
struct Geo<1> {
    static constexpr int CIN = 10, CHUNKS = 2, N = 32, PW = 32, PLANE = 9 * 32, MT = 2, UNITS = 4, TAIL = 64;
    static constexpr int THREADS = 128, CTAS_PER_SM = 4, ROWS_IN = 18;
    static constexpr int OUT_BYTES = 4 * 4 * 256 * 16;  // layer-2 planes
};
// layer 2: 31x31x32 -> 15x15x64
template <>
struct Geo<2> {
    static constexpr int CIN = 32, CHUNKS = 4, N = 64, PW = 16, PLANE = 256, MT = 2, UNITS = 1, TAIL = 32;
    static constexpr int THREADS = 256, CTAS_PER_SM = 2;
    static constexpr int OUT_BYTES = 4 * 8 * 64 * 16;  // layer-3 planes
};
// layer 3: 15x15x64 -> 7x7x64 = FC input
template <>
struct Geo<3> {
    static constexpr int CIN = 64, CHUNKS = 8, N = 64, PW = 8, PLANE = 64, MT = 1, UNITS = 1, TAIL = 80;
    static constexpr int THREADS = 256, CTAS_PER_SM = 2;
    static constexpr int OUT_BYTES = 49 * 64 * 2;
};
template <int L>
struct Lay {
    using G = Geo<L>;
    static constexpr int IN_BYTES = 4 * G::CHUNKS * G::PLANE * 16;     // planes of one unit
    static constexpr int IN_SMEM = IN_BYTES + G::TAIL * 16;            // + overrun pad
    static constexpr int W_BYTES = 9 * G::CHUNKS * G::N * 16;
    static constexpr int STAGE_BYTES = L == 1 ? 18 * CROP_PITCH * 2 : 0;  // crop rows of a quarter
    static constexpr int OFF_W = IN_SMEM, OFF_BIAS = OFF_W + W_BYTES, OFF_STAGE = OFF_BIAS + G::N * 4;
    static constexpr int OFF_BAR = (OFF_STAGE + STAGE_BYTES + 15) & ~15;
    static constexpr int SMEM = OFF_BAR + 64;
    static constexpr uint32_t TMEM_COLS = G::MT * G::N;
    static constexpr uint32_t IDESC =
        (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(G::N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
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
// Canonical K-major layout without swizzle: rows of 16 bytes, 8-row core
// matrices SBO = 128 B apart along M/N, the two 8-element K halves LBO apart.
__device__ __forceinline__ uint64_t desc_noswizzle(uint32_t addr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)(128u >> 4) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version
    return d;                // layout type 0: no swizzle
}
__device__ __forceinline__ void mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

#define D1_CONV_TMEM_LD32(taddr, v)                                                                                 \
    asm volatile(                                                                                                   \
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                             \
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),          \
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),    \
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),  \
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])   \
        : "r"(taddr))

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
// 32 accumulator columns -> bias, ReLU -> 4 x 16 bytes of bf16 (8 channels each)
__device__ __forceinline__ void finish32(const uint32_t *v, const float *bias, uint4 *o) {
#pragma unroll
    for (int c = 0; c < 4; c++) {
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; j++) f[j] = fmaxf(__uint_as_float(v[8 * c + j]) + bias[8 * c + j], 0.f);
        o[c] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                          pack_bf16x2(f[6], f[7]));
    }
}

// Layer-1 staging of a quarter env: its 18 crop rows (zero past row 62) are
// fetched into registers (the next unit's while the current unit's MMAs run),
// stored to shared memory, and every phase-plane pixel expanded to 16 channels:
// one-hot class (0-7), monster hp / 32 (8), on-the-map flag (9), zeros.
constexpr int STAGE_VECS = 18 * CROP_PITCH * 2 / 16;                    // uint4 per unit
constexpr int STAGE_REGS = (STAGE_VECS + Geo<1>::THREADS - 1) / Geo<1>::THREADS;
__device__ __forceinline__ void fetch_crop(const uint16_t *__restrict__ crop, int unit, int units, uint4 *r) {
    const int env = unit >> 2, quarter = unit & 3;
    const uint4 *src = reinterpret_cast<const uint4 *>(crop + (size_t)env * CROP_ROWS * CROP_PITCH);
    constexpr int VPR = CROP_PITCH * 2 / 16;
#pragma unroll
    for (int k = 0; k < STAGE_REGS; k++) {
        const int i = threadIdx.x + k * Geo<1>::THREADS;
        const int y = 16 * quarter + i / VPR;
        r[k] = (unit < units && i < STAGE_VECS && y < CROP_ROWS) ? __ldg(src + y * VPR + i % VPR)
                                                                  : make_uint4(0, 0, 0, 0);
    }
}
__device__ void expand_crop(const uint4 *r, uint8_t *smem) {
    using Y = Lay<1>;
    uint4 *st = reinterpret_cast<uint4 *>(smem + Y::OFF_STAGE);
#pragma unroll
    for (int k = 0; k < STAGE_REGS; k++) {
        const int i = threadIdx.x + k * Geo<1>::THREADS;
        if (i < STAGE_VECS) st[i] = r[k];
    }
    __syncthreads();
    const uint16_t *rows = reinterpret_cast<const uint16_t *>(st);
    uint4 *planes = reinterpret_cast<uint4 *>(smem);
    constexpr int PLANE = Geo<1>::PLANE;
    for (int e = threadIdx.x; e < 4 * PLANE; e += Geo<1>::THREADS) {
        const int phase = e / PLANE, pos = e - phase * PLANE;
        const int yl = pos >> 5, xp = pos & 31;
        const int y = 2 * yl + (phase >> 1), x = 2 * xp + (phase & 1);
        const uint32_t code = rows[y * CROP_PITCH + x];
        const uint32_t cls = code & 7u, one = 0x3F80u << (16 * (cls & 1u));
        const uint32_t w = cls >> 1;
        const uint4 c0 = make_uint4(w == 0 ? one : 0u, w == 1 ? one : 0u, w == 2 ? one : 0u, w == 3 ? one : 0u);
        const __nv_bfloat16 hp = __float2bfloat16_rn((float)((code >> 4) & 31u) * 0.03125f);
        const uint32_t lo = *reinterpret_cast<const uint16_t *>(&hp);
        const uint4 c1 = make_uint4(lo | (((code >> 3) & 1u) ? 0x3F800000u : 0u), 0u, 0u, 0u);
        planes[(phase * 2 + 0) * PLANE + pos] = c0;
        planes[(phase * 2 + 1) * PLANE + pos] = c1;
    }
}

template <int L>
__global__ void __launch_bounds__(Geo<L>::THREADS, Geo<L>::CTAS_PER_SM)
    conv_kernel(const void *__restrict__ in, int n, const uint4 *__restrict__ w, const float *__restrict__ bias,
                uint8_t *__restrict__ out) {
    using G = Geo<L>;
    using Y = Lay<L>;
    constexpr int THREADS = G::THREADS, WGROUPS = THREADS / 128;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Y::OFF_BAR);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2);
    int *abort_s = reinterpret_cast<int *>(bars + 3);
    const uint32_t in_bar = smem_u32(bars), mma_bar = smem_u32(bars + 1);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float *bias_s = reinterpret_cast<float *>(smem + Y::OFF_BIAS);

    // weights (already in the shared-memory layout) and bias, once per CTA
    uint4 *w_s = reinterpret_cast<uint4 *>(smem + Y::OFF_W);
    for (int i = tid; i < Y::W_BYTES / 16; i += THREADS) w_s[i] = __ldg(w + i);
    for (int i = tid; i < G::N; i += THREADS) bias_s[i] = bias[i];
    // zero the overrun pad after the last plane (read only by discarded rows)
    for (int i = tid; i < G::TAIL; i += THREADS) reinterpret_cast<uint4 *>(smem + Y::IN_BYTES)[i] = make_uint4(0, 0, 0, 0);
    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(in_bar) : "memory");
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mma_bar) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        *abort_s = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(Y::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fence_proxy_async();
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t in_base = smem_u32(smem), w_base = smem_u32(w_s);
    const int units = n * G::UNITS;
    uint32_t it = 0;
    uint4 pre[L == 1 ? STAGE_REGS : 1];
    if constexpr (L == 1) fetch_crop(static_cast<const uint16_t *>(in), blockIdx.x, units, pre);
    // Layers 2 and 3: one bulk copy of a unit's planes into the input buffer,
    // completing on in_bar.
    bool outstanding = false;  // thread 0: a requested copy not yet waited for
    uint32_t out_parity = 0;
    auto request = [&](int unit, uint32_t parity) {
        if constexpr (L != 1) {
            if (tid == 0 && unit < units) {
                outstanding = true;
                out_parity = parity;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(in_bar),
                             "r"((uint32_t)Y::IN_BYTES)
                             : "memory");
                const uint8_t *src = static_cast<const uint8_t *>(in) + (size_t)unit * Y::IN_BYTES;
                constexpr int PIECE = 16384;
#pragma unroll 1
                for (int off = 0; off < Y::IN_BYTES; off += PIECE)
                    bulk_load(in_base + off, src + off, (uint32_t)min(PIECE, Y::IN_BYTES - off), in_bar);
            }
        }
    };
    request(blockIdx.x, 0u);
    for (int u = blockIdx.x; u < units; u += gridDim.x, it++) {
        const int env = u / G::UNITS, part = u % G::UNITS;
        // ---- stage the unit's input planes
        if constexpr (L == 1) {
            expand_crop(pre, smem);
            fence_proxy_async();
            __syncthreads();
        } else {
            // the unit's planes were requested when the previous unit's MMAs
            // completed (or before the loop for the first unit)
            (void)env;
        }
        // ---- MMAs: M tiles x 9 taps x K steps
        if (tid == 0) {
            bool ok = true;
            if constexpr (L != 1) {
                ok = mbar_wait(in_bar, it & 1u);
                if (ok) outstanding = false;
            }
            if (!ok) {
                atomicExch(&g_error, 1);
                *abort_s = 1;
            } else {
                fence_after();
#pragma unroll 1
                for (int m = 0; m < G::MT; m++) {
#pragma unroll 1
                    for (int tap = 0; tap < 9; tap++) {
                        const int ky = tap / 3, kx = tap % 3;
                        const int phase = (ky & 1) * 2 + (kx & 1), shift = (ky >> 1) * G::PW + (kx >> 1);
#pragma unroll
                        for (int s = 0; s < G::CHUNKS / 2; s++) {
                            const uint32_t a = in_base + (uint32_t)(((phase * G::CHUNKS + 2 * s) * G::PLANE + m * 128 +
                                                                     shift) * 16);
                            const uint32_t b = w_base + (uint32_t)((tap * G::CHUNKS + 2 * s) * G::N * 16);
                            mma(tmem + (uint32_t)(m * G::N), desc_noswizzle(a, G::PLANE * 16),
                                desc_noswizzle(b, G::N * 16), Y::IDESC, (tap | s) ? 1u : 0u);
                        }
                    }
                }
                mma_commit(mma_bar);
            }
        }
        __syncthreads();
        if (*abort_s) break;
        // the next unit's crop rows load while the MMAs run
        if constexpr (L == 1) fetch_crop(static_cast<const uint16_t *>(in), u + gridDim.x, units, pre);
        const bool done = mbar_wait(mma_bar, it & 1u);
        if (!done) {
            atomicExch(&g_error, 2);
            *abort_s = 1;
        }
        fence_after();
        __syncthreads();
        if (*abort_s) break;
        // the input buffer is free: the next unit's planes load during the epilogue
        request(u + gridDim.x, (it + 1) & 1u);
        // ---- epilogue: warp w reads TMEM lanes 32*(w%4).. of its tiles / column chunks
        const int q = warp & 3, wh = warp >> 2;
        if constexpr (L == 1) {
#pragma unroll 1
            for (int m = wh; m < G::MT; m += WGROUPS) {
                uint32_t v[32];
                D1_CONV_TMEM_LD32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(m * G::N), v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int oy = 8 * part + m * 4 + q, ox = lane;
                if (oy < 31 && ox < 31) {
                    uint4 o[4];
                    finish32(v, bias_s, o);
                    uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)env * G::OUT_BYTES);
                    const int ph = (oy & 1) * 2 + (ox & 1), pos = (oy >> 1) * 16 + (ox >> 1);
#pragma unroll
                    for (int c = 0; c < 4; c++) dst[(ph * 4 + c) * 256 + pos] = o[c];
                }
            }
        } else if constexpr (L == 2) {
            const int m = wh;
            const int r = m * 128 + q * 32 + lane, oy = r >> 4, ox = r & 15;
#pragma unroll 1
            for (int cc = 0; cc < 2; cc++) {
                uint32_t v[32];
                D1_CONV_TMEM_LD32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(m * G::N + cc * 32), v);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (oy < 15 && ox < 15) {
                    uint4 o[4];
                    finish32(v, bias_s + cc * 32, o);
                    uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)env * G::OUT_BYTES);
                    const int ph = (oy & 1) * 2 + (ox & 1), pos = (oy >> 1) * 8 + (ox >> 1);
#pragma unroll
                    for (int c = 0; c < 4; c++) dst[(ph * 8 + cc * 4 + c) * 64 + pos] = o[c];
                }
            }
        } else {
            const int cc = wh;
            const int r = q * 32 + lane, oy = r >> 3, ox = r & 7;
            uint32_t v[32];
            D1_CONV_TMEM_LD32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(cc * 32), v);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (oy < 7 && ox < 7) {
                uint4 o[4];
                finish32(v, bias_s + cc * 32, o);
                uint4 *dst = reinterpret_cast<uint4 *>(out + (size_t)env * G::OUT_BYTES + ((oy * 7 + ox) * 64 + cc * 32) * 2);
#pragma unroll
                for (int c = 0; c < 4; c++) dst[c] = o[c];
            }
        }
        // TMEM and the input planes are free for the next unit
        fence_before();
        __syncthreads();
    }
    // after an abort, let a copy still in flight land before the CTA exits
    if (tid == 0 && outstanding) mbar_wait(in_bar, out_parity);
    fence_before();
    __syncthreads();
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Y::TMEM_COLS)
                     : "memory");
    }
}

// Pack torch-layout weights fp32 [Cout, Cin, 3, 3] into the shared-memory
// operand layout: [tap][chunk of 8 input channels][Cout][8] bf16, zero for
// channels >= Cin.
template <int L>
__global__ void pack_kernel(const float *__restrict__ wt, __nv_bfloat16 *__restrict__ out) {
    using G = Geo<L>;
    const int total = 9 * G::CHUNKS * G::N * 8;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int ci8 = i & 7, nn = (i >> 3) % G::N, chunk = (i >> 3) / G::N % G::CHUNKS, tap = (i >> 3) / G::N / G::CHUNKS;
        const int ci = chunk * 8 + ci8;
        const float v = ci < G::CIN ? wt[((size_t)nn * G::CIN + ci) * 9 + tap] : 0.f;
        out[i] = __float2bfloat16_rn(v);
    }
}

template <int L>
static int launch(const void *in, int n, const void *w, const float *bias, void *out, cudaStream_t stream) {
    using Y = Lay<L>;
    static uint64_t ready = 0;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 64 || !((ready >> dev) & 1)) {
        e = cudaFuncSetAttribute(conv_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize, Y::SMEM);
        if (e != cudaSuccess) return (int)e;
        if (dev < 64) ready |= 1ull << dev;
    }
    const int units = n * Geo<L>::UNITS, slots = Geo<L>::CTAS_PER_SM * 148;
    const int grid = units < slots ? units : slots;
    conv_kernel<L><<<grid, Geo<L>::THREADS, Y::SMEM, stream>>>(in, n, static_cast<const uint4 *>(w), bias,
                                                         static_cast<uint8_t *>(out));
    return (int)cudaGetLastError();
}

}  // namespace conv
}  // namespace d1

using namespace d1;

extern "C" {

int d1_conv_in_bytes(int layer) {
    switch (layer) {
        case 1: return conv::CROP_ROWS * conv::CROP_PITCH * 2;
        case 2: return conv::Lay<2>::IN_BYTES;
        case 3: return conv::Lay<3>::IN_BYTES;
        case 4: return conv::Geo<3>::OUT_BYTES;
        default: return 0;
    }
}

int d1_conv_weight_bytes(int layer) {
    switch (layer) {
        case 1: return conv::Lay<1>::W_BYTES;
        case 2: return conv::Lay<2>::W_BYTES;
        case 3: return conv::Lay<3>::W_BYTES;
        default: return 0;
    }
}

int d1_conv_pack_weights(int layer, const float *w, void *packed, void *stream) {
    if (!w || !packed) return D1_ERR_BAD_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    switch (layer) {
        case 1: conv::pack_kernel<1><<<16, 256, 0, s>>>(w, (__nv_bfloat16 *)packed); break;
        case 2: conv::pack_kernel<2><<<64, 256, 0, s>>>(w, (__nv_bfloat16 *)packed); break;
        case 3: conv::pack_kernel<3><<<128, 256, 0, s>>>(w, (__nv_bfloat16 *)packed); break;
        default: return D1_ERR_BAD_ARGUMENT;
    }
    return (int)cudaGetLastError();
}

int d1_conv_layer(int layer, const void *in, int n, const void *w_packed, const float *bias, void *out,
                  void *stream) {
    if (n < 0 || !in || !w_packed || !bias || !out) return D1_ERR_BAD_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(w_packed) | reinterpret_cast<uintptr_t>(out)) &
        15)
        return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    cudaStream_t s = (cudaStream_t)stream;
    switch (layer) {
        case 1: return conv::launch<1>(in, n, w_packed, bias, out, s);
        case 2: return conv::launch<2>(in, n, w_packed, bias, out, s);
        case 3: return conv::launch<3>(in, n, w_packed, bias, out, s);
        default: return D1_ERR_BAD_ARGUMENT;
    }
}

int d1_conv_error(void) {
    int h = 0;
    cudaDeviceSynchronize();
    cudaMemcpyFromSymbol(&h, conv::g_error, sizeof(int));
    const int zero = 0;
    cudaMemcpyToSymbol(conv::g_error, &zero, sizeof(int));
    return h;
}

}  // extern "C"
