// The tail of a PPO minibatch in one launch on the 5th-generation tensor cores
// (sm_100a tcgen05 + TMA): layer 2, the policy/value head, the clipped PPO
// loss and its backward down to the first hidden layer, for 128 rows per CTA.
// It replaces three launches of the unfused update (layer-2 GEMM, the loss
// kernel, the dh1 GEMM), whose fixed costs dominated their ~1.5 us of math.
//
//   h2     = relu(h1 W2^T + b2)                  MMA M128 N256, K 256     (TMEM cols 0-255)
//   head   = h2 Wh^T + bh  (12 logits, value)    MMA M128 N16, K 256      (cols 256-271)
//   loss, dhead (fp32, one thread per row; the reference's per-row formulas,
//          gpu-d1/scripts/run_ring_ablations.py:363-372 with BASELINE config
//          2's value clip and coefficients)
//   dh2    = relu'(h2) * (dhead Wh)              MMA M128 N256, K 16 x2 (dhead as bf16 hi + lo)
//   dWh^T  = h2^T [dhi | dlo] (CTA partial)      MMA M128 N32, K 128 x2 halves (cols 288-319, 320-351)
//   dh1    = relu'(h1) * (dh2 W2)                MMA M128 N256, K 256, W2 read MN-major from the same tile
// plus the partial sums db2 = sum_r dh2 (of the bf16 values), dbh = sum_r dhead
// and the loss terms, in the layout of d1_ppo_loss's block partials.
//
// Shared memory holds W2 (128 KB) for the whole CTA and one 128 x 256 bf16
// activation tile that is h1 (TMA), then h2, then dh2, then dh1 (written by
// the epilogue in the same 128-byte-swizzled layout the tensor cores read;
// dh2 and dh1 leave by TMA stores from it, so every global write is a full
// line). The rounding points are those of the unfused path: h2, dh2 and dh1
// are stored as bf16, dhead enters the products as two bf16 parts. Measured
// phase by phase (global timer stamps in a test build): per-thread 16-byte
// row stores of dh2 and dh1 and a re-read of h1 for dh1's mask took 9.8 of
// the kernel's 22 us; the TMA stores and h1's ReLU' bits kept in registers
// from step 1 replace them.
//
// Warp roles (320 threads): warp 0 issues the TMA loads; warp 1 owns the TMEM
// allocation and one lane issues the MMAs; warps 2-9 are the epilogue, warp w
// reading TMEM lanes 32 (w % 4) .. +31 (tile rows) and column half (w - 2) / 4.
// Every mbarrier wait is bounded: on expiry the kernel records an error (read
// by d1_ppo_tail_error), skips the rest of its work and still frees TMEM.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "../../include/d1.h"
#include "d1_pdl.cuh"
#include "tc_ptx.cuh"

namespace d1 {
namespace tail {
using namespace tcx;

__device__ int g_tail_error;  // read and cleared by d1_ppo_tail_error

constexpr int ROWS = 128, HID = 256, NOUT = 13, NACT = 12;
constexpr int PART = NOUT * HID + NOUT + HID + 8;  // d1_ppo_loss_part_len()
constexpr int EPI_WARPS = 8, THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t WAIT_LIMIT = 1u << 22;
// Shared memory, offsets from a 1024-byte aligned base.
constexpr int OFF_W2 = 0;       // W2 [kb 4][out 256][128 B]: columns 64 kb .. +63, 128-byte swizzle
constexpr int OFF_X = 131072;   // activation tile [kb 4][row 128][128 B], 128-byte swizzle
constexpr int OFF_HB = 196608;  // Wh as the head's B [c/8 32][j 16][8 c]; later dhead as dh2's A [part][j/8][row][8 j]
constexpr int OFF_WT = 204800;  // Wh as dh2's B [j/8 2][c 256][8 j]
constexpr int OFF_DB = 212992;  // dhead as dWh^T's B [r/8 16][part*16 + j 32][8 r]
constexpr int OFF_B2 = 221184;  // b2 [256] f32
constexpr int OFF_BH = 222208;  // bh [16] f32
constexpr int OFF_RED = 222272;  // [8 warps][16] f32: dbh sums; [8 warps][8] f32: loss terms
constexpr int OFF_BAR = OFF_RED + 8 * 16 * 4 + 8 * 8 * 4;
constexpr int SMEM = OFF_BAR + 64 + 1024;  // 4 load barriers, MMA, epilogue, abort flag, TMEM slot; slack
constexpr uint32_t TMEM_ALLOC = 512, D_MAIN = 0, D_HEAD = 256, D_DWH = 288;
constexpr uint32_t ID_L2 = idesc_bf16(128, 256, false, false), ID_HEAD = idesc_bf16(128, 16, false, false),
                   ID_DH2 = idesc_bf16(128, 256, false, false), ID_DWH = idesc_bf16(128, 32, true, false),
                   ID_DH1 = idesc_bf16(128, 256, false, true);

struct Args {
    const __nv_bfloat16 *wh;  // [13, 256]
    const float *b2, *bh;
    const int64_t *idx;       // [n] rollout sample ids
    const uint16_t *legal;    // [total]
    const int64_t *action;    // [total]
    const float *old_logp, *adv, *ret, *old_value;  // [total]
    const double *adv_stats;  // sum, sum of squares over adv_count samples
    double adv_count;
    int n;
    float clip, vclip, vf_coef, ent_coef;
    float *part;  // [gridDim.x][PART]
};

// Byte offset of element (row, col) in the swizzled activation tile.
__device__ __forceinline__ uint32_t x_off(int row, int col) {
    return (uint32_t)(OFF_X + (col >> 6) * 16384 + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + ((col & 7) << 1));
}
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

__global__ void __launch_bounds__(THREADS, 1)
    tail_kernel(const __grid_constant__ CUtensorMap map_h1, const __grid_constant__ CUtensorMap map_w2,
                const __grid_constant__ CUtensorMap map_dh2, const __grid_constant__ CUtensorMap map_dh1, Args a) {
    d1::pdl_wait();  // before any global access: h1 and the weights come from the previous kernels
    extern __shared__ uint8_t smem_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t base = smem_u32(sm);
    uint64_t *bars = reinterpret_cast<uint64_t *>(sm + OFF_BAR);
    // bars: load[4] (K block kb of W2 and of h1), MMA done, epilogue step done
    const uint32_t bar_load = smem_u32(bars), bar_mma = smem_u32(bars + 4), bar_epi = smem_u32(bars + 5);
    volatile int *abort_s = reinterpret_cast<volatile int *>(bars + 6);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 7);
    float *b2_s = reinterpret_cast<float *>(sm + OFF_B2), *bh_s = reinterpret_cast<float *>(sm + OFF_BH);
    float *red_bh = reinterpret_cast<float *>(sm + OFF_RED), *red_terms = red_bh + 8 * 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * ROWS;

    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < 4; kb++) mbar_init(bar_load + 8 * kb, 1);
        mbar_init(bar_mma, 1);
        mbar_init(bar_epi, EPI_WARPS);
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
        // ---- TMA: K block kb of this CTA's h1 rows (rows past n read as zero)
        // and of W2, one barrier per block so layer 2 starts on the first
        if (lane == 0) {
            for (int kb = 0; kb < 4; kb++) {
                mbar_expect_tx(bar_load + 8 * kb, 16384 + 32768);
                tma_load_2d(base + OFF_X + kb * 16384, &map_h1, bar_load + 8 * kb, kb * 64, r0);
                tma_load_2d(base + OFF_W2 + kb * 32768, &map_w2, bar_load + 8 * kb, kb * 64, 0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer: four groups, each released by the epilogue's previous step
            int issued = 0;
            bool ok = true;
            // layer 2, K block by K block as the loads land
            for (int kb = 0; kb < 4 && ok; kb++) {
                ok = mbar_wait(bar_load + 8 * kb, 0, WAIT_LIMIT);
                if (!ok) break;
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    mma_bf16(tmem + D_MAIN, desc_sw128_k(base + OFF_X + kb * 16384 + kk * 32),
                             desc_sw128_k(base + OFF_W2 + kb * 32768 + kk * 32), ID_L2, (kb | kk) ? 1u : 0u);
            }
            if (ok) {
                mma_commit(bar_mma);
                issued = 1;
            }
            // head: h2 (now in the tile) against Wh
            ok = ok && mbar_wait(bar_epi, 0, WAIT_LIMIT) && !*abort_s;
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int ks = 0; ks < 16; ks++)
                    mma_bf16(tmem + D_HEAD, desc_sw128_k(base + OFF_X + (ks >> 2) * 16384 + (ks & 3) * 32),
                             desc_plain_k(base + OFF_HB + ks * 512, 256), ID_HEAD, ks ? 1u : 0u);
                mma_commit(bar_mma);
                issued = 2;
            }
            // dh2 = dhead . Wh (hi + lo) and dWh^T = h2^T . dhead per column half
            ok = ok && mbar_wait(bar_epi, 1, WAIT_LIMIT) && !*abort_s;
            if (ok) {
                tc_fence_after();
#pragma unroll
                for (int p = 0; p < 2; p++)
                    mma_bf16(tmem + D_MAIN, desc_plain_k(base + OFF_HB + p * 4096, 2048),
                             desc_plain_k(base + OFF_WT, 4096), ID_DH2, p ? 1u : 0u);
#pragma unroll
                for (int hf = 0; hf < 2; hf++)
#pragma unroll
                    for (int ks = 0; ks < 8; ks++)
                        mma_bf16(tmem + D_DWH + 32 * hf, desc_sw128_mn(base + OFF_X + 2 * hf * 16384 + ks * 2048, 16384),
                                 desc_plain_k(base + OFF_DB + ks * 1024, 512), ID_DWH, ks ? 1u : 0u);
                mma_commit(bar_mma);
                issued = 3;
            }
            // dh1 = dh2 . W2: W2 read MN-major (n = in, k = out rows) from the same tile
            ok = ok && mbar_wait(bar_epi, 0, WAIT_LIMIT) && !*abort_s;
            if (ok) {
                tc_fence_after();
                for (int ko = 0; ko < 4; ko++)
#pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16(tmem + D_MAIN, desc_sw128_k(base + OFF_X + ko * 16384 + kk * 32),
                                 desc_sw128_mn(base + OFF_W2 + (64 * ko + 16 * kk) * 128, 32768), ID_DH1,
                                 (ko | kk) ? 1u : 0u);
                mma_commit(bar_mma);
                issued = 4;
            }
            if (!ok) {
                atomicExch(&g_tail_error, 5);
                *abort_s = 1;
            }
            // the tensor cores are done with TMEM and shared memory before teardown
            if (issued > 0) mbar_wait(bar_mma, (uint32_t)(issued - 1) & 1u, WAIT_LIMIT);
        }
    } else {
        // ---- epilogue: rows q*32 + lane, columns half*128 .. +127
        const int q = warp & 3, half = (warp - 2) >> 2, te = threadIdx.x - 64;
        const int row = q * 32 + lane, grow = r0 + row;
        const bool live = grow < a.n;
        // constants and operand layouts of Wh (the MMAs read them after the first release)
        b2_s[te] = __ldg(a.b2 + te);
        if (te < 16) bh_s[te] = te < NOUT ? __ldg(a.bh + te) : 0.f;
        {
            const int c = te;  // thread per hidden column
            uint16_t w[16];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const __nv_bfloat16 v = j < NOUT ? a.wh[j * HID + c] : __float2bfloat16_rn(0.f);
                w[j] = *reinterpret_cast<const uint16_t *>(&v);
            }
#pragma unroll
            for (int j = 0; j < 16; j++)
                *reinterpret_cast<uint16_t *>(sm + OFF_HB + (c >> 3) * 256 + j * 16 + (c & 7) * 2) = w[j];
#pragma unroll
            for (int h = 0; h < 2; h++)
                *reinterpret_cast<uint4 *>(sm + OFF_WT + h * 4096 + c * 16) =
                    make_uint4(w[8 * h] | ((uint32_t)w[8 * h + 1] << 16), w[8 * h + 2] | ((uint32_t)w[8 * h + 3] << 16),
                               w[8 * h + 4] | ((uint32_t)w[8 * h + 5] << 16),
                               w[8 * h + 6] | ((uint32_t)w[8 * h + 7] << 16));
        }
        fence_proxy_async();
        // this row's sample id (the loss threads: column half 0); its rollout
        // fields are gathered after step 1, off the path to layer 2's epilogue
        const int64_t sid = (half == 0 && live) ? a.idx[grow] : 0;
        const double mean = a.adv_stats[0] / a.adv_count;
        const double var = (a.adv_stats[1] - a.adv_stats[0] * mean) / (a.adv_count - 1.0);
        const float amean = (float)mean, astd = (float)sqrt(var > 0 ? var : 0.0);
        const float inv_n = 1.f / (float)a.n;
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");  // b2_s, bh_s written
        const uint32_t lanes = (uint32_t)(q * 32) << 16;
        bool ok = true;

        // ---- step 1: h2 = relu(acc + b2) as bf16 into the tile, over h1 (whose
        // ReLU' bits this thread keeps for dh1: bit 8u + i of h1m[cc])
        uint32_t h1m[4] = {0u, 0u, 0u, 0u};
        ok = mbar_wait(bar_mma, 0, WAIT_LIMIT);
        if (ok) {
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int c0 = half * 128 + cc * 32;
                uint32_t v[32];
                D1X_TMEM_LD32(tmem + lanes + D_MAIN + (uint32_t)c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    uint4 *cell = reinterpret_cast<uint4 *>(sm + x_off(row, c0 + 8 * u));
                    const uint4 hv = *cell;
                    const __nv_bfloat16 *h = reinterpret_cast<const __nv_bfloat16 *>(&hv);
                    float f[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        if (__bfloat162float(h[i]) > 0.f) h1m[cc] |= 1u << (8 * u + i);
                        f[i] = fmaxf(__uint_as_float(v[8 * u + i]) + b2_s[c0 + 8 * u + i], 0.f);
                    }
                    *cell = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                }
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_epi);

        uint32_t bits = 0;
        int act = 0;
        float olp = 0.f, advv = 0.f, R = 0.f, vold = 0.f;
        if (half == 0 && live) {
            bits = a.legal[sid];
            act = (int)a.action[sid];
            olp = a.old_logp[sid];
            advv = a.adv[sid];
            R = a.ret[sid];
            vold = a.old_value[sid];
        }

        // ---- step 2: head outputs -> loss, dhead (one thread per row)
        float t_pg = 0.f, t_vf = 0.f, t_ent = 0.f, t_clip = 0.f, t_kl = 0.f;
        float dl[16];
#pragma unroll
        for (int j = 0; j < 16; j++) dl[j] = 0.f;
        ok = ok && mbar_wait(bar_mma, 1, WAIT_LIMIT) && !*abort_s;
        if (ok && half == 0) {
            tc_fence_after();
            uint32_t v[16];
            D1X_TMEM_LD16(tmem + lanes + D_HEAD, v);
            tmem_wait_ld();
            if (live) {
                float l[NOUT];
#pragma unroll
                for (int j = 0; j < NOUT; j++) l[j] = __uint_as_float(v[j]) + bh_s[j];
                float m = -3.402823466e38f;
#pragma unroll
                for (int j = 0; j < NACT; j++)
                    if ((bits >> j) & 1u) m = fmaxf(m, l[j]);
                float e[NACT], z = 0.f;
#pragma unroll
                for (int j = 0; j < NACT; j++) {
                    e[j] = ((bits >> j) & 1u) ? expf(l[j] - m) : 0.f;
                    z += e[j];
                }
                const float lz = logf(z), rz = 1.f / z;
                float lp[NACT], p[NACT], ent = 0.f, la = 0.f;
#pragma unroll
                for (int j = 0; j < NACT; j++) {
                    const bool okj = (bits >> j) & 1u;
                    lp[j] = l[j] - m - lz;
                    p[j] = e[j] * rz;
                    if (okj) ent -= p[j] * lp[j];
                    if (j == act) la = lp[j];
                }
                const float value = l[NACT];
                const float adv = (advv - amean) / (astd + 1e-8f);
                const float ratio = expf(la - olp);
                const float s1 = ratio * adv, rc = fminf(fmaxf(ratio, 1.f - a.clip), 1.f + a.clip), s2 = rc * adv;
                const float pg = -fminf(s1, s2);
                float dpg_dr = 0.f;
                if (s1 <= s2) dpg_dr = -adv;
                else if (ratio > 1.f - a.clip && ratio < 1.f + a.clip) dpg_dr = -adv;
                const float dlogp = dpg_dr * ratio * inv_n;
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
#pragma unroll
                for (int j = 0; j < NACT; j++)
                    if ((bits >> j) & 1u)
                        dl[j] = dlogp * ((j == act ? 1.f : 0.f) - p[j]) + a.ent_coef * inv_n * p[j] * (lp[j] + ent);
                dl[NACT] = a.vf_coef * dvf * inv_n;
                t_pg = pg;
                t_vf = vf;
                t_ent = ent;
                t_clip = fabsf(ratio - 1.f) > a.clip ? 1.f : 0.f;
                t_kl = olp - la;
            }
            // dhead as bf16 hi + lo: dh2's A [part][j/8][row][8 j] and dWh^T's B [r/8][part*16 + j][8 r]
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                const __nv_bfloat162 h = __floats2bfloat162_rn(dl[j], dl[j + 1]);
                const float2 hf = __bfloat1622float2(h);
                const __nv_bfloat162 r = __floats2bfloat162_rn(dl[j] - hf.x, dl[j + 1] - hf.y);
                hi[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
                lo[j / 2] = *reinterpret_cast<const uint32_t *>(&r);
            }
#pragma unroll
            for (int h = 0; h < 2; h++) {
                *reinterpret_cast<uint4 *>(sm + OFF_HB + h * 2048 + row * 16) =
                    make_uint4(hi[4 * h], hi[4 * h + 1], hi[4 * h + 2], hi[4 * h + 3]);
                *reinterpret_cast<uint4 *>(sm + OFF_HB + 4096 + h * 2048 + row * 16) =
                    make_uint4(lo[4 * h], lo[4 * h + 1], lo[4 * h + 2], lo[4 * h + 3]);
            }
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const uint32_t sh = (j & 1) * 16;
                uint16_t *dst = reinterpret_cast<uint16_t *>(sm + OFF_DB + (row >> 3) * 512 + j * 16 + (row & 7) * 2);
                dst[0] = (uint16_t)(hi[j / 2] >> sh);
                dst[128] = (uint16_t)(lo[j / 2] >> sh);  // part 1: 16 rows (256 B) further
            }
            // this warp's dbh sums and loss terms (lane order, fixed)
#pragma unroll
            for (int j = 0; j < NOUT; j++) {
                float s = dl[j];
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0) red_bh[(warp - 2) * 16 + j] = s;
            }
            float tt[5] = {t_pg, t_vf, t_ent, t_clip, t_kl};
#pragma unroll
            for (int k = 0; k < 5; k++) {
                for (int o = 16; o > 0; o >>= 1) tt[k] += __shfl_xor_sync(0xffffffffu, tt[k], o);
                if (lane == 0) red_terms[(warp - 2) * 8 + k] = tt[k];
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_epi);

        // ---- step 3: dWh^T partial, dh2 = relu'(h2) * acc as bf16 into the tile
        float *out = a.part + (size_t)blockIdx.x * PART;
        ok = ok && mbar_wait(bar_mma, 0, WAIT_LIMIT) && !*abort_s;
        if (ok) {
            tc_fence_after();
            {
                uint32_t v[32];
                D1X_TMEM_LD32(tmem + lanes + D_DWH + 32 * (uint32_t)half, v);
                tmem_wait_ld();
                const int c = half * 128 + q * 32 + lane;
#pragma unroll
                for (int j = 0; j < NOUT; j++) out[j * HID + c] = __uint_as_float(v[j]) + __uint_as_float(v[16 + j]);
            }
#pragma unroll 1
            for (int cc = 0; cc < 4; cc++) {
                const int c0 = half * 128 + cc * 32;
                uint32_t v[32];
                D1X_TMEM_LD32(tmem + lanes + D_MAIN + (uint32_t)c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    uint4 *cell = reinterpret_cast<uint4 *>(sm + x_off(row, c0 + 8 * u));
                    const uint4 hv = *cell;
                    const __nv_bfloat16 *h = reinterpret_cast<const __nv_bfloat16 *>(&hv);
                    float f[8];
#pragma unroll
                    for (int i = 0; i < 8; i++)
                        f[i] = __bfloat162float(h[i]) > 0.f ? __uint_as_float(v[8 * u + i]) : 0.f;
                    *cell = make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                }
            }
        }
        fence_proxy_async();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_epi);
        // dh2 leaves by TMA stores from the tile; db2 (column sums of the stored
        // dh2), dbh and the loss terms meanwhile
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
        if (ok && te == 0) {
            for (int kb = 0; kb < 4; kb++) tma_store_2d(&map_dh2, base + OFF_X + kb * 16384, kb * 64, r0);
            bulk_commit();
        }
        if (ok) {
            float s = 0.f;
            for (int r = 0; r < ROWS; r++)
                s += __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(sm + x_off(r, te)));
            out[NOUT * HID + NOUT + te] = s;
            if (te < NOUT) {
                // warps 2-5 hold the loss rows: add their sums in warp order
                float b = 0.f;
                for (int w = 0; w < 4; w++) b += red_bh[w * 16 + te];
                out[NOUT * HID + te] = b;
            }
            if (te < 8) {
                float t = 0.f;
                if (te < 5)
                    for (int w = 0; w < 4; w++) t += red_terms[w * 8 + te];
                out[NOUT * HID + NOUT + HID + te] = t;
            }
        }

        // ---- step 4: dh1 = relu'(h1) * acc as bf16 into the tile (once the db2
        // sums and the dh2 stores are done reading it), then TMA stores
        ok = ok && mbar_wait(bar_mma, 1, WAIT_LIMIT) && !*abort_s;
        if (te == 0) bulk_wait_read();
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
        if (ok) {
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < 4; cc++) {
                const int c0 = half * 128 + cc * 32;
                uint32_t v[32];
                D1X_TMEM_LD32(tmem + lanes + D_MAIN + (uint32_t)c0, v);
                tmem_wait_ld();
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    float f[8];
#pragma unroll
                    for (int i = 0; i < 8; i++) f[i] = ((h1m[cc] >> (8 * u + i)) & 1u) ? __uint_as_float(v[8 * u + i]) : 0.f;
                    *reinterpret_cast<uint4 *>(sm + x_off(row, c0 + 8 * u)) =
                        make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
                }
            }
        }
        fence_proxy_async();
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
        if (te == 0) {
            if (ok) {
                for (int kb = 0; kb < 4; kb++) tma_store_2d(&map_dh1, base + OFF_X + kb * 16384, kb * 64, r0);
                bulk_commit();
            }
            bulk_wait_read();  // the tile may be released; the writes complete with the grid
        }
        if (!ok) {
            atomicExch(&g_tail_error, 6);
            *abort_s = 1;
        }
    }
    // ---- teardown: every TMA write has landed and TMEM is freed
    if (warp == 0 && lane == 0)
        for (int kb = 0; kb < 4; kb++) mbar_wait(bar_load + 8 * kb, 0, WAIT_LIMIT);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_ALLOC) : "memory");
    }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static bool map_bf16(CUtensorMap *m, const void *ptr, int rows, int cols, int box_rows) {
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
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64u, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tail
}  // namespace d1

extern "C" {

int d1_ppo_tail(const void *h1, const void *w2, const float *b2, const void *wh, const float *bh, const int64_t *idx,
                const uint16_t *legal, const int64_t *action, const float *old_logp, const float *adv,
                const float *ret, const float *old_value, const double *adv_stats, double adv_count, int n,
                float clip, float vclip, float vf_coef, float ent_coef, void *dh2, void *dh1, float *part,
                void *stream) {
    using namespace d1::tail;
    if (!h1 || !w2 || !b2 || !wh || !bh || !idx || !legal || !action || !old_logp || !adv || !ret || !old_value ||
        !adv_stats || !dh2 || !dh1 || !part || n <= 0 || adv_count < 2.0)
        return D1_ERR_BAD_ARGUMENT;
    if (((uintptr_t)h1 | (uintptr_t)w2 | (uintptr_t)dh2 | (uintptr_t)dh1) & 15) return D1_ERR_BAD_ARGUMENT;
    CUtensorMap mh, mw, md2, md1;
    if (!map_bf16(&mh, h1, n, HID, ROWS) || !map_bf16(&mw, w2, HID, HID, HID) || !map_bf16(&md2, dh2, n, HID, ROWS) ||
        !map_bf16(&md1, dh1, n, HID, ROWS))
        return D1_ERR_BAD_ARGUMENT;
    static uint64_t ready = 0;
    int dev = 0;
    if (cudaError_t e = cudaGetDevice(&dev)) return (int)e;
    if (dev >= 64 || !((ready >> dev) & 1)) {
        cudaError_t e = cudaFuncSetAttribute(tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return (int)e;
        if (dev < 64) ready |= 1ull << dev;
    }
    Args a{(const __nv_bfloat16 *)wh, b2, bh, idx, legal, action, old_logp, adv, ret, old_value, adv_stats,
           adv_count, n, clip, vclip, vf_coef, ent_coef, part};
    cudaLaunchAttribute attr;
    const cudaLaunchConfig_t cfg = d1::pdl_config(dim3((n + ROWS - 1) / ROWS), dim3(THREADS), SMEM,
                                                  (cudaStream_t)stream, &attr);
    return (int)cudaLaunchKernelEx(&cfg, tail_kernel, mh, mw, md2, md1, a);
}

int d1_ppo_tail_blocks(int n) { return n <= 0 ? 0 : (n + d1::tail::ROWS - 1) / d1::tail::ROWS; }

int d1_ppo_tail_error(void) {
    int h = 0, z = 0;
    if (cudaMemcpyFromSymbol(&h, d1::tail::g_tail_error, sizeof(int)) != cudaSuccess) return -1;
    if (h) cudaMemcpyToSymbol(d1::tail::g_tail_error, &z, sizeof(int));
    return h;
}

}  // extern "C"
