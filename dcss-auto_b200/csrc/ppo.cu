// Rollout-side and update-side kernels of PPO (sm_100a): GAE, minibatch
// gather, fused head/loss/backward-to-hidden, split-K reduction with bias
// column sums, gradient norm and Adam. The tensor-core GEMMs in between are
// d1_gemm (gemm_tc.cu).
//
// Reference update: gpu-d1/scripts/run_ring_ablations.py:354-372.
#include <cuda_bf16.h>
#include <stdint.h>

#include "d1_common.cuh"

namespace d1 {
namespace ppo {

// ------------------------------------------------------------------ GAE
// A_t = delta_t + gamma*lambda*(1 - done_t) * A_{t+1},
// delta_t = r_t + gamma * V_{t+1} * (1 - done_t) - V_t, returns = A + V.
// rewards/dones are read with element strides (they live in the env's
// outcome rows: reward at out[t, b, 0], done at out[t, b, 1]).
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
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(FULL, s1, o);
            s2 += __shfl_xor_sync(FULL, s2, o);
        }
        if ((threadIdx.x & 31) == 0) {
            atomicAdd(a.stats, s1);
            atomicAdd(a.stats + 1, s2);
        }
    }
}

// Warp-level segmented scan over time: the recurrence is an affine map
// A_t = d_t + c_t * A_{t+1}; maps compose associatively,
// (d1, c1) o (d2, c2) = (d1 + c1*d2, c1*c2), so each lane reduces its run of
// consecutive steps and the warp combines the runs with a reverse shuffle scan.
// A block stages 32 envs x T steps in shared memory with coalesced loads; warp
// w then scans envs w, w+8, ... Rounding differs from the sequential order
// (tolerance 1e-5 relative).
constexpr int SCAN_ENVS = 32, SCAN_WARPS = 8;
__global__ void __launch_bounds__(SCAN_WARPS * 32) gae_scan_kernel(GaeArgs a) {
    extern __shared__ float sh[];
    float *sd = sh;                            // delta   [T][32]
    float *sc = sd + a.T * SCAN_ENVS;          // c       [T][32]
    float *sv = sc + a.T * SCAN_ENVS;          // value   [T][32]
    const int e0 = blockIdx.x * SCAN_ENVS;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // stage: thread (t-row, env lane) loads reward/done/value and forms delta, c
    for (int t = warp; t < a.T; t += SCAN_WARPS) {
        const int b = e0 + lane;
        float d = 0.f, c = 0.f, v = 0.f;
        if (b < a.B) {
            const size_t o = (size_t)t * a.r_step + (size_t)b * a.r_env;
            const float live = 1.f - a.done[o];
            v = a.value[(size_t)t * a.B + b];
            const float nv = a.value[(size_t)(t + 1) * a.B + b];
            d = a.reward[o] + a.gamma * nv * live - v;
            c = a.gamma_lambda * live;
        }
        sd[t * SCAN_ENVS + lane] = d;
        sc[t * SCAN_ENVS + lane] = c;
        sv[t * SCAN_ENVS + lane] = v;
    }
    __syncthreads();
    const int per = (a.T + 31) / 32;  // consecutive steps per lane
    for (int env = warp; env < SCAN_ENVS; env += SCAN_WARPS) {
        // lane l owns steps [l*per, l*per + per); compose its run back to front
        const int t0 = lane * per, t1 = min(a.T, t0 + per);
        float D = 0.f, Cc = 1.f;  // identity map
        for (int t = t1 - 1; t >= t0; t--) {
            const float d = sd[t * SCAN_ENVS + env], c = sc[t * SCAN_ENVS + env];
            D = d + c * D;
            Cc = c * Cc;
        }
        // inclusive suffix scan: after it, (sD, sC) composes the runs of lanes [lane, 31]
        float sD = D, sC = Cc;
        for (int o = 1; o < 32; o <<= 1) {
            const float oD = __shfl_down_sync(FULL, sD, o), oC = __shfl_down_sync(FULL, sC, o);
            if (lane + o < 32) {
                // runs to the right are applied first: this(o) = this o right
                sD = sD + sC * oD;
                sC = sC * oC;
            }
        }
        // the value entering this lane's run is lanes [lane+1, 31] applied to A_T = 0
        float A = __shfl_down_sync(FULL, sD, 1);
        if (lane == 31) A = 0.f;
        for (int t = t1 - 1; t >= t0; t--) {
            A = sd[t * SCAN_ENVS + env] + sc[t * SCAN_ENVS + env] * A;
            sd[t * SCAN_ENVS + env] = A;
        }
    }
    __syncthreads();
    double s1 = 0.0, s2 = 0.0;
    for (int t = warp; t < a.T; t += SCAN_WARPS) {
        const int b = e0 + lane;
        if (b < a.B) {
            const float A = sd[t * SCAN_ENVS + lane];
            a.adv[(size_t)t * a.B + b] = A;
            a.ret[(size_t)t * a.B + b] = A + sv[t * SCAN_ENVS + lane];
            s1 += A;
            s2 += (double)A * A;
        }
    }
    if (a.stats) {
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(FULL, s1, o);
            s2 += __shfl_xor_sync(FULL, s2, o);
        }
        if (lane == 0) {
            atomicAdd(a.stats, s1);
            atomicAdd(a.stats + 1, s2);
        }
    }
}


// ------------------------------------------------------------------ minibatch gather
// X[i] = obs[idx[i]] (bf16 rows of F features) and X^T (feature-major, the
// B operand of the first-layer weight-gradient GEMM). A block moves 32 samples
// x 64 features per pass through a shared-memory tile so both writes coalesce.
constexpr int G_SAMPLES = 32, G_FEAT = 64;
__global__ void __launch_bounds__(256) gather_kernel(const __nv_bfloat16 *__restrict__ obs, int F,
                                                     const int64_t *__restrict__ idx, int n, __nv_bfloat16 *x,
                                                     __nv_bfloat16 *xt, int ldt) {
    __shared__ __align__(16) __nv_bfloat16 tile[G_SAMPLES][G_FEAT + 8];
    const int s0 = blockIdx.x * G_SAMPLES;
    const int t = threadIdx.x;
    const int ls = t / 8, part = t % 8;  // load: sample, 8-feature part
    const int gs = s0 + ls;
    const int64_t src = gs < n ? idx[gs] : 0;
    for (int f0 = 0; f0 < F; f0 += G_FEAT) {
        const int f = f0 + part * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (gs < n && f < F) {
            v = *reinterpret_cast<const uint4 *>(obs + (size_t)src * F + f);
            if (x) *reinterpret_cast<uint4 *>(x + (size_t)gs * F + f) = v;
        }
        *reinterpret_cast<uint4 *>(&tile[ls][part * 8]) = v;
        __syncthreads();
        if (xt) {
            const int feat = t / 4, q = t % 4;  // store: feature, 8-sample part
            const int ff = f0 + feat;
            if (ff < F && s0 + q * 8 < n) {
                __align__(16) __nv_bfloat16 o[8];
#pragma unroll
                for (int i = 0; i < 8; i++) o[i] = tile[q * 8 + i][feat];
                if (s0 + q * 8 + 8 <= n) {
                    *reinterpret_cast<uint4 *>(xt + (size_t)ff * ldt + s0 + q * 8) = *reinterpret_cast<uint4 *>(o);
                } else {
                    for (int i = 0; i < 8 && s0 + q * 8 + i < n; i++) xt[(size_t)ff * ldt + s0 + q * 8 + i] = o[i];
                }
            }
        }
        __syncthreads();
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
constexpr int L_ROWS = 32, L_HID = 256, L_NOUT = 13, L_NACT = 12;
constexpr int L_PART = L_NOUT * L_HID + L_NOUT + L_HID + 8;

struct LossSmem {
    float w_s[L_NOUT][L_HID];
    float hs[L_ROWS][L_HID + 4];  // h2 rows (fp32)
    float gs[L_ROWS][L_HID + 4];  // dh2 rows (fp32, masked)
    float dh_s[L_ROWS][L_NOUT];
    float terms_s[8][8];
};
__global__ void __launch_bounds__(256) loss_kernel(LossArgs a) {
    extern __shared__ __align__(16) uint8_t loss_raw[];
    LossSmem &S = *reinterpret_cast<LossSmem *>(loss_raw);
    auto &w_s = S.w_s;
    auto &hs = S.hs;
    auto &gs = S.gs;
    auto &dh_s = S.dh_s;
    auto &terms_s = S.terms_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < L_NOUT * L_HID; i += 256) w_s[i / L_HID][i % L_HID] = __bfloat162float(a.wh[i]);
    const double mean = a.adv_stats[0] / a.adv_count;
    const double var = (a.adv_stats[1] - a.adv_stats[0] * mean) / (a.adv_count - 1.0);
    const float amean = (float)mean, astd = (float)sqrt(var > 0 ? var : 0.0);
    const float inv_n = 1.f / (float)a.n;
    float acc_w[L_NOUT] = {0};  // this thread's dWh column (k = tid), summed over rows
    float acc_b2 = 0.f, acc_bh = 0.f;
    float t_pg = 0.f, t_vf = 0.f, t_ent = 0.f, t_clip = 0.f, t_kl = 0.f;
    __syncthreads();
    const int nb = (a.n + L_ROWS - 1) / L_ROWS;
    for (int blk = blockIdx.x; blk < nb; blk += gridDim.x) {
        const int r0 = blk * L_ROWS;
        // stage h2 rows as fp32
        for (int i = tid; i < L_ROWS * (L_HID / 8); i += 256) {
            const int r = i / (L_HID / 8), c = (i % (L_HID / 8)) * 8;
            float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            if (r0 + r < a.n) {
                const uint4 raw = *reinterpret_cast<const uint4 *>(a.h2 + (size_t)(r0 + r) * L_HID + c);
                const __nv_bfloat162 *p2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float2 ff = __bfloat1622float2(p2[j]);
                    f[2 * j] = ff.x;
                    f[2 * j + 1] = ff.y;
                }
            }
#pragma unroll
            for (int j = 0; j < 8; j++) hs[r][c + j] = f[j];
        }
        __syncthreads();
        // warp w handles rows w, w+8, w+16, w+24: each lane sums 8 of 256 elements
        for (int rr = warp; rr < L_ROWS; rr += 8) {
            const int row = r0 + rr;
            float acc[L_NOUT];
#pragma unroll
            for (int j = 0; j < L_NOUT; j++) {
                float sum = 0.f;
#pragma unroll
                for (int i = 0; i < 8; i++) sum += hs[rr][lane + 32 * i] * w_s[j][lane + 32 * i];
                acc[j] = sum;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int j = 0; j < L_NOUT; j++) acc[j] += __shfl_xor_sync(FULL, acc[j], o);
            float dl[L_NACT], dv = 0.f;
#pragma unroll
            for (int j = 0; j < L_NACT; j++) dl[j] = 0.f;
            if (row < a.n && lane == 0) {
                const int64_t sidx = a.idx[row];
                const uint32_t bits = a.legal[sidx];
                const int act = (int)a.action[sidx];
                float l[L_NACT], m = -3.402823466e38f;
#pragma unroll
                for (int j = 0; j < L_NACT; j++) {
                    l[j] = acc[j] + a.bh[j];
                    if ((bits >> j) & 1u) m = fmaxf(m, l[j]);
                }
                float z = 0.f;
#pragma unroll
                for (int j = 0; j < L_NACT; j++)
                    if ((bits >> j) & 1u) z += expf(l[j] - m);
                const float lz = logf(z);
                float p[L_NACT], ent = 0.f, la = 0.f;
#pragma unroll
                for (int j = 0; j < L_NACT; j++) {
                    const bool ok = (bits >> j) & 1u;
                    const float lp = l[j] - m - lz;
                    p[j] = ok ? expf(lp) : 0.f;
                    if (ok) ent -= p[j] * lp;
                    if (j == act) la = lp;
                }
                const float value = acc[L_NACT] + a.bh[L_NACT];
                const float adv = (a.adv[sidx] - amean) / (astd + 1e-8f);
                const float ratio = expf(la - a.old_logp[sidx]);
                const float s1 = ratio * adv, rc = fminf(fmaxf(ratio, 1.f - a.clip), 1.f + a.clip), s2 = rc * adv;
                const float pg = -fminf(s1, s2);
                // d pg / d logp(a): only the selected branch carries gradient
                // (the clamped branch is flat outside [1-clip, 1+clip])
                float dpg_dr = 0.f;
                if (s1 <= s2) dpg_dr = -adv;
                else if (ratio > 1.f - a.clip && ratio < 1.f + a.clip) dpg_dr = -adv;
                const float dlogp = dpg_dr * ratio * inv_n;
                // value term
                const float R = a.ret[sidx], vold = a.old_value[sidx];
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
                dv = a.vf_coef * dvf * inv_n;
                // d(-ent_coef * H)/dl_j = ent_coef * p_j * (log p_j + H)
#pragma unroll
                for (int j = 0; j < L_NACT; j++) {
                    if (!((bits >> j) & 1u)) continue;
                    const float lp = l[j] - m - lz;
                    float g = dlogp * ((j == act ? 1.f : 0.f) - p[j]);
                    g += a.ent_coef * inv_n * p[j] * (lp + ent);
                    dl[j] = g;
                }
                t_pg += pg;
                t_vf += vf;
                t_ent += ent;
                t_clip += fabsf(ratio - 1.f) > a.clip ? 1.f : 0.f;
                t_kl += a.old_logp[sidx] - la;
            }
#pragma unroll
            for (int j = 0; j < L_NACT; j++) dl[j] = __shfl_sync(FULL, dl[j], 0);
            dv = __shfl_sync(FULL, dv, 0);
            if (lane < L_NOUT) {
                float mine = dv;
#pragma unroll
                for (int j = 0; j < L_NACT; j++)
                    if (lane == j) mine = dl[j];
                dh_s[rr][lane] = row < a.n ? mine : 0.f;
            }
            // dh2 = dhead . Wh, masked by ReLU'(h2)
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int k = lane + 32 * i;
                float g = dv * w_s[L_NACT][k];
#pragma unroll
                for (int j = 0; j < L_NACT; j++) g += dl[j] * w_s[j][k];
                gs[rr][k] = (row < a.n && hs[rr][k] > 0.f) ? g : 0.f;
            }
        }
        __syncthreads();
        // partial dWh[j][k] += sum_r dhead[r][j] * h2[r][k]; db2[k] += sum_r dh2[r][k]; dbh
        {
            const int k = tid;
            float b2 = 0.f;
#pragma unroll 4
            for (int r = 0; r < L_ROWS; r++) {
                const float h = hs[r][k];
#pragma unroll
                for (int j = 0; j < L_NOUT; j++) acc_w[j] += dh_s[r][j] * h;
                b2 += gs[r][k];
            }
            acc_b2 += b2;
            if (tid < L_NOUT)
                for (int r = 0; r < L_ROWS; r++) acc_bh += dh_s[r][tid];
        }
        // dh2 row-major (coalesced: a row is 512 B) and transposed (a feature row of
        // 32 consecutive samples is 64 B)
        for (int i = tid; i < L_ROWS * (L_HID / 8); i += 256) {
            const int r = i / (L_HID / 8), c = (i % (L_HID / 8)) * 8;
            if (r0 + r < a.n && a.dh2) {
                __align__(16) __nv_bfloat16 o[8];
#pragma unroll
                for (int j = 0; j < 8; j++) o[j] = __float2bfloat16_rn(gs[r][c + j]);
                *reinterpret_cast<uint4 *>(a.dh2 + (size_t)(r0 + r) * L_HID + c) = *reinterpret_cast<uint4 *>(o);
            }
        }
        if (a.dh2t) {
            for (int i = tid; i < L_HID * (L_ROWS / 8); i += 256) {
                const int k = i / (L_ROWS / 8), q = (i % (L_ROWS / 8)) * 8;
                if (r0 + q < a.n) {
                    __align__(16) __nv_bfloat16 o[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) o[j] = __float2bfloat16_rn(gs[q + j][k]);
                    if (r0 + q + 8 <= a.n)
                        *reinterpret_cast<uint4 *>(a.dh2t + (size_t)k * a.ldt + r0 + q) = *reinterpret_cast<uint4 *>(o);
                    else
                        for (int j = 0; j < 8 && r0 + q + j < a.n; j++) a.dh2t[(size_t)k * a.ldt + r0 + q + j] = o[j];
                }
            }
        }
        __syncthreads();
    }
    // block partials
    float *out = a.part + (size_t)blockIdx.x * L_PART;
#pragma unroll
    for (int j = 0; j < L_NOUT; j++) out[j * L_HID + tid] = acc_w[j];
    if (tid < L_NOUT) out[L_NOUT * L_HID + tid] = acc_bh;
    out[L_NOUT * L_HID + L_NOUT + tid] = acc_b2;
    // loss terms: reduce the lane-0 values of every warp
    if (lane == 0) {
        terms_s[warp][0] = t_pg;
        terms_s[warp][1] = t_vf;
        terms_s[warp][2] = t_ent;
        terms_s[warp][3] = t_clip;
        terms_s[warp][4] = t_kl;
    }
    __syncthreads();
    if (tid < 5) {
        float v = 0.f;
        for (int w = 0; w < 8; w++) v += terms_s[w][tid];
        out[L_NOUT * L_HID + L_NOUT + L_HID + tid] = v;
    }
    if (tid >= 5 && tid < 8) out[L_NOUT * L_HID + L_NOUT + L_HID + tid] = 0.f;
}

// out[i] = sum over p of parts[p * stride + i] (loss-kernel block partials).
__global__ void sum_rows_kernel(const float *parts, int nparts, int stride, int len, float *out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= len) return;
    float s = 0.f;
    for (int p = 0; p < nparts; p++) s += parts[(size_t)p * stride + i];
    out[i] = s;
}

// out[i] = sum over splits of slabs[s][i] (split-K partial products), i < count.
__global__ void reduce_slabs_kernel(const float *__restrict__ slabs, int splits, int64_t count, float *out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    float s = 0.f;
    for (int k = 0; k < splits; k++) s += slabs[(size_t)k * count + i];
    out[i] = s;
}

// out[r] = sum of row r of a bf16 [rows, cols] matrix (pitch ld); one warp per row.
__global__ void row_sum_bf16_kernel(const __nv_bfloat16 *__restrict__ m, int rows, int cols, int ld, float *out) {
    const int r = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    float s = 0.f;
    for (int c = lane * 8; c < cols; c += 256) {
        if (c + 8 <= cols) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(m + (size_t)r * ld + c);
            const __nv_bfloat162 *p2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float2 f = __bfloat1622float2(p2[j]);
                s += f.x + f.y;
            }
        } else {
            for (int j = c; j < cols; j++) s += __bfloat162float(m[(size_t)r * ld + j]);
        }
    }
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
    if (lane == 0) out[r] = s;
}

// ------------------------------------------------------------------ optimizer
// sum of squares of g[0..n) into *out (double, accumulated)
__global__ void sumsq_kernel(const float *__restrict__ g, int64_t n, double *out) {
    double s = 0.0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        s += (double)g[i] * g[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
    __shared__ double ws[32];
    if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < blockDim.x / 32 ? ws[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(FULL, s, o);
        if (threadIdx.x == 0) atomicAdd(out, s);
    }
}

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
    const double *sumsq;
    const int64_t *step;  // device counter: the step being taken (1-based)
    float lr, beta1, beta2, eps, max_norm;
    AdamSeg seg[8];
    int nseg;
    int64_t total;
};
__global__ void adam_kernel(AdamArgs a) {
    const double norm = sqrt(*a.sumsq);
    const double t = (double)*a.step;
    const float bc1 = (float)(1.0 - pow((double)a.beta1, t));
    const float bc2_sqrt = (float)sqrt(1.0 - pow((double)a.beta2, t));
    float scale = 1.f;
    if (a.max_norm > 0.f) {
        const float coef = a.max_norm / ((float)norm + 1e-6f);
        if (coef < 1.f) scale = coef;
    }
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float g = a.grad[i] * scale;
        const float m = a.beta1 * a.m[i] + (1.f - a.beta1) * g;
        const float v = a.beta2 * a.v[i] + (1.f - a.beta2) * g * g;
        a.m[i] = m;
        a.v[i] = v;
        const float denom = sqrtf(v) / bc2_sqrt + a.eps;
        const float p = a.param[i] - (a.lr / bc1) * m / denom;
        a.param[i] = p;
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
}

__global__ void counter_add_kernel(int64_t *c, int64_t delta) { *c += delta; }

}  // namespace ppo
}  // namespace d1

using namespace d1;


extern "C" {

int d1_ppo_gather(const void *obs, int F, const int64_t *idx, int n, void *x, void *xt, int ldt, void *stream) {
    if (!obs || !idx || n <= 0 || F <= 0 || F % 8 || (xt && (ldt < n || ldt % 8))) return D1_ERR_BAD_ARGUMENT;
    ppo::gather_kernel<<<(n + ppo::G_SAMPLES - 1) / ppo::G_SAMPLES, 256, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16 *)obs, F, idx, n, (__nv_bfloat16 *)x, (__nv_bfloat16 *)xt, ldt);
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
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(ppo::loss_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)sizeof(ppo::LossSmem));
        if (e != cudaSuccess) return (int)e;
        attr = true;
    }
    ppo::LossArgs a{(const __nv_bfloat16 *)h2, (const __nv_bfloat16 *)wh, bh, idx, legal, action, old_logp, adv,
                    ret, old_value, adv_stats, adv_count, n, clip, vclip, vf_coef, ent_coef,
                    (__nv_bfloat16 *)dh2, (__nv_bfloat16 *)dh2t, ldt, part};
    ppo::loss_kernel<<<blocks, 256, sizeof(ppo::LossSmem), (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}

int d1_sum_rows(const float *parts, int nparts, int stride, int len, float *out, void *stream) {
    if (!parts || !out || nparts <= 0 || len <= 0 || stride < len) return D1_ERR_BAD_ARGUMENT;
    ppo::sum_rows_kernel<<<(len + 255) / 256, 256, 0, (cudaStream_t)stream>>>(parts, nparts, stride, len, out);
    return (int)cudaGetLastError();
}

int d1_reduce_slabs(const float *slabs, int splits, int64_t count, float *out, void *stream) {
    if (!slabs || !out || splits <= 0 || count <= 0) return D1_ERR_BAD_ARGUMENT;
    ppo::reduce_slabs_kernel<<<(unsigned)((count + 255) / 256), 256, 0, (cudaStream_t)stream>>>(slabs, splits, count,
                                                                                                 out);
    return (int)cudaGetLastError();
}

int d1_row_sum_bf16(const void *m, int rows, int cols, int ld, float *out, void *stream) {
    if (!m || !out || rows <= 0 || cols <= 0 || ld < cols || ld % 8) return D1_ERR_BAD_ARGUMENT;
    ppo::row_sum_bf16_kernel<<<(rows + 7) / 8, 256, 0, (cudaStream_t)stream>>>((const __nv_bfloat16 *)m, rows, cols,
                                                                                 ld, out);
    return (int)cudaGetLastError();
}

int d1_sumsq(const float *g, int64_t n, double *out, void *stream) {
    if (!g || !out || n <= 0) return D1_ERR_BAD_ARGUMENT;
    ppo::sumsq_kernel<<<296, 256, 0, (cudaStream_t)stream>>>(g, n, out);
    return (int)cudaGetLastError();
}

int d1_counter_add(int64_t *counter, int64_t delta, void *stream) {
    if (!counter) return D1_ERR_BAD_ARGUMENT;
    ppo::counter_add_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(counter, delta);
    return (int)cudaGetLastError();
}

int d1_adam(float *param, float *grad, float *m, float *v, const double *sumsq, int64_t total, float lr, float beta1,
            float beta2, float eps, float max_norm, const int64_t *step, const D1AdamSegment *segs, int nseg,
            void *stream) {
    if (!param || !grad || !m || !v || !sumsq || !step || total <= 0 || nseg < 0 || nseg > 8)
        return D1_ERR_BAD_ARGUMENT;
    ppo::AdamArgs a;
    a.param = param;
    a.grad = grad;
    a.m = m;
    a.v = v;
    a.sumsq = sumsq;
    a.lr = lr;
    a.beta1 = beta1;
    a.beta2 = beta2;
    a.eps = eps;
    a.max_norm = max_norm;
    a.step = step;
    a.nseg = nseg;
    a.total = total;
    for (int i = 0; i < nseg; i++) {
        a.seg[i].offset = segs[i].offset;
        a.seg[i].count = segs[i].count;
        a.seg[i].rows = segs[i].rows;
        a.seg[i].cols = segs[i].cols;
        a.seg[i].bf16 = (__nv_bfloat16 *)segs[i].bf16;
        a.seg[i].bf16_t = (__nv_bfloat16 *)segs[i].bf16_t;
    }
    ppo::adam_kernel<<<592, 256, 0, (cudaStream_t)stream>>>(a);
    return (int)cudaGetLastError();
}

int d1_gae(const float *reward, const float *done, int64_t r_step, int64_t r_env, const float *value, int T, int B,
           float gamma, float lambda, float *adv, float *ret, double *stats, int mode, void *stream) {
    if (T <= 0 || B <= 0 || !reward || !done || !value || !adv || !ret) return D1_ERR_BAD_ARGUMENT;
    ppo::GaeArgs a{reward, done, value, r_step, r_env, adv, ret, stats, T, B, gamma, (float)((double)gamma * lambda)};
    if (mode == 0) {
        ppo::gae_sequential_kernel<<<(B + 255) / 256, 256, 0, (cudaStream_t)stream>>>(a);
    } else {
        const size_t sm = (size_t)3 * T * ppo::SCAN_ENVS * sizeof(float);
        if (sm > 200 * 1024) return D1_ERR_BAD_ARGUMENT;
        if (sm > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(ppo::gae_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)sm);
            if (e != cudaSuccess) return (int)e;
        }
        ppo::gae_scan_kernel<<<(B + ppo::SCAN_ENVS - 1) / ppo::SCAN_ENVS, ppo::SCAN_WARPS * 32, sm,
                               (cudaStream_t)stream>>>(a);
    }
    return (int)cudaGetLastError();
}

}  // extern "C"
