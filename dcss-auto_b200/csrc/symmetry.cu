// Per-episode D4 camera augmentation of the BASELINE task's observation, the
// EpisodeSymmetry wrapper of gpu-d1/branches/vision15-symmetry-v1/scripts/
// symmetry.py:19-102 restated for the spec observation (15 x 15 cells x 8
// one-hot channels, then 32 scalars at element 1800):
//
//  * group g in 0..7 acts on a world offset (x, y) as the reference's xy():
//    mirror x when g >= 4, then g % 4 quarter turns (x, y) -> (-y, x);
//  * camera cell (x', y') shows world cell g^-1 (x', y') (all 8 channels);
//  * the scalar coordinate pairs follow the reference's rule -- camera
//    component d takes the world component s whose axis maps onto d, times
//    sign * units[s] / units[d], plus (center[d] - sign * center[s]) / units[d],
//    constants formed in double and rounded to float as the reference's float32
//    tables hold them, applied as a separately rounded multiply and add. Pairs
//    (element 1800 + k): player position (4, 5) about the grid centre (39.5,
//    34.5) in units (80, 70); nearest monster (9, 10) in (7, 7); stairs (15, 16)
//    in (80, 70); ogre (26, 27) in (7, 7). Every other scalar is unchanged;
//  * directional actions and legal bits 0-7 (compass order N, E, S, W, NE, SE,
//    SW, NW) are permuted: camera direction c is world direction g^-1(c), so a
//    camera action maps to the world as to_world() does and camera legal bit c
//    is world bit g^-1(c); actions and bits 8-11 are unchanged;
//  * a fresh group is drawn at an episode end: Philox purpose 4, word 0 >> 29.
//
// d4_observe is one warp per env: the 3,664-byte row is staged in shared memory
// (so the transform may run in place), then every lane writes 16-byte cells.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/d1.h"
#include "d1_philox.cuh"

namespace d1 {
namespace d4 {

constexpr int OBS = 1832, CELLS = 225, SCALARS = 1800, VEC = OBS * 2 / 16, WARPS = 8;

__device__ __forceinline__ void apply(int g, int &x, int &y) {
    if (g >= 4) x = -x;
    for (int r = 0; r < (g & 3); r++) {
        const int t = x;
        x = -y;
        y = t;
    }
}
__device__ __forceinline__ void unapply(int g, int &x, int &y) {
    for (int r = 0; r < (g & 3); r++) {
        const int t = x;
        x = y;
        y = -t;
    }
    if (g >= 4) x = -x;
}
__device__ __forceinline__ int dir_index(int x, int y) {
    // N, E, S, W, NE, SE, SW, NW, none
    if (x == 0) return y < 0 ? 0 : y > 0 ? 2 : 8;
    if (y == 0) return x > 0 ? 1 : 3;
    if (y < 0) return x > 0 ? 4 : 7;
    return x > 0 ? 5 : 6;
}
__device__ __forceinline__ void dir_vec(int a, int &x, int &y) {
    const int dx[9] = {0, 1, 0, -1, 1, 1, -1, -1, 0}, dy[9] = {-1, 0, 1, 0, -1, 1, 1, -1, 0};
    x = dx[a];
    y = dy[a];
}
// World direction shown as camera direction c under g.
__device__ __forceinline__ int world_dir(int g, int c) {
    int x, y;
    dir_vec(c, x, y);
    unapply(g, x, y);
    return dir_index(x, y);
}

__global__ void __launch_bounds__(WARPS * 32) observe_kernel(const uint4 *__restrict__ obs, const uint16_t *legal,
                                                             const uint8_t *__restrict__ groups, int n, uint4 *out,
                                                             uint16_t *legal_out) {
    __shared__ uint4 rows[WARPS][VEC];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int env = blockIdx.x * WARPS + w;
    if (env >= n) return;
    const int g = groups[env] & 7;
    uint4 *row = rows[w];
    const uint4 *src = obs + (size_t)env * VEC;
    for (int i = lane; i < VEC; i += 32) row[i] = src[i];
    const uint16_t world_legal = legal[env];
    __syncwarp();
    uint4 *dst = out + (size_t)env * VEC;
    for (int j = lane; j < CELLS; j += 32) {
        int x = j % 15 - 7, y = j / 15 - 7;
        unapply(g, x, y);
        dst[j] = row[(y + 7) * 15 + x + 7];
    }
    // scalars: lane k owns element 1800 + k
    const __nv_bfloat16 *sc = reinterpret_cast<const __nv_bfloat16 *>(row) + SCALARS;
    int base = -1;
    double ux = 1, uy = 1, cx = 0, cy = 0;
    if (lane == 4 || lane == 5) base = 4, ux = 80, uy = 70, cx = 39.5, cy = 34.5;
    else if (lane == 9 || lane == 10) base = 9, ux = 7, uy = 7;
    else if (lane == 15 || lane == 16) base = 15, ux = 80, uy = 70;
    else if (lane == 26 || lane == 27) base = 26, ux = 7, uy = 7;
    __nv_bfloat16 v = sc[lane];
    if (base >= 0) {
        const int d = lane - base;
        int exx = 1, exy = 0, eyx = 0, eyy = 1;
        apply(g, exx, exy);
        apply(g, eyx, eyy);
        const int ed = d == 0 ? exx : exy, fd = d == 0 ? eyx : eyy;
        const int s = ed != 0 ? 0 : 1, sign = ed != 0 ? ed : fd;
        const double us = s == 0 ? ux : uy, ud = d == 0 ? ux : uy;
        const double cs = s == 0 ? cx : cy, cd = d == 0 ? cx : cy;
        const float scale = (float)((double)sign * us / ud);
        const float offset = (float)((cd - (double)sign * cs) / ud);
        v = __float2bfloat16_rn(__fadd_rn(__fmul_rn(__bfloat162float(sc[base + s]), scale), offset));
    }
    __syncwarp();  // every lane has read its scalar source before any lane writes it (in place)
    reinterpret_cast<__nv_bfloat16 *>(dst)[SCALARS + lane] = v;
    if (lane == 0) {
        uint32_t bits = world_legal & ~0xffu;
        for (int c = 0; c < 8; c++) bits |= ((world_legal >> world_dir(g, c)) & 1u) << c;
        legal_out[env] = (uint16_t)bits;
    }
}

__global__ void actions_kernel(const int64_t *__restrict__ cam, const uint8_t *__restrict__ groups, int n,
                               int64_t *__restrict__ world) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t a = cam[i];
    world[i] = (a >= 0 && a < 8) ? world_dir(groups[i] & 7, (int)a) : a;
}

__global__ void draw_kernel(uint8_t *__restrict__ groups, int n, const float *__restrict__ out, int out_cols,
                            const bool *__restrict__ active, uint64_t seed, uint64_t step, int first_env) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (out && !(out[(size_t)i * out_cols + 1] > 0.f && (!active || active[i]))) return;
    groups[i] = (uint8_t)(policy_draw((uint32_t)(first_env + i), seed, step, 4u).x >> 29);
}

}  // namespace d4
}  // namespace d1

extern "C" {

int d1_spec_d4_observe(const void *obs_bf16, const uint16_t *legal, const uint8_t *groups, int n, void *obs_out_bf16,
                       uint16_t *legal_out, void *stream) {
    using namespace d1::d4;
    if (n < 0 || !obs_bf16 || !legal || !groups || !obs_out_bf16 || !legal_out) return D1_ERR_BAD_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(obs_bf16) & 15) || (reinterpret_cast<uintptr_t>(obs_out_bf16) & 15))
        return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    observe_kernel<<<(n + WARPS - 1) / WARPS, WARPS * 32, 0, (cudaStream_t)stream>>>(
        (const uint4 *)obs_bf16, legal, groups, n, (uint4 *)obs_out_bf16, legal_out);
    return (int)cudaGetLastError();
}

int d1_spec_d4_actions(const int64_t *camera_actions, const uint8_t *groups, int n, int64_t *world_actions,
                       void *stream) {
    using namespace d1::d4;
    if (n < 0 || !camera_actions || !groups || !world_actions) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    actions_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(camera_actions, groups, n, world_actions);
    return (int)cudaGetLastError();
}

int d1_spec_d4_draw(uint8_t *groups, int n, const float *out, int out_cols, const bool *active, uint64_t seed,
                    uint64_t step, int first_env, void *stream) {
    using namespace d1::d4;
    if (n < 0 || !groups || (out && out_cols < 2)) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    draw_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(groups, n, out, out_cols, active, seed, step,
                                                                     first_env);
    return (int)cudaGetLastError();
}

}  // extern "C"
