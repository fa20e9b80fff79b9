// Evaluation-loop and observation-wrapper kernels around the env step:
//
//  * eval_accumulate: the bookkeeping of the reference's evaluation loop
//    (gpu-d1/scripts/train_clear.py:42-58, run_ring_ablations.py:231-246):
//    returns += active * reward; envs whose episode ends this step record their
//    outcome row and leave the active set.
//  * uniform_legal: the random baseline (train_clear.py:52-53 samples the action
//    mask uniformly): action = the k-th legal action, k = floor(u * count) with
//    u the 32-bit Philox word 0 of purpose 3, computed as mulhi(word, count) so a
//    CPU restatement reproduces it exactly.
//  * frame_stack: the fixed observation history of gpu-d1/branches/
//    vision15-centered-map-v1/scripts/frame_stack.py:5-32 -- frames shift one
//    slot older, the new observation is appended, and at an episode end (done,
//    and active when a mask is given) every slot is the new observation. One
//    thread owns one 4-byte column of an env across all frames, so the shift is
//    in place without a copy.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/d1.h"
#include "d1_philox.cuh"

namespace d1 {
namespace ev {

__global__ void accumulate_kernel(const float *__restrict__ out, int out_cols, int n, bool *__restrict__ active,
                                  float *__restrict__ returns, float *__restrict__ terminal, int tcols) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n || !active[i]) return;
    const float *o = out + (size_t)i * out_cols;
    returns[i] += o[0];
    if (o[1] > 0.f) {
        for (int c = 0; c < tcols; c++) terminal[(size_t)i * tcols + c] = o[c];
        active[i] = false;
    }
}

__global__ void uniform_legal_kernel(const uint16_t *__restrict__ legal, int nact, int n, uint64_t seed,
                                     uint64_t step, int first_env, int64_t *__restrict__ action) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t bits = (uint32_t)legal[i] & ((1u << nact) - 1u);
    const int count = __popc(bits);
    if (count == 0) {
        action[i] = -1;
        return;
    }
    const uint4 o = policy_draw((uint32_t)(first_env + i), seed, step, 3u);
    uint32_t k = __umulhi(o.x, (uint32_t)count);
    uint32_t b = bits;
    for (; k > 0; k--) b &= b - 1u;  // drop the k lowest set bits
    action[i] = __ffs(b) - 1;
}

__global__ void frame_stack_kernel(uint32_t *__restrict__ stack, const uint32_t *__restrict__ obs, int words,
                                   int frames, int n, const float *__restrict__ out, int out_cols,
                                   const bool *__restrict__ active) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)n * words) return;
    const int i = (int)(t / words), j = (int)(t - (int64_t)i * words);
    bool ended = out ? out[(size_t)i * out_cols + 1] > 0.f : false;
    if (active) ended = ended && active[i];
    uint32_t *row = stack + (size_t)i * frames * words + j;
    const uint32_t fresh = obs[(size_t)i * words + j];
    for (int f = 0; f + 1 < frames; f++) row[(size_t)f * words] = ended ? fresh : row[(size_t)(f + 1) * words];
    row[(size_t)(frames - 1) * words] = fresh;
}

__global__ void frame_fill_kernel(uint32_t *__restrict__ stack, const uint32_t *__restrict__ obs, int words,
                                  int frames, int n) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (int64_t)n * words) return;
    const int i = (int)(t / words), j = (int)(t - (int64_t)i * words);
    const uint32_t fresh = obs[(size_t)i * words + j];
    for (int f = 0; f < frames; f++) stack[((size_t)i * frames + f) * words + j] = fresh;
}

}  // namespace ev
}  // namespace d1

using namespace d1;

extern "C" {

int d1_eval_accumulate(const float *out, int out_cols, int n, bool *active, float *returns, float *terminal,
                       int tcols, void *stream) {
    if (n < 0 || !out || !active || !returns || !terminal || tcols < 2 || tcols > out_cols) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    ev::accumulate_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(out, out_cols, n, active, returns,
                                                                             terminal, tcols);
    return (int)cudaGetLastError();
}

int d1_sample_uniform_legal(const uint16_t *legal, int nact, int n, uint64_t seed, uint64_t step, int first_env,
                            int64_t *action, void *stream) {
    if (n < 0 || !legal || !action || nact < 1 || nact > 16) return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    ev::uniform_legal_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(legal, nact, n, seed, step,
                                                                                first_env, action);
    return (int)cudaGetLastError();
}

int d1_frame_stack(void *stack, const void *obs, int row_bytes, int frames, int n, const float *out, int out_cols,
                   const bool *active, void *stream) {
    if (n < 0 || !stack || !obs || frames < 2 || row_bytes <= 0 || row_bytes % 4 ||
        ((reinterpret_cast<uintptr_t>(stack) | reinterpret_cast<uintptr_t>(obs)) & 3))
        return D1_ERR_BAD_ARGUMENT;
    if (n == 0) return 0;
    const int words = row_bytes / 4;
    const int64_t total = (int64_t)n * words;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (out)
        ev::frame_stack_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(
            (uint32_t *)stack, (const uint32_t *)obs, words, frames, n, out, out_cols, active);
    else
        ev::frame_fill_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((uint32_t *)stack, (const uint32_t *)obs,
                                                                        words, frames, n);
    return (int)cudaGetLastError();
}

}  // extern "C"
