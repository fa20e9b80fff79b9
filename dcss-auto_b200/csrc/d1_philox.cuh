// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
// as 1, 2, 3", SC'11) for the policy-side draws. Stream layout of every sampler:
// Philox(ctr = {lo(step), hi(step), hi(seed), purpose}, key = {env id, lo(seed)})
// with purpose 1 = flat categorical, 2 = autoregressive verb/target,
// 3 = uniform over the legal actions.
#pragma once
#include <stdint.h>

namespace d1 {

__device__ __forceinline__ uint4 philox4x32(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    }
    return c;
}

__device__ __forceinline__ uint4 policy_draw(uint32_t env, uint64_t seed, uint64_t step, uint32_t purpose) {
    return philox4x32(make_uint4((uint32_t)step, (uint32_t)(step >> 32), (uint32_t)(seed >> 32), purpose), env,
                      (uint32_t)seed);
}

}  // namespace d1
