// Portable float exp used wherever a result must be bit-identical between the
// CUDA kernels and the CPU oracle (action sampling). It is not CUDA's expf:
// Cody-Waite argument reduction x = k*ln2 + r with the two-constant ln2 split
// published in Moshier's Cephes library (C1 = 0.693359375, C2 = -2.12194440e-4),
// then the degree-7 Taylor polynomial of e^r (coefficients 1/k!) by Horner's
// rule, then scaling by 2^k through the exponent field. Compiled without FMA
// contraction on both sides, every operation is a correctly rounded IEEE op,
// so host and device agree bit for bit. Relative error is below 2e-7 on
// [-87, 0]; the argument range used here is x <= 0 (logit minus the maximum).
#pragma once
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define D1_HD __host__ __device__ __forceinline__
#else
#define D1_HD static inline
#endif

D1_HD float d1_bits_float(uint32_t u) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

// Separately rounded multiply and add: never contracted into an FMA, whatever
// the compiler's --fmad setting, so host and device round identically.
#ifdef __CUDA_ARCH__
#define D1_MUL(a, b) __fmul_rn((a), (b))
#define D1_ADD(a, b) __fadd_rn((a), (b))
#else
#define D1_MUL(a, b) ((a) * (b))
#define D1_ADD(a, b) ((a) + (b))
#endif

D1_HD float d1_rint(float x) {
#ifdef __CUDA_ARCH__
    return rintf(x);
#else
    return __builtin_rintf(x);
#endif
}

// e^x for x <= 0; 0 below -87 (where e^x is below the float normal range).
D1_HD float d1_exp_nonpos(float x) {
    if (x < -87.0f) return 0.0f;
    const float k = d1_rint(D1_MUL(x, 1.44269504088896341f));
    float r = D1_ADD(x, -D1_MUL(k, 0.693359375f));
    r = D1_ADD(r, -D1_MUL(k, -2.12194440e-4f));
    float p = 1.0f / 5040.0f;
    p = D1_ADD(D1_MUL(p, r), 1.0f / 720.0f);
    p = D1_ADD(D1_MUL(p, r), 1.0f / 120.0f);
    p = D1_ADD(D1_MUL(p, r), 1.0f / 24.0f);
    p = D1_ADD(D1_MUL(p, r), 1.0f / 6.0f);
    p = D1_ADD(D1_MUL(p, r), 0.5f);
    p = D1_ADD(D1_MUL(p, r), 1.0f);
    p = D1_ADD(D1_MUL(p, r), 1.0f);
    const int ki = (int)k;  // in [-126, 0]
    return D1_MUL(p, d1_bits_float((uint32_t)(ki + 127) << 23));
}
