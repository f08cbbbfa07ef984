// t3_expf.h — single-precision exp shared by host and device code.
//
// The reference sampler (src/main.cpp:756,787 in chatterbox.cpp) calls
// std::exp(float), i.e. the host C library's expf.  The device must produce
// the same float for every argument the sampler can reach (x <= 0), so this
// file defines exp in two layers:
//
//   t3_expf_core(x)  exp from first principles in double precision:
//                    x = k*ln2 + r with |r| <= ln2/2 (two-part ln2, fused
//                    multiply-adds), exp(r) by its Taylor series to r^13/13!
//                    (truncation < 2^-57 relative), times 2^k, rounded once
//                    to float.  Every operation is an IEEE double operation
//                    with an explicit fma, so host and device give
//                    bit-identical results.
//   fix-up table     the build (gen_expf_fixup.cpp) scans every float in
//                    [-104, 0] and records the arguments where the host
//                    libm's expf differs from t3_expf_core, together with
//                    the libm result.  The device looks those up in a hash
//                    table (t3b_abi.cu), so device exp == host expf exactly.
#pragma once

#include <stdint.h>
#include <math.h>

#if defined(__CUDACC__)
#define T3_HD __host__ __device__ __forceinline__
#else
#define T3_HD static inline
#endif

T3_HD double t3_pow2i(int k) {
    // 2^k for -1022 <= k <= 1023, built from its exponent field (exact).
    uint64_t bits = (uint64_t) (k + 1023) << 52;
    double d;
#if defined(__CUDA_ARCH__)
    d = __longlong_as_double((long long) bits);
#else
    __builtin_memcpy(&d, &bits, 8);
#endif
    return d;
}

T3_HD float t3_expf_core(float xf) {
    if (xf != xf) return xf;
    if (xf > 88.75f) return INFINITY;
    if (xf < -104.0f) return 0.0f;  // below half of the smallest subnormal
    const double x = (double) xf;
    const double kd = rint(x * 0x1.71547652b82fep+0);          // x / ln2
    double r = fma(-kd, 0x1.62e42fefa39efp-1, x);               // ln2 rounded to double
    r = fma(-kd, 0x1.abc9e3b39803fp-56, r);                     // ln2 - that double
    // sum_{n=0}^{13} r^n / n!  (Horner)
    double p = 0x1.6124613a86d09p-33;
    p = fma(p, r, 0x1.1eed8eff8d898p-29);
    p = fma(p, r, 0x1.ae64567f544e4p-26);
    p = fma(p, r, 0x1.27e4fb7789f5cp-22);
    p = fma(p, r, 0x1.71de3a556c734p-19);
    p = fma(p, r, 0x1.a01a01a01a01ap-16);
    p = fma(p, r, 0x1.a01a01a01a01ap-13);
    p = fma(p, r, 0x1.6c16c16c16c17p-10);
    p = fma(p, r, 0x1.1111111111111p-7);
    p = fma(p, r, 0x1.5555555555555p-5);
    p = fma(p, r, 0x1.5555555555555p-3);
    p = fma(p, r, 0x1.0000000000000p-1);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    const double y = p * t3_pow2i((int) kd);
    return (float) y;
}

// The two candidate buckets of a float's bit pattern in a table of 2^bits
// buckets (two-choice hashing: an entry lives in the emptier of the two, so
// a lookup reads exactly two buckets).
T3_HD uint32_t t3_expf_hash1(uint32_t key, int bits) {
    return (key * 2654435761u) >> (32 - bits);
}
T3_HD uint32_t t3_expf_hash2(uint32_t key, int bits) {
    uint32_t h = key ^ (key >> 15);
    h *= 0x2c1b3c6du;
    h ^= h >> 12;
    h *= 0x297a2d39u;
    h ^= h >> 15;
    return h >> (32 - bits);
}
#define T3_EXPF_SLOTS 4   /* 8-byte slots per bucket: one 32-byte sector */
