// t3_expf.h — single-precision exp shared by host and device code.
//
// The reference sampler (src/main.cpp:756,787 in chatterbox.cpp) calls
// std::exp(float), i.e. the host C library's expf.  The device must produce
// the same float for every argument the sampler can reach (x <= 0), so this
// file defines exp in two layers:
//
//   t3_expf_core(x)  a restatement of glibc's expf (the published
//                    ARM optimized-routines algorithm, glibc >= 2.28):
//                    k = round(x*32/ln2) by the 1.5*2^52 shift trick,
//                    r = x*32/ln2 - k, 2^(k/32) from a 32-entry table of
//                    2^(i/32), exp = 2^(k/32) * (1 + C2 r + C1 r^2 + C0 r^3),
//                    every step an IEEE double operation and the steps
//                    fused the way GCC contracts them in glibc's x86-64 FMA
//                    build; one rounding to float at the end.  Host and
//                    device evaluate it bit-identically.
//   fix-up list      the build (gen_expf_fixup.cpp) scans every float in
//                    [-104, 0] and records the arguments where the host
//                    libm's expf differs from t3_expf_core, with the libm
//                    result (none for glibc's FMA build); the device looks
//                    those up in a hash table (t3b_abi.cu) only when the
//                    list is not empty.
#pragma once

#include <stdint.h>
#include <math.h>

#if defined(__CUDACC__)
#define T3_HD __host__ __device__ __forceinline__
#else
#define T3_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define T3_DMUL(a, b) __dmul_rn((a), (b))
#define T3_DADD(a, b) __dadd_rn((a), (b))
#define T3_DFMA(a, b, c) __fma_rn((a), (b), (c))
#else
#define T3_DMUL(a, b) ((a) * (b))
#define T3_DADD(a, b) ((a) + (b))
#define T3_DFMA(a, b, c) fma((a), (b), (c))
#endif

// Bits of 2^(i/32) rounded to the nearest double, minus i << 47, i = 0..31:
// adding k << 47 for an integer k = 32*q + i gives the bits of 2^(q + i/32).
#define T3_EXP2_TAB_INIT {                                                              \
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull, \
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, \
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull, \
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull, \
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull, \
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull, \
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull, \
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull }

T3_HD double t3_bits_to_double(uint64_t u) {
    double d;
#if defined(__CUDA_ARCH__)
    d = __longlong_as_double((long long) u);
#else
    __builtin_memcpy(&d, &u, 8);
#endif
    return d;
}
T3_HD uint64_t t3_double_to_bits(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t) __double_as_longlong(d);
#else
    uint64_t u;
    __builtin_memcpy(&u, &d, 8);
    return u;
#endif
}

// tab: the 32 words of T3_EXP2_TAB_INIT (any address space).
T3_HD float t3_expf_core(float xf, const unsigned long long * tab) {
    if (xf != xf) return xf + xf;
    if (xf > 0x1.62e42ep6f) return INFINITY;      // above log(FLT_MAX): overflow
    if (xf < -0x1.9fe368p6f) return 0.0f;         // below log(2^-150): underflow to +0
    const double xd = (double) xf;
    const double InvLn2N = 0x1.71547652b82fep+0 * 32.0;   // 32 / ln 2
    const double SHIFT = 0x1.8p+52;
    double kd = T3_DFMA(InvLn2N, xd, SHIFT);            // round(x*32/ln2) in the low bits
    const uint64_t ki = t3_double_to_bits(kd);
    kd = T3_DADD(kd, -SHIFT);
    const double r = T3_DFMA(InvLn2N, xd, -kd);          // |r| <= 1/2
    const double s = t3_bits_to_double(tab[ki & 31u] + (ki << 47));
    const double C0 = 0x1.c6af84b912394p-5 / 32768.0;    // minimax cubic for 2^(r/32)
    const double C1 = 0x1.ebfce50fac4f3p-3 / 1024.0;
    const double C2 = 0x1.62e42ff0c52d6p-1 / 32.0;
    const double z = T3_DFMA(C0, r, C1);
    const double r2 = T3_DMUL(r, r);
    double y = T3_DFMA(C2, r, 1.0);
    y = T3_DFMA(z, r2, y);
    y = T3_DMUL(y, s);
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
