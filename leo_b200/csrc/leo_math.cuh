// Exact-parity scalar math shared by the kernels and the host-side table
// generator.
//
// The reference evaluates f32::exp / f32::ln through the platform libm (glibc
// expf / logf) and f32::powi through right-to-left binary exponentiation.  To
// reproduce those bits on the GPU:
//   * leo_expf / leo_logf evaluate the function in double precision with our
//     own Cody-Waite range reduction and Taylor / atanh series (derived from
//     the mathematics: exp(k ln2 + r) = 2^k e^r, log(2^e m) = e ln2 +
//     2 atanh((m-1)/(m+1))), round once to float, and then consult a table of
//     the inputs where glibc's float result differs from that rounding.  The
//     table is produced by leo_b200/csrc/gen_libm_tables.cpp, which compares
//     against the platform libm exhaustively over the domain the step uses.
//   * leo_powi is right-to-left binary exponentiation, the published method.
// All double arithmetic is unfused: build device code with -fmad=false and
// host code with -ffp-contract=off.
#pragma once

#include <stdint.h>
#include <string.h>

#ifndef __CUDACC__
#define LEO_HD inline
#else
#define LEO_HD __host__ __device__ __forceinline__
#endif

namespace leo_math {

// ln 2 split so that k * LN2_HI is exact for |k| < 2^20.
constexpr double LN2_HI = 0.6931471803691238;        // 0x3fe62e42fee00000
constexpr double LN2_LO = 1.9082149292705877e-10;     // ln2 - LN2_HI
constexpr double INV_LN2 = 1.4426950408889634;
constexpr double SQRT2 = 1.4142135623730951;

LEO_HD double bits_to_double(uint64_t b) {
#ifdef __CUDA_ARCH__
    return __longlong_as_double((long long)b);
#else
    double d;
    memcpy(&d, &b, 8);
    return d;
#endif
}
LEO_HD uint64_t double_to_bits(double d) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t b;
    memcpy(&b, &d, 8);
    return b;
#endif
}
LEO_HD uint32_t float_to_bits(float f) {
#ifdef __CUDA_ARCH__
    return __float_as_uint(f);
#else
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
#endif
}
LEO_HD float bits_to_float(uint32_t b) {
#ifdef __CUDA_ARCH__
    return __uint_as_float(b);
#else
    float f;
    memcpy(&f, &b, 4);
    return f;
#endif
}
LEO_HD double round_to_integer(double x) {
#ifdef __CUDA_ARCH__
    return rint(x);
#else
    return __builtin_rint(x);
#endif
}
LEO_HD float double_to_float_rn(double x) {
#ifdef __CUDA_ARCH__
    return __double2float_rn(x);
#else
    return (float)x;
#endif
}

// exp(x) in double for x in [-1022 ln2, 709]; Taylor degree 13 on |r| <= ln2/2.
LEO_HD double exp_double(double x) {
    double k = round_to_integer(x * INV_LN2);
    double r = (x - k * LN2_HI) - k * LN2_LO;
    double p = 1.0 / 6227020800.0;           // 1/13!
    p = p * r + 1.0 / 479001600.0;           // 1/12!
    p = p * r + 1.0 / 39916800.0;            // 1/11!
    p = p * r + 1.0 / 3628800.0;             // 1/10!
    p = p * r + 1.0 / 362880.0;              // 1/9!
    p = p * r + 1.0 / 40320.0;               // 1/8!
    p = p * r + 1.0 / 5040.0;                // 1/7!
    p = p * r + 1.0 / 720.0;                 // 1/6!
    p = p * r + 1.0 / 120.0;                 // 1/5!
    p = p * r + 1.0 / 24.0;                  // 1/4!
    p = p * r + 1.0 / 6.0;                   // 1/3!
    p = p * r + 0.5;                         // 1/2!
    p = p * r + 1.0;                         // 1/1!
    p = p * r + 1.0;                         // 1/0!
    int ki = (int)k;
    return p * bits_to_double((uint64_t)(int64_t)(ki + 1023) << 52);
}

// log(x) in double for a positive normal float input.
LEO_HD double log_double_of_float(float xf) {
    uint32_t b = float_to_bits(xf);
    int e = (int)((b >> 23) & 0xffu) - 127;
    double m = (double)bits_to_float((b & 0x007fffffu) | 0x3f800000u);  // [1, 2)
    if (m > SQRT2) {
        m = m * 0.5;
        e += 1;
    }
    double f = (m - 1.0) / (m + 1.0);
    double f2 = f * f;
    // 2 atanh(f) = 2 (f + f^3/3 + f^5/5 + ...), |f| <= 0.1716, terms to f^27.
    double s = 1.0 / 27.0;
    s = s * f2 + 1.0 / 25.0;
    s = s * f2 + 1.0 / 23.0;
    s = s * f2 + 1.0 / 21.0;
    s = s * f2 + 1.0 / 19.0;
    s = s * f2 + 1.0 / 17.0;
    s = s * f2 + 1.0 / 15.0;
    s = s * f2 + 1.0 / 13.0;
    s = s * f2 + 1.0 / 11.0;
    s = s * f2 + 1.0 / 9.0;
    s = s * f2 + 1.0 / 7.0;
    s = s * f2 + 1.0 / 5.0;
    s = s * f2 + 1.0 / 3.0;
    double logm = 2.0 * f + 2.0 * f * (f2 * s);
    double ed = (double)e;
    return ed * LN2_HI + (logm + ed * LN2_LO);
}

// Right-to-left binary exponentiation (f32::powi with a runtime exponent).
LEO_HD float powi(float base, int32_t exponent) {
    bool recip = exponent < 0;
    uint32_t e = recip ? (uint32_t)(-(int64_t)exponent) : (uint32_t)exponent;
    float result = 1.0f;
    float a = base;
    for (;;) {
        if (e & 1u) result = result * a;
        e >>= 1;
        if (e == 0) break;
        a = a * a;
    }
    return recip ? 1.0f / result : result;
}

// runtime.rs:78-85 decay_for_elapsed
LEO_HD float decay_for_elapsed(float base, uint32_t elapsed) {
    if (elapsed == 0) return 1.0f;
    if (elapsed == 1) return base;
    return powi(base, (int32_t)(elapsed > 0x7fffffffu ? 0x7fffffffu : elapsed));
}

// Binary search in a sorted table of (input bits, output bits) pairs.
LEO_HD bool table_lookup(const uint32_t* keys, const uint32_t* values, int count, uint32_t key, uint32_t* out) {
    int lo = 0, hi = count;
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        uint32_t k = keys[mid];
        if (k == key) {
            *out = values[mid];
            return true;
        }
        if (k < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    return false;
}

}  // namespace leo_math
