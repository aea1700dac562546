// Packed fp32 arithmetic and a special-function-unit-free exp2 for sm_100a: shared by the
// attention softmax and the bf16/fp16 logsumexp folds, where the 16-per-clock-per-SM exponential
// unit, not memory or the tensor cores, would set the pace.
#pragma once

#include <stdint.h>

namespace nb200 {

// Pairs of fp32 values in one 64-bit register, for the sm_100 packed f32x2 instructions.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
    return (uint64_t)__float_as_uint(lo) | ((uint64_t)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float f2lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// 2^x on the special-function unit; subnormal results flush to zero (every caller adds them to a
// sum that already holds the maximum's 2^0 = 1, where they vanish).
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x for a pair on the FMA pipe, to take part of the exponentials off the special-function unit.
// Cody-Waite style range reduction x = j + f with j = round(x) (adding and subtracting 1.5 * 2^23
// rounds to an integer in the low mantissa bits of t) and f in [-1/2, 1/2]; 2^f from a degree-4
// polynomial fitted here for minimum relative error on [-1/2, 1/2] (max relative error 2.6e-6:
// far below a bf16 probability's 2^-9 rounding, and small enough that the row sums, hence the
// log-sum-exp, keep fp32-level accuracy); 2^j is added to the exponent field as j << 23,
// which the integer multiply-add bits(t) * 2^23 + bits(2^f) produces because bits(t) = 0x4B400000
// + j and 0x4B400000 * 2^23 vanishes mod 2^32. x must be >= -126 (the caller clamps).
constexpr float kPolyC0 = 0.9999992847442627f, kPolyC1 = 0.6931217908859253f;
constexpr float kPolyC2 = 0.2402474582195282f, kPolyC3 = 0.05591786280274391f;
constexpr float kPolyC4 = 0.00957004725933075f;
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x) {
    const float magic = 12582912.f;  // 1.5 * 2^23
    const uint64_t t = add2(x, f2(magic, magic));
    const uint64_t jf = add2(t, f2(-magic, -magic));
    const uint64_t f = fma2(jf, f2(-1.f, -1.f), x);
    uint64_t p = fma2(f2(kPolyC4, kPolyC4), f, f2(kPolyC3, kPolyC3));
    p = fma2(p, f, f2(kPolyC2, kPolyC2));
    p = fma2(p, f, f2(kPolyC1, kPolyC1));
    p = fma2(p, f, f2(kPolyC0, kPolyC0));
    const uint32_t lo = (uint32_t)t * 0x800000u + (uint32_t)p;
    const uint32_t hi = (uint32_t)(t >> 32) * 0x800000u + (uint32_t)(p >> 32);
    return (uint64_t)lo | ((uint64_t)hi << 32);
}

}  // namespace nb200
