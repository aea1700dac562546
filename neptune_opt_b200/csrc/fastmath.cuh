// Packed fp32 arithmetic for sm_100a, shared by the attention softmax and the bf16/fp16
// logsumexp folds: pairs of fp32 values in one 64-bit register for the f32x2 instructions, the
// three-input max, and 2^x on the special-function unit.
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

}  // namespace nb200
