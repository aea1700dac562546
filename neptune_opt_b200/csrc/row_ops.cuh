// The fused row operations (Ops) shared by the bulk-copy streaming kernel (stream.cu) and the
// register-row kernel (rows_ldg.cu), with the packed-arithmetic helpers they use.
//   FoldOp    the serial repaired fold of any skeleton (template.py:41-54, two-pass :62-103)
//   SoftmaxOp softmax / log_softmax + logsumexp (the lowering of neptune_recognize/lowering.py:80-99)
//   L2Op      stable_l2 norm and x / norm
//   RmsOp     RMSNorm with the reference's fp32 stages (emitters.py:576-595)
#pragma once

#include <type_traits>

#include "stream.cuh"

namespace nb200 {

// ------------------------------------------------------------------ packed arithmetic helpers
__device__ __forceinline__ unsigned long long pk(float a, float b) {
    return (static_cast<unsigned long long>(__float_as_uint(b)) << 32) | __float_as_uint(a);
}
__device__ __forceinline__ float lo_f(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi_f(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ unsigned long long mul_f32x2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Two storage values of one 32-bit word as fp32 (low half first).
template <typename T> struct Word;
template <> struct Word<__nv_bfloat16> {
    __device__ __forceinline__ static unsigned long long unpack(uint32_t w) {
        return pk(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
    // RN(a * g) of bf16 pairs: the product of two bf16 values is exact in fp32, so this is the
    // reference's fp32 product rounded to bf16.
    __device__ __forceinline__ static uint32_t round_pair(unsigned long long v) {
        __nv_bfloat162 h = __floats2bfloat162_rn(lo_f(v), hi_f(v));
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static uint32_t mul_pair(uint32_t a, uint32_t g) {
        uint32_t d;
        asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(g));
        return d;
    }
};
template <> struct Word<__half> {
    __device__ __forceinline__ static unsigned long long unpack(uint32_t w) {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        float2 f = __half22float2(h);
        return pk(f.x, f.y);
    }
    __device__ __forceinline__ static uint32_t round_pair(unsigned long long v) {
        __half2 h = __floats2half2_rn(lo_f(v), hi_f(v));
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static uint32_t mul_pair(uint32_t a, uint32_t g) {
        uint32_t d;
        asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(g));
        return d;
    }
};

__device__ __forceinline__ uint32_t word(const uint4& u, int i) {
    return i == 0 ? u.x : i == 1 ? u.y : i == 2 ? u.z : u.w;
}

// ------------------------------------------------------------------ Ops
// Each Op's row() takes the row as a row source (SmemRow: staged in shared memory; RegRow: held in
// registers), so the same arithmetic serves the bulk-copy kernel and the register kernel.
template <int S, typename T>
struct FoldOp {
    T* out;
    Params p;
    int nv;
    __device__ __forceinline__ void prologue(unsigned char*) const {}
    template <class Src>
    __device__ __forceinline__ void row(const Src& src, int64_t r, int lane, const unsigned char*) const {
        float res;
        if constexpr (Sk<S>::kind == K_TWOPASS) {
            constexpr int V = Elem<T>::V;
            float sv[V], av[V];
#pragma unroll
            for (int e = 0; e < V; ++e) { sv[e] = 0.f; av[e] = 0.f; }
            src.for_each([&](const uint4& u, int) {
#pragma unroll
                for (int e = 0; e < V; ++e) sv[e] += Elem<T>::lane(u, e) * p.invN;
            });
            const float mean = warp_sum(combine_sum<V>(sv));
            src.for_each([&](const uint4& u, int) {
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const float d = Elem<T>::lane(u, e) - mean;
                    av[e] += p.invN * (d * d);
                }
            });
            res = Sk<S>::fin(warp_sum(combine_sum<V>(av)));
        } else {
            res = finalize<S>(row_state<S, T>(src, p), p);
        }
        if (lane == 0) out[r] = Elem<T>::from_f(res);
    }
};

// Row sources that hold the whole row in registers (the register-row kernel's full rows).
template <class Src, class = void> struct HoldsRegisters : std::false_type {};
template <class Src> struct HoldsRegisters<Src, std::void_t<decltype(Src::kRegisters)>> : std::true_type {};

template <typename T>
struct SoftmaxOp {
    T* y;
    T* lse;
    int64_t ncols;
    int nv, mode;
    __device__ __forceinline__ void prologue(unsigned char*) const {}

    // softmax of an fp32 row held whole in registers: the exponentials of the sum pass are kept
    // (over the row's own registers) and scaled by 1/sum for the output, so every element takes
    // one exponential instead of two. Rows with a NaN or an infinity return false and take the
    // general path below (exact status semantics).
    template <class Src>
    __device__ __forceinline__ bool softmax_in_registers(const Src& src, int64_t r, int lane) const {
        constexpr int NV = sizeof(src.r) / sizeof(uint4);
        float mx[4] = {-NB200_INF, -NB200_INF, -NB200_INF, -NB200_INF}, probe = 0.f;
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const uint4 u = src.r[k];
            mx[0] = fmaxf(mx[0], __uint_as_float(u.x));
            mx[1] = fmaxf(mx[1], __uint_as_float(u.y));
            mx[2] = fmaxf(mx[2], __uint_as_float(u.z));
            mx[3] = fmaxf(mx[3], __uint_as_float(u.w));
            probe = fmaf(__uint_as_float(u.x) + __uint_as_float(u.y) + __uint_as_float(u.z) + __uint_as_float(u.w),
                         0.f, probe);
        }
        if (!__all_sync(0xffffffffu, probe == 0.f)) return false;
        const float m = warp_max(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
        const float nm = -m * kLog2e;
        uint4 e[NV];
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            const uint4 u = src.r[k];
            const float e0 = ex2(fmaf(__uint_as_float(u.x), kLog2e, nm)), e1 = ex2(fmaf(__uint_as_float(u.y), kLog2e, nm));
            const float e2 = ex2(fmaf(__uint_as_float(u.z), kLog2e, nm)), e3 = ex2(fmaf(__uint_as_float(u.w), kLog2e, nm));
            acc[0] += e0;
            acc[1] += e1;
            acc[2] += e2;
            acc[3] += e3;
            e[k] = make_uint4(__float_as_uint(e0), __float_as_uint(e1), __float_as_uint(e2), __float_as_uint(e3));
        }
        const float s = warp_sum((acc[0] + acc[1]) + (acc[2] + acc[3]));
        const float inv = 1.0f / s;
        float* yrow = reinterpret_cast<float*>(y) + r * ncols;
#pragma unroll
        for (int k = 0; k < NV; ++k)
            st_stream(yrow + (int64_t)(lane + 32 * k) * 4,
                      make_uint4(__float_as_uint(__uint_as_float(e[k].x) * inv), __float_as_uint(__uint_as_float(e[k].y) * inv),
                                 __float_as_uint(__uint_as_float(e[k].z) * inv), __float_as_uint(__uint_as_float(e[k].w) * inv)));
        if (lse != nullptr && lane == 0) reinterpret_cast<float*>(lse)[r] = m + logf(s);
        return true;
    }

    template <class Src>
    __device__ __forceinline__ void row(const Src& src, int64_t r, int lane, const unsigned char*) const {
        if constexpr (std::is_same<T, float>::value && HoldsRegisters<Src>::value) {
            if (mode == 0 && softmax_in_registers(src, r, lane)) return;
        }
        constexpr int V = Elem<T>::V;
        const Params p{0.f, 0.f, 1.f, 1.f, 0.f, 0.f, 0.f};
        const St s = row_state<NB200_LOGSUMEXP, T>(src, p);
        const bool bad = s.status != 0 || !s.seen;
        const float m = s.m, inv = 1.0f / s.acc, lg = logf(s.acc);
        T* yrow = y + r * ncols;
        src.for_each([&](const uint4& u, int j) {
            float f[V];
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float d = Elem<T>::lane(u, e) - m;
                f[e] = bad ? NB200_NAN : (mode == 0 ? fexp(d) * inv : d - lg);
            }
            st_stream(yrow + (int64_t)j * V, Elem<T>::pack(f));
        });
        if (lse != nullptr && lane == 0) lse[r] = Elem<T>::from_f(finalize<NB200_LOGSUMEXP>(s, p));
    }
};

template <typename T>
struct L2Op {
    T* y;
    T* norm;
    int64_t ncols;
    int nv;
    __device__ __forceinline__ void prologue(unsigned char*) const {}
    template <class Src>
    __device__ __forceinline__ void row(const Src& src, int64_t r, int lane, const unsigned char*) const {
        constexpr int V = Elem<T>::V;
        const Params p{0.f, 0.f, 1.f, 1.f, 0.f, 0.f, 0.f};
        const float nrm = finalize<NB200_STABLE_L2>(row_state<NB200_STABLE_L2, T>(src, p), p);
        const float inv = 1.0f / nrm;
        T* yrow = y + r * ncols;
        src.for_each([&](const uint4& u, int j) {
            float f[V];
#pragma unroll
            for (int e = 0; e < V; ++e) f[e] = Elem<T>::lane(u, e) * inv;
            st_stream(yrow + (int64_t)j * V, Elem<T>::pack(f));
        });
        if (norm != nullptr && lane == 0) norm[r] = Elem<T>::from_f(nrm);
    }
};

// gamma (ncols values) is staged once per CTA at the start of shared memory.
template <typename T>
struct RmsOp {
    T* y;
    const T* gamma;
    int64_t ncols, sg;
    int nv;
    float eps, count;
    __device__ __forceinline__ void prologue(unsigned char* smem) const {
        T* g = reinterpret_cast<T*>(smem);
        for (int64_t c = threadIdx.x; c < ncols; c += blockDim.x) g[c] = gamma[c * sg];
    }
    template <class Src>
    __device__ __forceinline__ void row(const Src& src, int64_t r, int lane, const unsigned char* smem) const {
        constexpr int V = Elem<T>::V;
        const uint4* g = reinterpret_cast<const uint4*>(smem);
        T* yrow = y + r * ncols;
        if constexpr (sizeof(T) == 2) {
            // sum of squares: every square and every add rounded (no contraction), two lanes of
            // fp32 per instruction
            unsigned long long acc[4] = {0ull, 0ull, 0ull, 0ull};
            src.for_each([&](const uint4& u, int) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const unsigned long long f = Word<T>::unpack(word(u, i));
                    acc[i] = add_f32x2(acc[i], mul_f32x2(f, f));
                }
            });
            const unsigned long long a01 = add_f32x2(acc[0], acc[1]), a23 = add_f32x2(acc[2], acc[3]);
            const unsigned long long a = add_f32x2(a01, a23);
            const float total = warp_sum(__fadd_rn(lo_f(a), hi_f(a)));
            const float mean = __fdiv_rn(total, count);
            const float scale = __frsqrt_rn(__fadd_rn(mean, eps));
            const unsigned long long sc = pk(scale, scale);
            src.for_each([&](const uint4& u, int j) {
                const uint4 gg = g[j];
                uint4 o;
                o.x = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(u.x), sc)), gg.x);
                o.y = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(u.y), sc)), gg.y);
                o.z = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(u.z), sc)), gg.z);
                o.w = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(u.w), sc)), gg.w);
                st_stream(yrow + (int64_t)j * V, o);
            });
        } else {
            unsigned long long acc0 = 0ull, acc1 = 0ull;
            src.for_each([&](const uint4& u, int) {
                const unsigned long long a = pk(__uint_as_float(u.x), __uint_as_float(u.y));
                const unsigned long long b = pk(__uint_as_float(u.z), __uint_as_float(u.w));
                acc0 = add_f32x2(acc0, mul_f32x2(a, a));
                acc1 = add_f32x2(acc1, mul_f32x2(b, b));
            });
            const unsigned long long acc = add_f32x2(acc0, acc1);
            const float total = warp_sum(__fadd_rn(lo_f(acc), hi_f(acc)));
            const float mean = __fdiv_rn(total, count);
            const float scale = __frsqrt_rn(__fadd_rn(mean, eps));
            const unsigned long long sc = pk(scale, scale);
            src.for_each([&](const uint4& u, int j) {
                const uint4 gg = g[j];
                const unsigned long long a = mul_f32x2(mul_f32x2(pk(__uint_as_float(u.x), __uint_as_float(u.y)), sc),
                                                       pk(__uint_as_float(gg.x), __uint_as_float(gg.y)));
                const unsigned long long b = mul_f32x2(mul_f32x2(pk(__uint_as_float(u.z), __uint_as_float(u.w)), sc),
                                                       pk(__uint_as_float(gg.z), __uint_as_float(gg.w)));
                st_stream(yrow + (int64_t)j * V, make_uint4(static_cast<uint32_t>(a), static_cast<uint32_t>(a >> 32),
                                                            static_cast<uint32_t>(b), static_cast<uint32_t>(b >> 32)));
            });
        }
    }
};

// Register-row kernel (rows_ldg.cu): one warp per row, the whole row loaded into registers with
// plain vector loads. For contiguous, 16-byte-aligned rows of 64..512 vectors (1-8 KB); smem holds
// what op.prologue stages (RMSNorm's gamma).
template <typename T, class Op>
int launch_ldg_rows(const T* x, int64_t rows, int64_t srow, const Op& op, uint32_t smem, cudaStream_t st,
                    const char* what);

// Column-span folds (split-plan chunks, or whole rows with finalize = 1) with register sub-blocks
// (rows_ldg.cu). Returns 1 when launched, 0 for a skeleton it does not take, negative on error.
// Requires x, the span starts and the row stride 16-byte aligned.
template <typename T>
int launch_ldg_span(int sk, const Params& p, const T* x, int64_t rows, int64_t cb, int64_t ns, int64_t srow,
                    int64_t cc, int64_t nparts, nb200_state* states, T* out, int finalize, cudaStream_t st);

// Whether the register-row kernel takes a row of `row_bytes` (16-byte multiple) by default.
inline bool ldg_rows_eligible(uint32_t row_bytes) { return row_bytes >= 1024 && row_bytes <= 8192; }

}  // namespace nb200
