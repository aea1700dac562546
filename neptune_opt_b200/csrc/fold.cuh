// The repaired fold of two dependent row reductions, as device algebra.
//
// A fold state is (m, acc, seen, status): the raw producer value, the fp32 accumulator, whether
// any element reached the accumulator, and nonfinite status bits (log family only: bit 0 NaN,
// bit 1 +inf). This is the state of the reference's generated chunk/merge helpers
// (neptune_codegen/emitters.py:436-519) and its finaliser (emitters.py:522-532); the per-skeleton
// term, repair factor and readout follow the merge certificates derived in
// neptune_codegen/algebra.py:348-403 for the eleven skeletons of neptune_codegen/library.py.
#pragma once

#include "common.cuh"

namespace nb200 {

// fp32 copies of the skeleton scalars. invT = 1/T and invN = 1/ncols are formed on the host in
// binary64 and narrowed once, as the reference's literal `1.0 / T` is.
struct Params {
    float tiny, alpha, invT, beta, N, eps, invN;
};

enum Kind { K_LOG = 0, K_MAXABS = 1, K_SUMMAX = 2, K_TWOPASS = 3 };

struct St {
    float m, acc;
    int seen, status;
};

template <int S> struct Sk;

// ---- exponential (log) family: g = exp(phi(c) - s); producer max phi, consumer sum.
template <> struct Sk<NB200_LOGSUMEXP> {
    static constexpr int kind = K_LOG;
    __device__ __forceinline__ static float phi(float v, const Params&) { return v; }
};
template <> struct Sk<NB200_LSE_BIASED> {
    static constexpr int kind = K_LOG;
    __device__ __forceinline__ static float phi(float v, const Params& p) { return p.alpha + v; }
};
template <> struct Sk<NB200_LSE_SCALED> {
    static constexpr int kind = K_LOG;
    __device__ __forceinline__ static float phi(float v, const Params& p) { return v * p.invT; }
};
template <> struct Sk<NB200_SOFTCAP_LSE> {
    static constexpr int kind = K_LOG;
    __device__ __forceinline__ static float phi(float v, const Params& p) { return tanhf(p.beta * v); }
};

// ---- max|c| producer, sum consumer. `floor` marks the zero-singular coordinate that the
// reference floors at 1e-30 on both repair endpoints (algebra.py:329-345).
// term(v, den) is the consumer term; prep(den) and term_r(v, c) give the same term with the
// per-chunk constant c = prep(den) hoisted out of the element loop (a reciprocal instead of a
// division per element; the two differ by at most one rounding).
template <> struct Sk<NB200_STABLE_L2> {
    static constexpr int kind = K_MAXABS;
    static constexpr bool floor = true;
    __device__ __forceinline__ static float term(float v, float den, const Params&) {
        const float r = v / den;
        return r * r;
    }
    __device__ __forceinline__ static float prep(float den, const Params&) { return 1.0f / den; }
    __device__ __forceinline__ static float term_r(float v, float c) {
        const float r = v * c;
        return r * r;
    }
    __device__ __forceinline__ static float factor(float q, float qn, const Params&) {
        const float r = q / qn;
        return r * r;
    }
    __device__ __forceinline__ static float fin(float m, float acc, const Params&) {
        return fmaxf(m, 1e-30f) * sqrtf(acc);
    }
};
template <> struct Sk<NB200_LINEAR_ATTN> {
    static constexpr int kind = K_MAXABS;
    static constexpr bool floor = true;
    __device__ __forceinline__ static float term(float v, float den, const Params&) { return v / den; }
    __device__ __forceinline__ static float prep(float den, const Params&) { return 1.0f / den; }
    __device__ __forceinline__ static float term_r(float v, float c) { return v * c; }
    __device__ __forceinline__ static float factor(float q, float qn, const Params&) { return q / qn; }
    __device__ __forceinline__ static float fin(float, float acc, const Params&) { return acc; }
};
template <> struct Sk<NB200_DECAY_RENORM> {
    static constexpr int kind = K_MAXABS;
    static constexpr bool floor = false;
    __device__ __forceinline__ static float term(float v, float den, const Params& p) { return v / (den + p.N); }
    __device__ __forceinline__ static float prep(float den, const Params& p) { return 1.0f / (den + p.N); }
    __device__ __forceinline__ static float term_r(float v, float c) { return v * c; }
    __device__ __forceinline__ static float factor(float q, float qn, const Params& p) {
        return (q + p.N) / (qn + p.N);
    }
    __device__ __forceinline__ static float fin(float, float acc, const Params&) { return acc; }
};
template <> struct Sk<NB200_SUMSQ_DIV> {
    static constexpr int kind = K_MAXABS;
    static constexpr bool floor = true;
    __device__ __forceinline__ static float term(float v, float den, const Params&) {
        return (v * v) * (1.0f / den);
    }
    __device__ __forceinline__ static float prep(float den, const Params&) { return 1.0f / den; }
    __device__ __forceinline__ static float term_r(float v, float c) { return (v * v) * c; }
    __device__ __forceinline__ static float factor(float q, float qn, const Params&) { return q / qn; }
    __device__ __forceinline__ static float fin(float, float acc, const Params&) { return acc; }
};

// ---- sum producer mean(c^2), max consumer c / sqrt(s + eps): the paper's RMSNorm+max.
template <> struct Sk<NB200_RMSNORM_MAX> {
    static constexpr int kind = K_SUMMAX;
    static constexpr bool floor = false;
    __device__ __forceinline__ static float operand(float v, const Params& p) { return (v * v) * p.invN; }
    __device__ __forceinline__ static float term_scale(float den, const Params& p) {
        return 1.0f / sqrtf(den + p.eps);
    }
    __device__ __forceinline__ static float factor(float q, float qn, const Params& p) {
        return sqrtf(q + p.eps) * (1.0f / sqrtf(qn + p.eps));
    }
    __device__ __forceinline__ static float fin(float, float acc, const Params&) { return acc; }
};

// ---- two-pass plan (template.py:62-103): no repair exists; the producer is final in pass 2.
template <> struct Sk<NB200_VARIANCE> {
    static constexpr int kind = K_TWOPASS;
    __device__ __forceinline__ static float fin(float acc) { return acc; }
};
template <> struct Sk<NB200_STD> {
    static constexpr int kind = K_TWOPASS;
    __device__ __forceinline__ static float fin(float acc) { return sqrtf(acc); }
};

__device__ __forceinline__ St empty_state() { return St{-NB200_INF, 0.f, 0, 0}; }

// State of one resident chunk (columns [c0, c_hi) of the chunk's span are valid). This is the
// reference's `{sk}_chunk` helper (emitters.py:459-488): for the log family the max and the sum
// run over finite phi only, with NaN/+inf recorded in status; otherwise every in-range column
// enters both reductions.
template <int S, typename CH, bool CTA>
__device__ __forceinline__ St chunk_state(const CH& ch, int64_t c0, int64_t c_hi, int t, int G,
                                          Group<CTA>& grp, const Params& p) {
    using K = Sk<S>;
    if constexpr (K::kind == K_LOG) {
        float mloc = -NB200_INF;
        int st = 0;
#pragma unroll
        for (int i = 0; i < CH::E; ++i) {
            if (CH::valid(c0, c_hi, t, G, i)) {
                const float ph = K::phi(ch.get(i), p);
                if (ph != ph) st |= 1;
                else if (ph == NB200_INF) st |= 2;
                else mloc = fmaxf(mloc, ph);
            }
        }
        const float m = grp.reduce(mloc, RED_MAX);
        st = grp.reduce_or(st);
        const bool seen = m != -NB200_INF;
        const float den = seen ? m : 0.f;
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < CH::E; ++i) {
            if (CH::valid(c0, c_hi, t, G, i)) {
                const float ph = K::phi(ch.get(i), p);
                if (fabsf(ph) < NB200_INF) a += expf(ph - den);
            }
        }
        a = grp.reduce(a, RED_SUM);
        return St{m, a, seen ? 1 : 0, st};
    } else if constexpr (K::kind == K_MAXABS) {
        float mloc = 0.f;
#pragma unroll
        for (int i = 0; i < CH::E; ++i)
            if (CH::valid(c0, c_hi, t, G, i)) mloc = fmaxf(mloc, fabsf(ch.get(i)));
        const float m = grp.reduce(mloc, RED_MAX);
        const float den = K::floor ? fmaxf(m, 1e-30f) : m;
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < CH::E; ++i)
            if (CH::valid(c0, c_hi, t, G, i)) a += K::term(ch.get(i), den, p);
        a = grp.reduce(a, RED_SUM);
        return St{m, a, 1, 0};
    } else {  // K_SUMMAX
        float sl = 0.f;
#pragma unroll
        for (int i = 0; i < CH::E; ++i)
            if (CH::valid(c0, c_hi, t, G, i)) sl += K::operand(ch.get(i), p);
        const float m = grp.reduce(sl, RED_SUM);
        const float r = K::term_scale(m, p);
        float a = -NB200_INF;
#pragma unroll
        for (int i = 0; i < CH::E; ++i)
            if (CH::valid(c0, c_hi, t, G, i)) a = fmaxf(a, ch.get(i) * r);
        a = grp.reduce(a, RED_MAX);
        return St{m, a, 1, 0};
    }
}

// merge_state: A is the left (earlier columns / lower part index), B the right operand.
template <int S>
__device__ __forceinline__ St merge(const St& A, const St& B, const Params& p) {
    using K = Sk<S>;
    const int status = A.status | B.status;
    if (!B.seen) return St{A.m, A.acc, A.seen, status};
    if (!A.seen) return St{B.m, B.acc, 1, status};
    St r;
    r.seen = 1;
    r.status = status;
    if constexpr (K::kind == K_LOG) {
        r.m = fmaxf(A.m, B.m);
        r.acc = A.acc * expf(A.m - r.m) + B.acc * expf(B.m - r.m);
    } else if constexpr (K::kind == K_MAXABS) {
        r.m = fmaxf(A.m, B.m);
        const float qa = K::floor ? fmaxf(A.m, 1e-30f) : A.m;
        const float qb = K::floor ? fmaxf(B.m, 1e-30f) : B.m;
        const float qn = K::floor ? fmaxf(r.m, 1e-30f) : r.m;
        r.acc = A.acc * K::factor(qa, qn, p) + B.acc * K::factor(qb, qn, p);
    } else {  // K_SUMMAX
        r.m = A.m + B.m;
        r.acc = fmaxf(A.acc * K::factor(A.m, r.m, p), B.acc * K::factor(B.m, r.m, p));
    }
    return r;
}

template <int S>
__device__ __forceinline__ float finalize(const St& s, const Params& p) {
    using K = Sk<S>;
    if constexpr (K::kind == K_LOG) {
        if (s.status & 1) return NB200_NAN;
        if (s.status & 2) return NB200_INF;
        if (!s.seen) return -NB200_INF;
        return s.m + logf(s.acc + p.tiny);
    } else {
        return K::fin(s.m, s.acc, p);
    }
}

}  // namespace nb200
