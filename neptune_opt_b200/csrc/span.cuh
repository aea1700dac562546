// The column-span fold shared by the split plan's span kernel (rows_ldg.cu) and the fused
// exchange of the column-sharded split across GPUs (fold.cu): a warp folds one item (row, column
// span) in sub-blocks of 32 x kSpanNV vectors (4 KB) loaded into registers at once. Per lane a
// running fold state absorbs each sub-block; at the item's end the 32 lane states merge in a fixed
// tree (lower lane on the left). Measured on B200 (bf16 [512, 262144], 16K-column chunks): single
// 4 KB blocks with ~2x the resident warps beat double-buffered blocks, 54.9 us against 70.8 us.
#pragma once

#include <type_traits>

#include "fastmath.cuh"
#include "stream.cuh"

namespace nb200 {

constexpr int kLdgThreads = 128;  // threads of the register-row and span kernels
constexpr int kSpanNV = 8;

struct LdgSpan {
    int64_t rows, srow, cb, ns, cc, nparts, nitems;
    int finalize;
};

template <int NV, typename T>
__device__ __forceinline__ void load_block(RegRow<NV>& b, const uint4* base, int v0, int nvec, int lane) {
    b.lane = lane;
    b.nv = min(32 * NV, nvec - v0);
#pragma unroll
    for (int k = 0; k < NV; ++k)
        b.r[k] = (lane + 32 * k < b.nv) ? ld_stream(base + v0 + lane + 32 * k) : make_uint4(0u, 0u, 0u, 0u);
}

// 16-bit logsumexp sub-block: packed max with NaN propagation (a NaN or +inf in the block sends it
// to the exact path), an online rescale of the lane's running sum when the block raises its max,
// and 2^(x log2 e - m log2 e) on packed fp32 pairs. (Moving a share of the exponentials to an
// FMA-pipe polynomial was measured slower here: this loop is bound by instruction issue, not by
// the special-function unit.)
template <typename T>
__device__ __forceinline__ uint32_t max_nan2(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (sizeof(T) == 2 && Elem<T>::V == 8 && std::is_same<T, __half>::value)
        asm("max.NaN.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else
        asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
template <typename T>
__device__ __forceinline__ uint64_t widen2(uint32_t w) {
    if constexpr (std::is_same<T, __half>::value) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w));
        return f2(f.x, f.y);
    } else {
        return f2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
    }
}

template <typename T, int NV = kSpanNV>
__device__ __forceinline__ void lse16_block(const RegRow<NV>& blk, St& run, const Params& p) {
    const uint32_t ninf = std::is_same<T, __half>::value ? 0xFC00FC00u : 0xFF80FF80u;
    uint32_t mw[4] = {ninf, ninf, ninf, ninf};
    blk.for_each([&](const uint4& u, int) {
        mw[0] = max_nan2<T>(mw[0], u.x);
        mw[1] = max_nan2<T>(mw[1], u.y);
        mw[2] = max_nan2<T>(mw[2], u.z);
        mw[3] = max_nan2<T>(mw[3], u.w);
    });
    const uint64_t m2 = widen2<T>(max_nan2<T>(max_nan2<T>(mw[0], mw[1]), max_nan2<T>(mw[2], mw[3])));
    const float bm = fmaxf(f2lo(m2), f2hi(m2));
    if (f2lo(m2) != f2lo(m2) || f2hi(m2) != f2hi(m2) || bm == NB200_INF) {  // NaN or +inf: exact status
        run = merge_fast<NB200_LOGSUMEXP>(run, lane_state<NB200_LOGSUMEXP, T>(blk, p), p);
        return;
    }
    if (bm == -NB200_INF) return;  // nothing above -inf (or no element) in this lane's part
    if (!run.seen || bm > run.m) {
        if (run.seen) run.acc *= fexp(run.m - bm);
        run.m = bm;
        run.seen = 1;
    }
    const float nm = -run.m * kLog2e;
    const uint64_t l2e = f2(kLog2e, kLog2e), nm2 = f2(nm, nm);
    uint64_t acc[2] = {0ull, 0ull};
#pragma unroll
    for (int k = 0; k < NV; ++k) {
        if (blk.lane + 32 * k >= blk.nv) continue;
        const uint32_t w[4] = {blk.r[k].x, blk.r[k].y, blk.r[k].z, blk.r[k].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint64_t x = fma2(widen2<T>(w[i]), l2e, nm2);
            acc[i & 1] = add2(acc[i & 1], f2(ex2_ftz(f2lo(x)), ex2_ftz(f2hi(x))));
        }
    }
    const uint64_t a = add2(acc[0], acc[1]);
    run.acc += f2lo(a) + f2hi(a);
}


// States of G whole 16-bit logsumexp items resident in `blk[g]`, each formed as row_state forms a
// resident row (warp max first, every exponential against it, one warp sum; no repair) on packed
// pairs: max.NaN on raw 16-bit pairs, exponent arguments and sums on fp32 pairs. The G items'
// reductions interleave (one shuffle chain for all of them). A NaN or +inf anywhere in any of them
// sends the warp to the exact lane-state merge for each item.
template <typename T, int NV, int G>
__device__ __forceinline__ void lse16_rows_state(const RegRow<NV> (&blk)[G], St (&out)[G], const Params& p) {
    const uint32_t ninf = std::is_same<T, __half>::value ? 0xFC00FC00u : 0xFF80FF80u;
    float m[G];
    bool exact = false;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        uint32_t mw[4] = {ninf, ninf, ninf, ninf};
        blk[g].for_each([&](const uint4& u, int) {
            mw[0] = max_nan2<T>(mw[0], u.x);
            mw[1] = max_nan2<T>(mw[1], u.y);
            mw[2] = max_nan2<T>(mw[2], u.z);
            mw[3] = max_nan2<T>(mw[3], u.w);
        });
        const uint64_t m2 = widen2<T>(max_nan2<T>(max_nan2<T>(mw[0], mw[1]), max_nan2<T>(mw[2], mw[3])));
        m[g] = fmaxf(f2lo(m2), f2hi(m2));
        exact |= f2lo(m2) != f2lo(m2) || f2hi(m2) != f2hi(m2) || m[g] == NB200_INF;
    }
    if (__any_sync(0xffffffffu, exact)) {
#pragma unroll
        for (int g = 0; g < G; ++g)
            out[g] = warp_merge<NB200_LOGSUMEXP>(lane_state<NB200_LOGSUMEXP, T>(blk[g], p), blk[g].lane, p);
        return;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) m[g] = fmaxf(m[g], __shfl_xor_sync(0xffffffffu, m[g], o));
    }
    const uint64_t l2e = f2(kLog2e, kLog2e);
    float sum[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        // an item with no element above -inf keeps an empty sum (its exponent arguments are not formed)
        const float nm = m[g] == -NB200_INF ? 0.f : -m[g] * kLog2e;
        const uint64_t nm2 = f2(nm, nm);
        uint64_t acc[2] = {0ull, 0ull};
#pragma unroll
        for (int k = 0; k < NV; ++k) {
            if (blk[g].lane + 32 * k >= blk[g].nv || m[g] == -NB200_INF) continue;
            const uint32_t w[4] = {blk[g].r[k].x, blk[g].r[k].y, blk[g].r[k].z, blk[g].r[k].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint64_t x = fma2(widen2<T>(w[i]), l2e, nm2);
                acc[i & 1] = add2(acc[i & 1], f2(ex2_ftz(f2lo(x)), ex2_ftz(f2hi(x))));
            }
        }
        const uint64_t a = add2(acc[0], acc[1]);
        sum[g] = f2lo(a) + f2hi(a);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int g = 0; g < G; ++g) sum[g] += __shfl_xor_sync(0xffffffffu, sum[g], o);
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
        out[g] = m[g] == -NB200_INF ? St{m[g], 0.f, 0, 0} : St{m[g], sum[g], 1, 0};
}

// States of G whole items resident in `blk[g]` (load_item), every lane returning the same states.
template <int S, typename T, int NV, int G>
__device__ __forceinline__ void resident_items_state(const RegRow<NV> (&blk)[G], St (&out)[G], const Params& p) {
    if constexpr (S == NB200_LOGSUMEXP && sizeof(T) == 2) {
        lse16_rows_state<T, NV, G>(blk, out, p);
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) out[g] = row_state<S, T>(blk[g], p);
    }
}

// Loads the vectors of span item `item` (row item / nparts, chunk item % nparts) into `blk`, which
// must hold the whole item (the caller checks chunk <= 32 NV vectors); an item past the end loads
// nothing.
template <int NV, typename T>
__device__ __forceinline__ void load_item(RegRow<NV>& blk, const T* __restrict__ x, const LdgSpan& pl, int64_t item,
                                          int lane) {
    constexpr int V = Elem<T>::V;
    if (item >= pl.nitems) {
        blk.lane = lane;
        blk.nv = 0;
        return;
    }
    int64_t row;
    if (pl.nitems <= 0x7fffffff)  // 32-bit division: a 64-bit one is a long software sequence
        row = (int64_t)((uint32_t)item / (uint32_t)pl.nparts);
    else
        row = item / pl.nparts;
    const int64_t part = item - row * pl.nparts;
    const int64_t lo = pl.cb + part * pl.cc, hi = min(lo + pl.cc, pl.cb + pl.ns);
    load_block<NV, T>(blk, reinterpret_cast<const uint4*>(x + row * pl.srow + lo), 0, (int)((hi - lo) / V), lane);
}

// Warp-merged state of span item `item` (row item / nparts, chunk item % nparts). Every lane of the
// warp must call it; every lane returns the same state.
template <int S, typename T>
__device__ __forceinline__ St span_item_state(const T* __restrict__ x, const LdgSpan& pl, int64_t item, int lane,
                                              const Params& p) {
    constexpr int V = Elem<T>::V;
    constexpr bool kFast = S == NB200_LOGSUMEXP && sizeof(T) == 2;
    const int64_t row = item / pl.nparts, part = item - row * pl.nparts;
    const int64_t lo = pl.cb + part * pl.cc, hi = min(lo + pl.cc, pl.cb + pl.ns);
    const uint4* base = reinterpret_cast<const uint4*>(x + row * pl.srow + lo);
    const int nvec = (int)((hi - lo) / V);
    St run = empty_state();
    for (int v0 = 0; v0 < nvec; v0 += 32 * kSpanNV) {
        RegRow<kSpanNV> blk;
        load_block<kSpanNV, T>(blk, base, v0, nvec, lane);
        if constexpr (kFast)
            lse16_block<T>(blk, run, p);
        else
            run = merge_fast<S>(run, lane_state<S, T>(blk, p), p);
    }
    return warp_merge<S>(run, lane, p);
}

}  // namespace nb200
