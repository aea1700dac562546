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

// Warp-merged state of vectors [v0, v1) of a column span starting at `base`, folded in sub-blocks of
// 32 x kSpanNV vectors. Every lane of the warp must call it; every lane returns the same state.
template <int S, typename T>
__device__ __forceinline__ St span_range_state(const uint4* base, int v0, int v1, int lane, const Params& p) {
    constexpr bool kFast = S == NB200_LOGSUMEXP && sizeof(T) == 2;
    St run = empty_state();
    for (int v = v0; v < v1; v += 32 * kSpanNV) {
        RegRow<kSpanNV> blk;
        load_block<kSpanNV, T>(blk, base, v, v1, lane);
        if constexpr (kFast)
            lse16_block<T>(blk, run, p);
        else
            run = merge_fast<S>(run, lane_state<S, T>(blk, p), p);
    }
    return warp_merge<S>(run, lane, p);
}

// First vector and vector count of span item `item` (row item / nparts, chunk item % nparts).
template <typename T>
__device__ __forceinline__ const uint4* span_item_base(const T* __restrict__ x, const LdgSpan& pl, int64_t item,
                                                       int& nvec) {
    constexpr int V = Elem<T>::V;
    const int64_t row = item / pl.nparts, part = item - row * pl.nparts;
    const int64_t lo = pl.cb + part * pl.cc, hi = min(lo + pl.cc, pl.cb + pl.ns);
    nvec = (int)((hi - lo) / V);
    return reinterpret_cast<const uint4*>(x + row * pl.srow + lo);
}

// Warp-merged state of span item `item`. Every lane of the warp must call it; every lane returns
// the same state.
template <int S, typename T>
__device__ __forceinline__ St span_item_state(const T* __restrict__ x, const LdgSpan& pl, int64_t item, int lane,
                                              const Params& p) {
    int nvec;
    const uint4* base = span_item_base<T>(x, pl, item, nvec);
    return span_range_state<S, T>(base, 0, nvec, lane, p);
}

// Warps that fold one span item. One, unless the items are too few to occupy the GPU: then the 4
// warps of a CTA share an item, each folding a contiguous quarter of its columns (at least one
// sub-block each), and their 4 states merge in column order. The rule depends only on the item
// count, the item width and the SM count, so every kernel that folds the same items (the split
// plan's partial fold, the exchange's fused fold) decomposes them the same way and produces the
// same states bit for bit. Resident warps are counted at 6 CTAs of kLdgThreads per SM. Measured on
// B200 with bf16 16384-column chunks (split plan, interleaved A/B): 1024 items 15.7 -> 12.9 µs;
// 2 warps per item at 2048 items neutral (20.0 vs 19.8 µs), so it is not used; at 4096 or more
// items sharing costs more than the last uneven round of whole items (62.8 vs 51.3 µs at 8192).
inline int span_item_warps(int64_t nitems, int64_t nvec, int sms) {
    const int64_t slots = (int64_t)sms * 6 * (kLdgThreads / 32);
    return (nvec >= 4 * 32 * kSpanNV && nitems * 4 <= slots + slots / 4) ? 4 : 1;
}

// Folds every span item with W warps per item (W = 2 or 4; the rule above uses 4) and hands each item's state to
// sink(item, state), called by one thread per item. A CTA takes (kLdgThreads / 32) / W items at a
// time; warp w folds part w % W of item w / W, lane 0 leaves its state in shared memory, and after
// one barrier thread t merges item t's W states left to right. The shared states alternate
// between two halves, so one barrier per round suffices. Every thread of the CTA must call it.
template <int S, typename T, int W, class Sink>
__device__ __forceinline__ void span_items_shared(const T* __restrict__ x, const LdgSpan& pl, const Params& p,
                                                  Sink&& sink) {
    constexpr int kPer = (kLdgThreads / 32) / W;
    __shared__ float4 part_state[2][kLdgThreads / 32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int half = 0;
    for (int64_t unit = blockIdx.x; unit * kPer < pl.nitems; unit += gridDim.x, half ^= 1) {
        const int64_t item = unit * kPer + warp / W;
        if (item < pl.nitems) {
            int nvec;
            const uint4* base = span_item_base<T>(x, pl, item, nvec);
            int64_t a, b;
            split_range(nvec, W, warp % W, a, b);
            const St w = span_range_state<S, T>(base, (int)a, (int)b, lane, p);
            if (lane == 0)
                part_state[half][warp] = make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status));
        }
        __syncthreads();
        if (threadIdx.x < kPer && unit * kPer + threadIdx.x < pl.nitems) {
            St s = empty_state();
#pragma unroll
            for (int i = 0; i < W; ++i) {
                const float4 v = part_state[half][threadIdx.x * W + i];
                s = merge_fast<S>(s, St{v.x, v.y, __float_as_int(v.z), __float_as_int(v.w)}, p);
            }
            sink(unit * kPer + threadIdx.x, s);
        }
    }
}

}  // namespace nb200
