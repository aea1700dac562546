// Register-row kernel for contiguous rows of 1-8 KB on sm_100a.
//
// One warp per row: all of the row's 16-byte vectors are loaded with plain vector loads at once
// (NV per lane, every load in flight together), then the fused Op (row_ops.cuh) runs on the
// registers -- both passes of the fold and the readout store -- so the row is read from HBM
// once with nothing staged. Rows go to warps round-robin, so the rows being read at any moment
// form one contiguous band of the tensor. Read-heavy rows of this size reach more of HBM's
// bandwidth this way than with per-warp bulk copies into shared memory (measured on B200: a
// plain-load reader sustains ~5.8 TB/s on a 67 MB read, the bulk-copy ring ~4.1 TB/s).
#include <type_traits>

#include "fastmath.cuh"
#include "launch.h"
#include "row_ops.cuh"

namespace nb200 {

constexpr int kLdgThreads = 128;

// CTA size per Op: RMSNorm stages gamma (ncols values) into every CTA's shared memory, so fewer,
// larger CTAs do less of that (measured 47.3 vs 48.9 us for bf16 [16384, 4096]); the others keep
// the finer 4-warp CTAs (softmax fp32 [8192, 2048]: 26.7 vs 27.6 us).
template <class Op> struct LdgThreads { static constexpr int value = kLdgThreads; };
template <typename T> struct LdgThreads<RmsOp<T>> { static constexpr int value = 256; };
// The softmax readout and the folds are held to 5 CTAs per SM worth of registers (at most 102 per
// thread): 20 resident rows per SM instead of 16 (fp32 [8192, 2048]: softmax 23.7 vs 26.6 us,
// logsumexp 14.4 vs 15.8 us, no spills). softcap_lse and variance would spill under the cap and
// keep the compiler's choice, as do L2 and RMSNorm.
template <class Op> struct LdgMinBlocks { static constexpr int value = 1; };
template <typename T> struct LdgMinBlocks<SoftmaxOp<T>> { static constexpr int value = 5; };
template <int S, typename T> struct LdgMinBlocks<FoldOp<S, T>> {
    static constexpr int value = (S == NB200_SOFTCAP_LSE || S == NB200_VARIANCE) ? 1 : 5;
};

template <typename T, class Op, int NV, int kThreads = LdgThreads<Op>::value>
__global__ void __launch_bounds__(kThreads, LdgMinBlocks<Op>::value)
    ldg_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t srow, Op op) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smem[];
    op.prologue(smem);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
    const int64_t GW = (int64_t)gridDim.x * (kThreads / 32);
    for (int64_t r = gw; r < rows; r += GW) {
        RegRow<NV> rr;
        rr.nv = op.nv;
        rr.lane = lane;
        const uint4* row = reinterpret_cast<const uint4*>(x + r * srow);
#pragma unroll
        for (int k = 0; k < NV; ++k)
            rr.r[k] = (lane + 32 * k < op.nv) ? ld_stream(row + lane + 32 * k) : make_uint4(0u, 0u, 0u, 0u);
        op.row(rr, r, lane, smem);
    }
}

template <typename T, class Op, int NV>
int launch_ldg_nv(const T* x, int64_t rows, int64_t srow, const Op& op, uint32_t smem, cudaStream_t st,
                  const char* what) {
    constexpr int kThreads = LdgThreads<Op>::value;
    auto k = ldg_rows_kernel<T, Op, NV>;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, smem) != cudaSuccess || occ < 1) occ = 1;
    const int64_t need = (rows + kThreads / 32 - 1) / (kThreads / 32);
    const int g = (int)std::min<int64_t>(need, (int64_t)sm_count() * occ);
    launch_pdl(k, (unsigned)std::max(g, 1), kThreads, smem, st, x, rows, srow, op);
    count_launch();
    return finish_launch(what);
}

template <typename T, class Op>
int launch_ldg_rows(const T* x, int64_t rows, int64_t srow, const Op& op, uint32_t smem, cudaStream_t st,
                    const char* what) {
    if (op.nv <= 32 * 4) return launch_ldg_nv<T, Op, 4>(x, rows, srow, op, smem, st, what);
    return launch_ldg_nv<T, Op, 16>(x, rows, srow, op, smem, st, what);
}

// ------------------------------------------------------------------ column spans
// Split-plan chunks, and rows too long for one warp's registers: a warp folds one item (row,
// column span) in sub-blocks of 32 x kSpanNV vectors (4 KB) loaded into registers at once. Per
// lane a running fold state absorbs each sub-block; at the item's end the 32 lane states merge in
// a fixed tree (lower lane on the left). Measured on B200 (bf16 [512, 262144], 16K-column
// chunks): single 4 KB blocks with ~2x the resident warps beat double-buffered blocks, 54.9 us
// against 70.8 us.
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

template <typename T>
__device__ __forceinline__ void lse16_block(const RegRow<kSpanNV>& blk, St& run, const Params& p) {
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
    for (int k = 0; k < kSpanNV; ++k) {
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

template <int S, typename T>
__global__ void __launch_bounds__(kLdgThreads) ldg_span_kernel(const T* __restrict__ x, LdgSpan pl, Params p,
                                                               nb200_state* __restrict__ states, T* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    constexpr int V = Elem<T>::V;
    constexpr bool kFast = S == NB200_LOGSUMEXP && sizeof(T) == 2;
    const int lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (kLdgThreads / 32) + (threadIdx.x >> 5);
    const int64_t GW = (int64_t)gridDim.x * (kLdgThreads / 32);
    for (int64_t item = gw; item < pl.nitems; item += GW) {
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
        const St w = warp_merge<S>(run, lane, p);
        if (lane == 0) {
            if (pl.finalize) out[row] = Elem<T>::from_f(finalize<S>(w, p));
            else reinterpret_cast<float4*>(states)[item] =
                     make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status));
        }
    }
}

template <typename T>
int launch_ldg_span(int sk, const Params& p, const T* x, int64_t rows, int64_t cb, int64_t ns, int64_t srow,
                    int64_t cc, int64_t nparts, nb200_state* states, T* out, int finalize, cudaStream_t st) {
    LdgSpan pl{rows, srow, cb, ns, cc, nparts, rows * nparts, finalize};
    int rc = NB200_OK;
    auto go = [&](auto k) {
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kLdgThreads, 0) != cudaSuccess || occ < 1) occ = 1;
        const int64_t need = (pl.nitems + kLdgThreads / 32 - 1) / (kLdgThreads / 32);
        const int g = (int)std::min<int64_t>(need, (int64_t)sm_count() * occ);
        launch_pdl(k, (unsigned)std::max(g, 1), kLdgThreads, 0, st, x, pl, p, states, out);
        count_launch();
        rc = finish_launch(finalize ? "nb200_fold" : "nb200_fold_partial");
    };
    switch (sk) {
#define X(S) case S: go(ldg_span_kernel<S, T>); break;
        X(NB200_LOGSUMEXP) X(NB200_LSE_BIASED) X(NB200_LSE_SCALED) X(NB200_SOFTCAP_LSE) X(NB200_STABLE_L2)
        X(NB200_LINEAR_ATTN) X(NB200_DECAY_RENORM) X(NB200_SUMSQ_DIV) X(NB200_RMSNORM_MAX)
#undef X
        default: return 0;
    }
    return rc ? rc : 1;
}
template int launch_ldg_span<float>(int, const Params&, const float*, int64_t, int64_t, int64_t, int64_t, int64_t,
                                    int64_t, nb200_state*, float*, int, cudaStream_t);
template int launch_ldg_span<__nv_bfloat16>(int, const Params&, const __nv_bfloat16*, int64_t, int64_t, int64_t,
                                            int64_t, int64_t, int64_t, nb200_state*, __nv_bfloat16*, int,
                                            cudaStream_t);
template int launch_ldg_span<__half>(int, const Params&, const __half*, int64_t, int64_t, int64_t, int64_t, int64_t,
                                     int64_t, nb200_state*, __half*, int, cudaStream_t);

#define NB200_LDG_INST(T)                                                                                          \
    template int launch_ldg_rows<T, SoftmaxOp<T>>(const T*, int64_t, int64_t, const SoftmaxOp<T>&, uint32_t,        \
                                                  cudaStream_t, const char*);                                      \
    template int launch_ldg_rows<T, L2Op<T>>(const T*, int64_t, int64_t, const L2Op<T>&, uint32_t, cudaStream_t,    \
                                             const char*);                                                         \
    template int launch_ldg_rows<T, RmsOp<T>>(const T*, int64_t, int64_t, const RmsOp<T>&, uint32_t, cudaStream_t,  \
                                              const char*);
#define NB200_LDG_FOLD(S, T)                                                                                      \
    template int launch_ldg_rows<T, FoldOp<S, T>>(const T*, int64_t, int64_t, const FoldOp<S, T>&, uint32_t,      \
                                                  cudaStream_t, const char*);
#define NB200_LDG_FOLDS(T)                                                                                        \
    NB200_LDG_FOLD(NB200_LOGSUMEXP, T) NB200_LDG_FOLD(NB200_LSE_BIASED, T) NB200_LDG_FOLD(NB200_LSE_SCALED, T)    \
    NB200_LDG_FOLD(NB200_SOFTCAP_LSE, T) NB200_LDG_FOLD(NB200_STABLE_L2, T) NB200_LDG_FOLD(NB200_LINEAR_ATTN, T)  \
    NB200_LDG_FOLD(NB200_DECAY_RENORM, T) NB200_LDG_FOLD(NB200_SUMSQ_DIV, T) NB200_LDG_FOLD(NB200_RMSNORM_MAX, T)  \
    NB200_LDG_FOLD(NB200_VARIANCE, T) NB200_LDG_FOLD(NB200_STD, T)

NB200_LDG_INST(float)
NB200_LDG_INST(__nv_bfloat16)
NB200_LDG_INST(__half)
NB200_LDG_FOLDS(float)
NB200_LDG_FOLDS(__nv_bfloat16)
NB200_LDG_FOLDS(__half)

}  // namespace nb200
