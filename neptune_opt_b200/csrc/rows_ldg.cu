// Register-row kernel for contiguous rows of 1-8 KB on sm_100a.
//
// One warp per row: all of the row's 16-byte vectors are loaded with plain vector loads at once
// (NV per lane, every load in flight together), then the fused Op (row_ops.cuh) runs on the
// registers -- both passes of the fold and the readout store -- so the row is read from HBM
// once with nothing staged. Rows go to warps round-robin, so the rows being read at any moment
// form one contiguous band of the tensor. Read-heavy rows of this size reach more of HBM's
// bandwidth this way than with per-warp bulk copies into shared memory (measured on B200: a
// plain-load reader sustains ~5.8 TB/s on a 67 MB read, the bulk-copy ring ~4.1 TB/s).
#include <atomic>
#include <type_traits>

#include "fastmath.cuh"
#include "launch.h"
#include "row_ops.cuh"
#include "span.cuh"

namespace nb200 {


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

// A row of exactly 32 * NV vectors: every lane holds NV of them, so loads and Op passes run with no
// per-vector bounds test (the common power-of-two widths: fp32 2048, bf16 4096, ...).
template <int NV>
struct RegRowFull {
    uint4 r[NV];
    static constexpr int nv = 32 * NV;
    static constexpr bool kRegisters = true;  // the whole row, lane-strided, in r[]
    int lane;
    template <class F>
    __device__ __forceinline__ void for_each(F&& f) const {
#pragma unroll
        for (int k = 0; k < NV; ++k) f(r[k], lane + 32 * k);
    }
};

template <typename T, class Op, int NV, bool kFull, int kThreads = LdgThreads<Op>::value>
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
        const uint4* row = reinterpret_cast<const uint4*>(x + r * srow);
        if constexpr (kFull) {
            RegRowFull<NV> rr;
            rr.lane = lane;
#pragma unroll
            for (int k = 0; k < NV; ++k) rr.r[k] = ld_stream(row + lane + 32 * k);
            op.row(rr, r, lane, smem);
        } else {
            RegRow<NV> rr;
            rr.nv = op.nv;
            rr.lane = lane;
#pragma unroll
            for (int k = 0; k < NV; ++k)
                rr.r[k] = (lane + 32 * k < op.nv) ? ld_stream(row + lane + 32 * k) : make_uint4(0u, 0u, 0u, 0u);
            op.row(rr, r, lane, smem);
        }
    }
}

// Grid: enough warps for every row when they fit in one wave of resident warps; otherwise as few
// warps as keep the same number of waves, so that every warp folds the same number of rows (to
// within one). Measured on B200 with logsumexp fp32 [8192, 2048]: 2732 warps taking 3 rows each
// against 2960 resident warps, 740 of them taking 2 rows, 11.9 vs 12.8 us per launch.
template <typename T, class Op, int NV, bool kFull>
int launch_ldg_nv(const T* x, int64_t rows, int64_t srow, const Op& op, uint32_t smem, cudaStream_t st,
                  const char* what) {
    constexpr int kThreads = LdgThreads<Op>::value;
    constexpr int64_t kWarps = kThreads / 32;
    auto k = ldg_rows_kernel<T, Op, NV, kFull>;
    static std::atomic<int64_t> cached{-1};  // (smem << 8) | occupancy of the last query
    int occ = 0;
    const int64_t c = cached.load(std::memory_order_relaxed);
    if (c >= 0 && (uint32_t)(c >> 8) == smem) {
        occ = (int)(c & 255);
    } else {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kThreads, smem) != cudaSuccess || occ < 1) occ = 1;
        cached.store(((int64_t)smem << 8) | std::min(occ, 255), std::memory_order_relaxed);
    }
    const int64_t slots = (int64_t)sm_count() * occ * kWarps;
    const int64_t waves = (rows + slots - 1) / slots;
    const int64_t warps = (rows + waves - 1) / std::max<int64_t>(waves, 1);
    const int g = (int)std::max<int64_t>((warps + kWarps - 1) / kWarps, 1);
    launch_pdl(k, (unsigned)g, kThreads, smem, st, x, rows, srow, op);
    count_launch();
    return finish_launch(what);
}

// Full-row instantiations where they keep every value in registers: fp32 rows, and the 16-bit
// RMSNorm / L2 readouts (no register cap). The capped 16-bit folds and softmax would spill with all
// 128 values of a lane unpacked at once, so they keep the bounds-tested form.
template <typename T, class Op> struct LdgFull { static constexpr bool value = sizeof(T) == 4; };
template <typename T> struct LdgFull<T, RmsOp<T>> { static constexpr bool value = true; };
template <typename T> struct LdgFull<T, L2Op<T>> { static constexpr bool value = true; };

template <typename T, class Op>
int launch_ldg_rows(const T* x, int64_t rows, int64_t srow, const Op& op, uint32_t smem, cudaStream_t st,
                    const char* what) {
    constexpr bool kFull = LdgFull<T, Op>::value;
    if (op.nv <= 32 * 4) {
        if (kFull && op.nv == 32 * 4) return launch_ldg_nv<T, Op, 4, kFull>(x, rows, srow, op, smem, st, what);
        return launch_ldg_nv<T, Op, 4, false>(x, rows, srow, op, smem, st, what);
    }
    if (kFull && op.nv == 32 * 16) return launch_ldg_nv<T, Op, 16, kFull>(x, rows, srow, op, smem, st, what);
    return launch_ldg_nv<T, Op, 16, false>(x, rows, srow, op, smem, st, what);
}

// ------------------------------------------------------------------ column spans (span.cuh)
template <int S, typename T>
__device__ __forceinline__ void span_store(const LdgSpan& pl, int64_t item, const St& w, const Params& p,
                                           nb200_state* __restrict__ states, T* __restrict__ out) {
    if (pl.finalize) out[item / pl.nparts] = Elem<T>::from_f(finalize<S>(w, p));
    else reinterpret_cast<float4*>(states)[item] = make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status));
}

// How a span kernel holds its items:
//   kSpanStream   items of any width, folded in 4 KB sub-blocks (span_item_state);
//   G = 1, 2, 4   every item fits 32 x kSpanNV / G vectors (chunks of at most 2048 / G 16-bit or
//                 1024 / G fp32 columns): a warp loads G consecutive items into one 4 KB register
//                 block and each is a resident row whose state is formed the way the reference
//                 forms one chunk's (resident_items_state: the producer reduced across the warp
//                 first, every term against it, one warp sum; no per-lane repair and no 32-state
//                 merge tree), the G items' warp reductions interleaved.
//   G = -4        too few wide items to occupy the GPU (span_item_warps): the 4 warps of a CTA
//                 share each item (span_items_shared).
constexpr int kSpanStream = 0;

template <int S, typename T, int G>
__global__ void __launch_bounds__(kLdgThreads) ldg_span_kernel(const T* __restrict__ x, LdgSpan pl, Params p,
                                                               nb200_state* __restrict__ states, T* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (kLdgThreads / 32) + (threadIdx.x >> 5);
    const int64_t GW = (int64_t)gridDim.x * (kLdgThreads / 32);
    if constexpr (G < 0) {
        span_items_shared<S, T, -G>(x, pl, p, [&](int64_t item, const St& w) { span_store<S, T>(pl, item, w, p, states, out); });
    } else if constexpr (G == kSpanStream) {
        for (int64_t item = gw; item < pl.nitems; item += GW) {
            const St w = span_item_state<S, T>(x, pl, item, lane, p);
            if (lane == 0) span_store<S, T>(pl, item, w, p, states, out);
        }
    } else {
        constexpr int NV = kSpanNV / G;
        for (int64_t item = gw * G; item < pl.nitems; item += GW * G) {
            RegRow<NV> blk[G];
#pragma unroll
            for (int g = 0; g < G; ++g) load_item<NV, T>(blk[g], x, pl, item + g, lane);
            St w[G];
            resident_items_state<S, T, NV, G>(blk, w, p);
#pragma unroll
            for (int g = 0; g < G; ++g)
                if (lane == g && item + g < pl.nitems) span_store<S, T>(pl, item + g, w[g], p, states, out);
        }
    }
}

template <typename T>
int launch_ldg_span(int sk, const Params& p, const T* x, int64_t rows, int64_t cb, int64_t ns, int64_t srow,
                    int64_t cc, int64_t nparts, nb200_state* states, T* out, int finalize, cudaStream_t st) {
    LdgSpan pl{rows, srow, cb, ns, cc, nparts, rows * nparts, finalize};
    const int64_t nvec = cc / Elem<T>::V;  // vectors of the widest item
    int group = nvec <= 32 * kSpanNV / 4 ? 4 : nvec <= 32 * kSpanNV / 2 ? 2 : nvec <= 32 * kSpanNV ? 1
                                                                                                : kSpanStream;
    if (group == kSpanStream) group = -span_item_warps(pl.nitems, nvec, sm_count());  // -1: one warp per item
    int rc = NB200_OK;
    auto go = [&](auto k) {
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kLdgThreads, 0) != cudaSuccess || occ < 1) occ = 1;
        // warps wanted: one per G items, one per item, or W per item
        const int64_t warps = group > 1 ? (pl.nitems + group - 1) / group : pl.nitems * (group < 0 ? -group : 1);
        const int64_t need = (warps + kLdgThreads / 32 - 1) / (kLdgThreads / 32);
        const int g = (int)std::min<int64_t>(need, (int64_t)sm_count() * occ);
        launch_pdl(k, (unsigned)std::max(g, 1), kLdgThreads, 0, st, x, pl, p, states, out);
        count_launch();
        rc = finish_launch(finalize ? "nb200_fold" : "nb200_fold_partial");
    };
    switch (sk) {
#define X(S)                                                                                   \
    case S:                                                                                    \
        if (group == -4) go(ldg_span_kernel<S, T, -4>);                                        \
        else if (group == 4) go(ldg_span_kernel<S, T, 4>);                                     \
        else if (group == 2) go(ldg_span_kernel<S, T, 2>);                                     \
        else if (group == 1) go(ldg_span_kernel<S, T, 1>);                                     \
        else go(ldg_span_kernel<S, T, kSpanStream>);                                           \
        break;
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

// ------------------------------------------------------------------ cluster rows
// Few, very wide rows in ONE launch: a thread-block cluster of C CTAs per row (up to 16, one
// cluster per row), each CTA folding a contiguous column range of the row with its 8 warps (4 KB
// register sub-blocks and a running lane state, as the span kernel), its warps' states merged in
// ascending warp order. The C CTA states then meet in the leader CTA's shared memory through
// distributed shared memory (st.shared::cluster after mapa), one cluster barrier, and the leader
// merges them in ascending CTA rank -- the split plan's certified order with the CTA ranges as
// chunks -- and finalises. No scratch in global memory and no second launch; a single row is
// spread over C SMs instead of one.
constexpr int kClThreads = 256;
constexpr int kClWarps = kClThreads / 32;
constexpr int kClMax = 16;

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
    uint32_t n;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(n));
    return n;
}
__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t c;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(c));
    return c;
}
// Address of `p` (this CTA's shared memory) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* p, uint32_t rank) {
    uint32_t local = static_cast<uint32_t>(__cvta_generic_to_shared(p)), remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
    return remote;
}
__device__ __forceinline__ void dsmem_st4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}
__device__ __forceinline__ void dsmem_st1(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// [v0, v1) of n vectors for part i of k (contiguous, ascending, sizes differing by at most one).

template <int S, typename T>
__global__ void __launch_bounds__(kClThreads) cluster_fold_kernel(const T* __restrict__ x, int64_t rows,
                                                                  int64_t nvec, int64_t srow, Params p,
                                                                  T* __restrict__ out) {
    constexpr bool kFast = S == NB200_LOGSUMEXP && sizeof(T) == 2;
    __shared__ float4 cta_state[kClMax];
    __shared__ float4 warp_state[kClWarps];
    pdl_wait();
    pdl_trigger();
    const uint32_t crank = cluster_rank(), csize = cluster_size();
    const int64_t row = cluster_index();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (row < rows) {
        int64_t c0, c1, w0, w1;
        split_range(nvec, csize, crank, c0, c1);
        split_range(c1 - c0, kClWarps, warp, w0, w1);
        const uint4* base = reinterpret_cast<const uint4*>(x + row * srow) + c0 + w0;
        const int n = (int)(w1 - w0);
        St run = empty_state();
        for (int v0 = 0; v0 < n; v0 += 32 * kSpanNV) {
            RegRow<kSpanNV> blk;
            load_block<kSpanNV, T>(blk, base, v0, n, lane);
            if constexpr (kFast)
                lse16_block<T>(blk, run, p);
            else
                run = merge_fast<S>(run, lane_state<S, T>(blk, p), p);
        }
        const St w = warp_merge<S>(run, lane, p);
        if (lane == 0) warp_state[warp] = make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        St c = empty_state();
        if (row < rows) {
            for (int i = 0; i < kClWarps; ++i) {
                const float4 v = warp_state[i];
                c = merge_fast<S>(c, St{v.x, v.y, __float_as_int(v.z), __float_as_int(v.w)}, p);
            }
        }
        dsmem_st4(dsmem_addr(&cta_state[crank], 0), __float_as_uint(c.m), __float_as_uint(c.acc), (uint32_t)c.seen,
                  (uint32_t)c.status);
    }
    cluster_sync();
    if (crank == 0 && threadIdx.x == 0 && row < rows) {
        St s = empty_state();
        for (uint32_t i = 0; i < csize; ++i) {
            const float4 v = cta_state[i];
            s = merge_fast<S>(s, St{v.x, v.y, __float_as_int(v.z), __float_as_int(v.w)}, p);
        }
        out[row] = Elem<T>::from_f(finalize<S>(s, p));
    }
}

// RMSNorm of few, very wide rows: each CTA of the row's cluster keeps its column range in
// registers (kClRV vectors per thread), forms its sum of squares with the RMSNorm stages' rounding
// (every square and add rounded, in a fixed order: thread, warp tree, warps ascending), writes it
// into every cluster CTA's shared memory, and after one cluster barrier every CTA adds the C
// partial sums in ascending rank (the same total everywhere), forms mean and scale and writes its
// own range of y = round(round(x * scale) * gamma).
constexpr int kClRV = 8;

template <typename T>
__global__ void __launch_bounds__(kClThreads) cluster_rms_kernel(const T* __restrict__ x, const T* __restrict__ gamma,
                                                                 int64_t rows, int64_t nvec, int64_t srow, float eps,
                                                                 float count, T* __restrict__ y) {
    constexpr int V = Elem<T>::V;
    __shared__ float part[kClMax];
    __shared__ float warp_sum_s[kClWarps];
    pdl_wait();
    pdl_trigger();
    const uint32_t crank = cluster_rank(), csize = cluster_size();
    const int64_t row = cluster_index();
    const bool live = row < rows;
    int64_t c0, c1;
    split_range(nvec, csize, crank, c0, c1);
    const int64_t n = c1 - c0;
    const uint4* xr = reinterpret_cast<const uint4*>(x + row * srow) + c0;
    const uint4* gr = reinterpret_cast<const uint4*>(gamma) + c0;
    uint4 v[kClRV];
#pragma unroll
    for (int k = 0; k < kClRV; ++k) {
        const int64_t j = threadIdx.x + (int64_t)kClThreads * k;
        v[k] = (live && j < n) ? ld_stream(xr + j) : make_uint4(0u, 0u, 0u, 0u);
    }
    unsigned long long acc[2] = {0ull, 0ull};
#pragma unroll
    for (int k = 0; k < kClRV; ++k) {
        if constexpr (sizeof(T) == 2) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const unsigned long long f = Word<T>::unpack(word(v[k], i));
                acc[i & 1] = add_f32x2(acc[i & 1], mul_f32x2(f, f));
            }
        } else {
            const unsigned long long a = pk(__uint_as_float(v[k].x), __uint_as_float(v[k].y));
            const unsigned long long b = pk(__uint_as_float(v[k].z), __uint_as_float(v[k].w));
            acc[0] = add_f32x2(acc[0], mul_f32x2(a, a));
            acc[1] = add_f32x2(acc[1], mul_f32x2(b, b));
        }
    }
    const unsigned long long a = add_f32x2(acc[0], acc[1]);
    const float t = warp_sum(__fadd_rn(lo_f(a), hi_f(a)));
    if ((threadIdx.x & 31) == 0) warp_sum_s[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x < csize) {  // thread r sends this CTA's partial sum to cluster CTA r
        float cta = 0.f;
        for (int i = 0; i < kClWarps; ++i) cta = __fadd_rn(cta, warp_sum_s[i]);
        dsmem_st1(dsmem_addr(&part[crank], threadIdx.x), cta);
    }
    cluster_sync();
    if (!live) return;
    float total = 0.f;
    for (uint32_t i = 0; i < csize; ++i) total = __fadd_rn(total, part[i]);
    const float mean = __fdiv_rn(total, count);
    const float scale = __frsqrt_rn(__fadd_rn(mean, eps));
    const unsigned long long sc = pk(scale, scale);
    uint4* yr = reinterpret_cast<uint4*>(y + row * (nvec * V)) + c0;
#pragma unroll
    for (int k = 0; k < kClRV; ++k) {
        const int64_t j = threadIdx.x + (int64_t)kClThreads * k;
        if (j >= n) continue;
        const uint4 g = __ldg(gr + j);
        uint4 o;
        if constexpr (sizeof(T) == 2) {
            o.x = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(v[k].x), sc)), g.x);
            o.y = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(v[k].y), sc)), g.y);
            o.z = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(v[k].z), sc)), g.z);
            o.w = Word<T>::mul_pair(Word<T>::round_pair(mul_f32x2(Word<T>::unpack(v[k].w), sc)), g.w);
        } else {
            const unsigned long long p0 = mul_f32x2(mul_f32x2(pk(__uint_as_float(v[k].x), __uint_as_float(v[k].y)), sc),
                                                    pk(__uint_as_float(g.x), __uint_as_float(g.y)));
            const unsigned long long p1 = mul_f32x2(mul_f32x2(pk(__uint_as_float(v[k].z), __uint_as_float(v[k].w)), sc),
                                                    pk(__uint_as_float(g.z), __uint_as_float(g.w)));
            o = make_uint4((uint32_t)p0, (uint32_t)(p0 >> 32), (uint32_t)p1, (uint32_t)(p1 >> 32));
        }
        st_stream(yr + j, o);
    }
}

// Cluster size for `rows` rows: as many CTAs per row as keep every SM busy, at most 16 (8 when the
// hardware cannot place 16-CTA clusters of these 256-thread kernels), at least 2.
template <typename K>
static int cluster_ctas(K kernel, int64_t rows) {
    static std::atomic<int> max16{-1};  // one answer per kernel signature: a property of the device
    int m = max16.load(std::memory_order_relaxed);
    if (m < 0) {
        m = 0;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(16);
            cfg.blockDim = dim3(kClThreads);
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 16;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            m = (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) == cudaSuccess && n > 0) ? 1 : 0;
        }
        cudaGetLastError();
        max16.store(m, std::memory_order_relaxed);
    }
    // About 1.75 CTAs per SM in all, in power-of-two clusters: measured on B200 (logsumexp fp32,
    // 16.8 MB, graph-timed) the best cluster size gave 256-296 CTAs for 16 to 128 rows -- [128,
    // 32768] 7.9 µs at 2 CTAs per row against 9.7 at 4; [64, 65536] 8.0 at 4 against 9.1 at 2;
    // [32, 131072] 8.2 at 8 against 9.4 at 4 -- and never fewer than 2 per row ([256, 16384] 9.1
    // µs at 2, 13.0 at 4). Non-power-of-two clusters schedule worse ([64, 65536] at 7: 12.2 µs).
    const int64_t want = std::min<int64_t>((7 * (int64_t)sm_count() / 4) / std::max<int64_t>(rows, 1), m ? 16 : 8);
    int c = 2;
    while (2 * c <= want) c *= 2;
    return c;
}

template <typename K, typename... Args>
static int launch_cluster(K kernel, int64_t rows, int csize, cudaStream_t st, const char* what, Args... args) {
    if (csize > 8 && cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
        cudaGetLastError();
        set_error("%s: %d-CTA clusters are not available", what, csize);
        return NB200_ERR_LAUNCH;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * csize));
    cfg.blockDim = dim3(kClThreads);
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)csize;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    // programmatic dependent launch, as the other kernels: the launch overlaps the previous
    // kernel's tail, and the kernel's griddepcontrol.wait holds its reads until that kernel is done
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (e != cudaSuccess) {
        cudaGetLastError();
        set_error("%s: cluster launch failed: %s", what, cudaGetErrorString(e));
        return NB200_ERR_LAUNCH;
    }
    count_launch();
    return finish_launch(what);
}

template <typename T>
int launch_cluster_fold(int sk, const Params& p, const T* x, int64_t rows, int64_t ncols, int64_t srow, T* out,
                        int csize_request, cudaStream_t st) {
    const int64_t nvec = ncols / Elem<T>::V;
    int rc = NB200_OK;
    auto go = [&](auto k) {
        const int c = csize_request > 0 ? std::min(csize_request, kClMax) : cluster_ctas(k, rows);
        rc = launch_cluster(k, rows, c, st, "nb200_fold (cluster)", x, rows, nvec, srow, p, out);
    };
    switch (sk) {
#define X(S) case S: go(cluster_fold_kernel<S, T>); break;
        X(NB200_LOGSUMEXP) X(NB200_LSE_BIASED) X(NB200_LSE_SCALED) X(NB200_SOFTCAP_LSE) X(NB200_STABLE_L2)
        X(NB200_LINEAR_ATTN) X(NB200_DECAY_RENORM) X(NB200_SUMSQ_DIV) X(NB200_RMSNORM_MAX)
#undef X
        default: return 0;
    }
    return rc ? rc : 1;
}

template <typename T>
int launch_cluster_rms(const T* x, const T* gamma, int64_t rows, int64_t ncols, int64_t srow, float eps, T* y,
                       int csize_request, cudaStream_t st) {
    const int64_t nvec = ncols / Elem<T>::V;
    auto k = cluster_rms_kernel<T>;
    const int c = csize_request > 0 ? std::min(csize_request, kClMax) : cluster_ctas(k, rows);
    if ((nvec + c - 1) / c > (int64_t)kClThreads * kClRV) return 0;  // a CTA's range exceeds its registers
    const int rc = launch_cluster(k, rows, c, st, "nb200_rms_norm (cluster)", x, gamma, rows, nvec, srow, eps,
                                  (float)ncols, y);
    return rc ? rc : 1;
}

template int launch_cluster_fold<float>(int, const Params&, const float*, int64_t, int64_t, int64_t, float*, int,
                                        cudaStream_t);
template int launch_cluster_fold<__nv_bfloat16>(int, const Params&, const __nv_bfloat16*, int64_t, int64_t, int64_t,
                                                __nv_bfloat16*, int, cudaStream_t);
template int launch_cluster_fold<__half>(int, const Params&, const __half*, int64_t, int64_t, int64_t, __half*, int,
                                         cudaStream_t);
template int launch_cluster_rms<float>(const float*, const float*, int64_t, int64_t, int64_t, float, float*, int,
                                       cudaStream_t);
template int launch_cluster_rms<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, int64_t, int64_t, int64_t,
                                               float, __nv_bfloat16*, int, cudaStream_t);
template int launch_cluster_rms<__half>(const __half*, const __half*, int64_t, int64_t, int64_t, float, __half*, int,
                                        cudaStream_t);

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
