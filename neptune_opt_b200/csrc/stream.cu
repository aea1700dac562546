// Streaming (bulk-copy staged) kernels for contiguous, 16-byte-aligned rows on sm_100a.
//
// rows_kernel: every warp owns a ring of S shared-memory stages, each holding R whole rows. Lane 0
// refills a stage with cp.async.bulk as soon as the warp has read it, so S-1 stages per warp are
// in flight while the warp computes on the third; the row is read from HBM exactly once and every
// further pass (max, sum, readout) reads shared memory. One Op per fused region:
//   FoldOp    the serial repaired fold of any skeleton (template.py:41-54, two-pass :62-103)
//   SoftmaxOp softmax / log_softmax + logsumexp (the lowering of neptune_recognize/lowering.py:80-99)
//   L2Op      stable_l2 norm and x / norm
//   RmsOp     RMSNorm with the reference's fp32 stages (emitters.py:576-595)
// span_kernel: every warp folds a contiguous column span of one row (a split-plan chunk, or a whole
// row too wide for one stage) through its ring in sub-blocks, keeping a per-lane fold state; at the
// span's end the 32 lane states merge in a fixed tree and the warp writes the chunk state (split
// plan, template.py:137-165) or the finalised result.
#include <algorithm>

#include "launch.h"
#include "row_ops.cuh"

namespace nb200 {

struct RowPlan {
    int64_t rows, ncols, srow;  // srow in elements
    int64_t nblocks;            // ceil(rows / R)
    uint32_t row_bytes, stage_bytes, extra_bytes, bar_offset, stage_offset;
    int R, S, packed, warps;
};

// ------------------------------------------------------------------ resident-row kernel
template <typename T, class Op>
__global__ void __launch_bounds__(512) rows_kernel(const T* __restrict__ x, RowPlan pl, Op op) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + pl.bar_offset) + warp * pl.S;
    unsigned char* ring = smem + pl.stage_offset + (size_t)warp * pl.S * pl.stage_bytes;
    op.prologue(smem);
    if (lane == 0) {
        for (int s = 0; s < pl.S; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int64_t gw = (int64_t)blockIdx.x * nw + warp, GW = (int64_t)gridDim.x * nw;
    auto issue = [&](int64_t b, int s) {
        const int64_t r0 = b * pl.R;
        const int nr = (int)min((int64_t)pl.R, pl.rows - r0);
        unsigned char* dst = ring + (size_t)s * pl.stage_bytes;
        mbar_expect_tx(&bar[s], (uint32_t)nr * pl.row_bytes);
        if (pl.packed) {
            bulk_load(dst, x + r0 * pl.srow, (uint32_t)nr * pl.row_bytes, &bar[s]);
        } else {
            for (int i = 0; i < nr; ++i) bulk_load(dst + (size_t)i * pl.row_bytes, x + (r0 + i) * pl.srow, pl.row_bytes, &bar[s]);
        }
    };
    if (lane == 0)
        for (int s = 0; s < pl.S; ++s)
            if (gw + s * GW < pl.nblocks) issue(gw + s * GW, s);
    __syncwarp();
    int64_t k = 0;
    for (int64_t b = gw; b < pl.nblocks; b += GW, ++k) {
        const int s = (int)(k % pl.S);
        const uint32_t parity = (uint32_t)((k / pl.S) & 1);
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[s], parity))) {
            // A wait ran out (fault bit already set): give the copies still in flight a bounded
            // chance to land before the CTA's shared memory is released, then stop.
            for (int64_t kk = k; kk < k + pl.S; ++kk)
                if (gw + kk * GW < pl.nblocks) mbar_wait(&bar[kk % pl.S], (uint32_t)((kk / pl.S) & 1));
            return;
        }
        const unsigned char* stage = ring + (size_t)s * pl.stage_bytes;
        const int64_t r0 = b * pl.R;
        const int nr = (int)min((int64_t)pl.R, pl.rows - r0);
        for (int i = 0; i < nr; ++i)
            op.row(SmemRow{reinterpret_cast<const uint4*>(stage + (size_t)i * pl.row_bytes), op.nv, lane}, r0 + i,
                   lane, smem);
        __syncwarp();
        if (lane == 0 && b + pl.S * GW < pl.nblocks) {
            fence_proxy_async();
            issue(b + pl.S * GW, s);
        }
        __syncwarp();
    }
}

// ------------------------------------------------------------------ span kernel
struct SpanPlan {
    int64_t rows, srow, cb, ns, cc, nparts, nitems;  // items = rows * nparts
    int64_t sub_cols;                                // columns per staged sub-block
    int nsub;                                        // sub-blocks per item (upper bound)
    int S;
    uint32_t stage_bytes, bar_offset, stage_offset;
    int finalize;                                    // 1: write out[r]; 0: write states[item]
};

template <int S_, typename T>
__global__ void __launch_bounds__(512) span_kernel(const T* __restrict__ x, SpanPlan pl, Params p,
                                                   nb200_state* __restrict__ states, T* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(128) unsigned char smem[];
    constexpr int V = Elem<T>::V;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + pl.bar_offset) + warp * pl.S;
    unsigned char* ring = smem + pl.stage_offset + (size_t)warp * pl.S * pl.stage_bytes;
    if (lane == 0) {
        for (int s = 0; s < pl.S; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    const int64_t gw = (int64_t)blockIdx.x * nw + warp, GW = (int64_t)gridDim.x * nw;
    // Task cursors walk (item, sub-block) pairs of this warp: items gw, gw + GW, ..., nsub
    // sub-blocks each. `next` is the task to issue, `cur` the task to consume; both advance by
    // increments, so the loop does no integer division per task.
    struct Cursor {
        int64_t item, row, lo, hi;  // item index, its row and its column span
        int sub;
    };
    auto start_item = [&](Cursor& c, int64_t item) {
        c.item = item;
        c.sub = 0;
        if (item < pl.nitems) {
            c.row = item / pl.nparts;
            const int64_t part = item - c.row * pl.nparts;
            c.lo = pl.cb + part * pl.cc;
            c.hi = min(c.lo + pl.cc, pl.cb + pl.ns);
        }
    };
    auto advance = [&](Cursor& c) {
        if (++c.sub == pl.nsub) start_item(c, c.item + GW);
    };
    int stage_issue = 0, stage_use = 0;
    uint32_t parity = 0;
    auto issue = [&](const Cursor& c) {
        const int64_t c0 = c.lo + (int64_t)c.sub * pl.sub_cols;
        const int64_t c1 = max(c0, min(c0 + pl.sub_cols, c.hi));
        const uint32_t bytes = (uint32_t)((c1 - c0) * (int64_t)sizeof(T));
        uint64_t* b = &bar[stage_issue];
        if (bytes == 0) {  // an empty tail sub-block: complete the phase without a copy
            mbar_arrive(b);
        } else {
            mbar_expect_tx(b, bytes);
            bulk_load(ring + (size_t)stage_issue * pl.stage_bytes, x + c.row * pl.srow + c0, bytes, b);
        }
        stage_issue = stage_issue + 1 == pl.S ? 0 : stage_issue + 1;
    };
    Cursor next, cur;
    start_item(next, gw);
    start_item(cur, gw);
    if (lane == 0)
        for (int s = 0; s < pl.S && next.item < pl.nitems; ++s) {
            issue(next);
            advance(next);
        }
    __syncwarp();
    St run = empty_state();
    while (cur.item < pl.nitems) {
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[stage_use], parity))) {
            // bounded drain of the copies still in flight, then stop
            int s = stage_use;
            uint32_t ph = parity;
            for (int k = 0; k < pl.S; ++k) {
                mbar_wait(&bar[s], ph);
                if (++s == pl.S) { s = 0; ph ^= 1u; }
            }
            return;
        }
        const int64_t c0 = cur.lo + (int64_t)cur.sub * pl.sub_cols;
        const int64_t c1 = max(c0, min(c0 + pl.sub_cols, cur.hi));
        const int nv = (int)((c1 - c0) / V);
        const St sub = lane_state<S_, T>(
            SmemRow{reinterpret_cast<const uint4*>(ring + (size_t)stage_use * pl.stage_bytes), nv, lane}, p);
        run = merge_fast<S_>(run, sub, p);
        __syncwarp();
        if (lane == 0 && next.item < pl.nitems) {
            fence_proxy_async();
            issue(next);
        }
        if (next.item < pl.nitems) advance(next);
        if (++stage_use == pl.S) {
            stage_use = 0;
            parity ^= 1u;
        }
        if (cur.sub == pl.nsub - 1) {  // the item's last sub-block
            const St w = warp_merge<S_>(run, lane, p);
            if (lane == 0) {
                if (pl.finalize) out[cur.row] = Elem<T>::from_f(finalize<S_>(w, p));
                else reinterpret_cast<float4*>(states)[cur.item] =
                         make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status));
            }
            run = empty_state();
        }
        advance(cur);
        __syncwarp();
    }
}

// ================================================================== host side
namespace {

constexpr int kStreamThreads = 128;  // 4 warps per CTA, several CTAs per SM
constexpr int kSpanWarps = 4;
constexpr int kSpanStages = 2;
constexpr uint32_t kSpanStageBytes = 4096;  // small sub-blocks: more CTAs (warps) per SM
constexpr uint32_t kSmemBudget = 224 * 1024;

inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

template <typename K>
int ensure_smem(K kernel, uint32_t bytes) {
    static_assert(sizeof(K) > 0, "");
    if (bytes <= 48 * 1024) return NB200_OK;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess) {
        cudaGetLastError();
        set_error("cannot reserve %u bytes of shared memory", bytes);
        return NB200_ERR_LAUNCH;
    }
    return NB200_OK;
}

// Rows are eligible when each row is a 16-byte-aligned, 16-byte-multiple contiguous run.
template <typename T>
bool rows_streamable(const T* x, int64_t rows, int64_t ncols, int64_t srow, int64_t scol) {
    const int64_t rb = ncols * (int64_t)sizeof(T);
    return scol == 1 && aligned16(x) && rb % 16 == 0 && (rows <= 1 || (srow * (int64_t)sizeof(T)) % 16 == 0) &&
           rb <= 32768;
}

bool make_row_plan(int64_t rows, int64_t ncols, int64_t srow, size_t esize, uint32_t extra, RowPlan& pl,
                   int nw, int want_stages) {
    pl.rows = rows;
    pl.ncols = ncols;
    pl.srow = srow;
    pl.row_bytes = (uint32_t)(ncols * (int64_t)esize);
    pl.packed = (rows <= 1 || srow == ncols) ? 1 : 0;
    int R = (int)std::max<int64_t>(1, 8192 / pl.row_bytes);
    if (!pl.packed) R = std::min(R, 4);
    pl.R = R;
    pl.stage_bytes = align_up((uint32_t)R * pl.row_bytes, 128);
    pl.nblocks = (rows + R - 1) / R;
    pl.extra_bytes = align_up(extra, 128);
    pl.bar_offset = pl.extra_bytes;
    pl.stage_offset = align_up(pl.bar_offset + nw * 8 * 8, 128);
    const int fit = (int)((kSmemBudget - pl.stage_offset) / ((uint32_t)nw * pl.stage_bytes));
    const int S = want_stages > 0 ? want_stages : std::min(fit, 2);
    if (S < 2 || S > fit || S > 8) return false;
    pl.S = S;
    pl.warps = nw;
    return true;
}

uint32_t row_smem(const RowPlan& pl) { return pl.stage_offset + (uint32_t)pl.warps * pl.S * pl.stage_bytes; }

template <typename T, class Op>
int launch_rows(const T* x, const RowPlan& pl, const Op& op, cudaStream_t st, const char* what, int cps) {
    auto k = rows_kernel<T, Op>;
    const uint32_t smem = row_smem(pl);
    int rc = ensure_smem(k, smem);
    if (rc) return rc;
    const int threads = pl.warps * 32;
    const int g = persistent_grid(k, threads, smem, (pl.nblocks + pl.warps - 1) / pl.warps, cps);
    launch_pdl(k, g, threads, smem, st, x, pl, op);
    count_launch();
    return finish_launch(what);
}

}  // namespace

int stream_fault_take(unsigned int* bits) {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_stream_fault, sizeof(v)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_stream_fault, &zero, sizeof(zero)) != cudaSuccess) {
        set_error("cannot read the streaming fault word: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    *bits = v;
    return NB200_OK;
}

// Returns 1 (and launches) when the streaming path applies, 0 when the caller should use the
// register-tiled kernels, negative on error.
// The library's own policy (no launch given, or variant AUTO) sends 1-8 KB rows to the register-row
// kernel; an explicit STREAM launch keeps the bulk-copy ring.
template <typename T>
inline bool use_ldg(const nb200_launch* L, int64_t ncols) {
    return (!L || L->variant == NB200_VARIANT_AUTO) && ldg_rows_eligible((uint32_t)(ncols * (int64_t)sizeof(T)));
}
inline int plan_warps(const nb200_launch* L) { return (L && L->threads) ? L->threads / 32 : kStreamThreads / 32; }
inline int plan_stages(const nb200_launch* L) { return L ? L->stages : 0; }
inline int plan_cps(const nb200_launch* L) { return L ? L->ctas_per_sm : 0; }

template <typename T>
int stream_fold_t(int sk, const Params& p, const T* x, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
                  T* out, const nb200_launch* L, cudaStream_t st) {
    if (!rows_streamable(x, rows, ncols, srow, scol)) return 0;
    const int nv = (int)(ncols / Elem<T>::V);
    int rc;
    if (use_ldg<T>(L, ncols)) {
        switch (sk) {
#define X(S) case S: rc = launch_ldg_rows(x, rows, srow, FoldOp<S, T>{out, p, nv}, 0, st, "nb200_fold"); break;
            X(NB200_LOGSUMEXP) X(NB200_LSE_BIASED) X(NB200_LSE_SCALED) X(NB200_SOFTCAP_LSE) X(NB200_STABLE_L2)
            X(NB200_LINEAR_ATTN) X(NB200_DECAY_RENORM) X(NB200_SUMSQ_DIV) X(NB200_RMSNORM_MAX) X(NB200_VARIANCE)
            X(NB200_STD)
#undef X
            default: return 0;
        }
        return rc ? rc : 1;
    }
    RowPlan pl;
    if (!make_row_plan(rows, ncols, srow, sizeof(T), 0, pl, plan_warps(L), plan_stages(L))) return 0;
    switch (sk) {
#define X(S) case S: rc = launch_rows(x, pl, FoldOp<S, T>{out, p, nv}, st, "nb200_fold", plan_cps(L)); break;
        X(NB200_LOGSUMEXP) X(NB200_LSE_BIASED) X(NB200_LSE_SCALED) X(NB200_SOFTCAP_LSE) X(NB200_STABLE_L2)
        X(NB200_LINEAR_ATTN) X(NB200_DECAY_RENORM) X(NB200_SUMSQ_DIV) X(NB200_RMSNORM_MAX) X(NB200_VARIANCE)
        X(NB200_STD)
#undef X
        default: return 0;
    }
    return rc ? rc : 1;
}

template <typename T>
int stream_softmax_t(int mode, const T* x, int64_t rows, int64_t ncols, int64_t srow, int64_t scol, T* y, T* lse,
                     const nb200_launch* L, cudaStream_t st) {
    if (!rows_streamable(x, rows, ncols, srow, scol) || !aligned16(y)) return 0;
    const SoftmaxOp<T> op{y, lse, ncols, (int)(ncols / Elem<T>::V), mode};
    if (use_ldg<T>(L, ncols)) {
        const int rc = launch_ldg_rows(x, rows, srow, op, 0, st, "nb200_softmax");
        return rc ? rc : 1;
    }
    RowPlan pl;
    if (!make_row_plan(rows, ncols, srow, sizeof(T), 0, pl, plan_warps(L), plan_stages(L))) return 0;
    const int rc = launch_rows(x, pl, op, st, "nb200_softmax", plan_cps(L));
    return rc ? rc : 1;
}

template <typename T>
int stream_l2_t(const T* x, int64_t rows, int64_t ncols, int64_t srow, int64_t scol, T* y, T* norm,
                const nb200_launch* L, cudaStream_t st) {
    if (!rows_streamable(x, rows, ncols, srow, scol) || !aligned16(y)) return 0;
    const L2Op<T> op{y, norm, ncols, (int)(ncols / Elem<T>::V)};
    if (use_ldg<T>(L, ncols)) {
        const int rc = launch_ldg_rows(x, rows, srow, op, 0, st, "nb200_l2_normalize");
        return rc ? rc : 1;
    }
    RowPlan pl;
    if (!make_row_plan(rows, ncols, srow, sizeof(T), 0, pl, plan_warps(L), plan_stages(L))) return 0;
    const int rc = launch_rows(x, pl, op, st, "nb200_l2_normalize", plan_cps(L));
    return rc ? rc : 1;
}

template <typename T>
int stream_rms_t(const T* x, const T* gamma, int64_t rows, int64_t ncols, int64_t srow, int64_t scol, int64_t sg,
                 float eps, T* y, const nb200_launch* L, cudaStream_t st) {
    if (!rows_streamable(x, rows, ncols, srow, scol) || !aligned16(y)) return 0;
    const RmsOp<T> op{y, gamma, ncols, sg, (int)(ncols / Elem<T>::V), eps, static_cast<float>(ncols)};
    if (use_ldg<T>(L, ncols)) {
        const uint32_t gbytes = (uint32_t)(ncols * (int64_t)sizeof(T));
        int rc = gbytes > 48 * 1024 ? NB200_ERR_LAUNCH : NB200_OK;
        if (!rc) rc = launch_ldg_rows(x, rows, srow, op, gbytes, st, "nb200_rms_norm");
        return rc ? rc : 1;
    }
    RowPlan pl;
    if (!make_row_plan(rows, ncols, srow, sizeof(T), (uint32_t)(ncols * (int64_t)sizeof(T)), pl, plan_warps(L),
                       plan_stages(L)))
        return 0;
    const int rc = launch_rows(x, pl, op, st, "nb200_rms_norm", plan_cps(L));
    return rc ? rc : 1;
}

// Column spans [cb + part * cc, ...) of every row, staged through 4 KB sub-blocks. finalize = 1
// requires nparts == 1 (a whole row per item) and writes out[rows].
template <typename T>
int stream_span_t(int sk, const Params& p, const T* x, int64_t rows, int64_t cb, int64_t ns, int64_t srow,
                  int64_t scol, int64_t cc, int64_t nparts, nb200_state* states, T* out, int finalize,
                  const nb200_launch* L, cudaStream_t st) {
    constexpr int V = Elem<T>::V;
    if (scol != 1 || !aligned16(x) || (rows > 1 && (srow * (int64_t)sizeof(T)) % 16 != 0) || cb % V || ns % V ||
        cc % V)
        return 0;
    if (sk == NB200_VARIANCE || sk == NB200_STD) return 0;
    if (!L || L->variant == NB200_VARIANT_AUTO) return launch_ldg_span<T>(sk, p, x, rows, cb, ns, srow, cc, nparts,
                                                                          states, out, finalize, st);
    SpanPlan pl;
    pl.rows = rows;
    pl.srow = srow;
    pl.cb = cb;
    pl.ns = ns;
    pl.cc = cc;
    pl.nparts = nparts;
    pl.nitems = rows * nparts;
    pl.sub_cols = kSpanStageBytes / (int64_t)sizeof(T);
    pl.nsub = (int)((cc + pl.sub_cols - 1) / pl.sub_cols);
    pl.stage_bytes = kSpanStageBytes;
    pl.bar_offset = 0;
    const int nw = (L && L->threads) ? L->threads / 32 : kSpanWarps;
    pl.stage_offset = align_up(nw * 8 * 8, 128);
    pl.S = (L && L->stages) ? L->stages : kSpanStages;
    if (pl.S < 2 || pl.stage_offset + (uint32_t)nw * pl.S * pl.stage_bytes > kSmemBudget) return 0;
    pl.finalize = finalize;
    const uint32_t smem = pl.stage_offset + (uint32_t)nw * pl.S * pl.stage_bytes;
    int rc = NB200_OK;
    auto go = [&](auto k) {
        rc = ensure_smem(k, smem);
        if (rc) return;
        const int g = persistent_grid(k, nw * 32, smem, (pl.nitems + nw - 1) / nw, L ? L->ctas_per_sm : 0);
        launch_pdl(k, g, nw * 32, smem, st, x, pl, p, states, out);
        count_launch();
        rc = finish_launch(finalize ? "nb200_fold" : "nb200_fold_partial");
    };
    switch (sk) {
#define X(S) case S: go(span_kernel<S, T>); break;
        X(NB200_LOGSUMEXP) X(NB200_LSE_BIASED) X(NB200_LSE_SCALED) X(NB200_SOFTCAP_LSE) X(NB200_STABLE_L2)
        X(NB200_LINEAR_ATTN) X(NB200_DECAY_RENORM) X(NB200_SUMSQ_DIV) X(NB200_RMSNORM_MAX)
#undef X
        default: return 0;
    }
    return rc ? rc : 1;
}

#define NB200_STREAM_DTYPES(dtype, CALL)                            \
    switch (dtype) {                                                \
        case NB200_F32: { using T = float; return CALL; }           \
        case NB200_BF16: { using T = __nv_bfloat16; return CALL; }  \
        case NB200_F16: { using T = __half; return CALL; }          \
    }                                                               \
    return 0;

int stream_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow,
                int64_t scol, void* out, const nb200_launch* L, cudaStream_t st) {
    NB200_STREAM_DTYPES(dtype, stream_fold_t<T>(sk, p, (const T*)x, rows, ncols, srow, scol, (T*)out, L, st))
}
int stream_softmax(int mode, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
                   void* y, void* lse, const nb200_launch* L, cudaStream_t st) {
    NB200_STREAM_DTYPES(dtype, stream_softmax_t<T>(mode, (const T*)x, rows, ncols, srow, scol, (T*)y, (T*)lse, L, st))
}
int stream_l2(const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol, void* y, void* norm,
              const nb200_launch* L, cudaStream_t st) {
    NB200_STREAM_DTYPES(dtype, stream_l2_t<T>((const T*)x, rows, ncols, srow, scol, (T*)y, (T*)norm, L, st))
}
int stream_rms(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
               int64_t sg, float eps, void* y, const nb200_launch* L, cudaStream_t st) {
    NB200_STREAM_DTYPES(dtype, stream_rms_t<T>((const T*)x, (const T*)gamma, rows, ncols, srow, scol, sg, eps, (T*)y, L,
                                               st))
}
int stream_span(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t cb, int64_t ns,
                int64_t srow, int64_t scol, int64_t cc, int64_t nparts, nb200_state* states, void* out,
                int finalize, const nb200_launch* L, cudaStream_t st) {
    NB200_STREAM_DTYPES(dtype, stream_span_t<T>(sk, p, (const T*)x, rows, cb, ns, srow, scol, cc, nparts, states,
                                                (T*)out, finalize, L, st))
}

}  // namespace nb200
