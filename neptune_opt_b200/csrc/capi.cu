// The extern "C" boundary: argument validation, error reporting and launch bookkeeping.
// Nothing here allocates device memory; every pointer is caller-owned.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "fold.cuh"
#include "launch.h"

namespace nb200 {

namespace {
thread_local char g_error[512] = "";
std::atomic<uint64_t> g_launches{0};
std::mutex g_sm_mutex;
int g_sm_count[64] = {0};
}  // namespace

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(g_sm_mutex);
    if (g_sm_count[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

void count_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int finish_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(e));
        return NB200_ERR_LAUNCH;
    }
    return NB200_OK;
}

}  // namespace nb200

using namespace nb200;

namespace {

bool valid_dtype(int d) { return d == NB200_F32 || d == NB200_BF16 || d == NB200_F16; }

// Declared-parameter checks of the reference's certificate (algebra.py:285-302): every declared
// scalar finite, T/beta/N/eps strictly positive, tiny nonnegative.
int check_params(int sk, const nb200_params* q, nb200_params* out) {
    nb200_params p{};
    if (q) p = *q;
    *out = p;
    auto finite = [](double v) { return std::isfinite(v); };
    switch (sk) {
        case NB200_LOGSUMEXP:
            if (!finite(p.tiny) || p.tiny < 0) { set_error("parameter 'tiny' must be finite and nonnegative"); return NB200_ERR_ARG; }
            return NB200_OK;
        case NB200_LSE_BIASED:
            if (!finite(p.tiny) || p.tiny < 0) { set_error("parameter 'tiny' must be finite and nonnegative"); return NB200_ERR_ARG; }
            if (!finite(p.alpha)) { set_error("parameter 'alpha' must be finite"); return NB200_ERR_ARG; }
            return NB200_OK;
        case NB200_LSE_SCALED:
            if (!finite(p.tiny) || p.tiny < 0) { set_error("parameter 'tiny' must be finite and nonnegative"); return NB200_ERR_ARG; }
            if (!finite(p.T) || p.T <= 0) { set_error("parameter 'T' must be finite and positive"); return NB200_ERR_ARG; }
            return NB200_OK;
        case NB200_SOFTCAP_LSE:
            if (!finite(p.tiny) || p.tiny < 0) { set_error("parameter 'tiny' must be finite and nonnegative"); return NB200_ERR_ARG; }
            if (!finite(p.beta) || p.beta <= 0) { set_error("parameter 'beta' must be finite and positive"); return NB200_ERR_ARG; }
            return NB200_OK;
        case NB200_DECAY_RENORM:
            if (!finite(p.N) || p.N <= 0) { set_error("parameter 'N' must be finite and positive"); return NB200_ERR_ARG; }
            return NB200_OK;
        case NB200_RMSNORM_MAX:
            if (!finite(p.eps) || p.eps <= 0) { set_error("parameter 'eps' must be finite and positive"); return NB200_ERR_ARG; }
            return NB200_OK;
        case NB200_STABLE_L2: case NB200_LINEAR_ATTN: case NB200_SUMSQ_DIV:
        case NB200_VARIANCE: case NB200_STD:
            return NB200_OK;
    }
    set_error("unknown skeleton %d", sk);
    return NB200_ERR_ARG;
}

int check_rows(const void* x, int dtype, int64_t rows, int64_t ncols, const void* out, const char* what) {
    if (!valid_dtype(dtype)) { set_error("%s: unsupported dtype %d; expected float16/bfloat16/float32", what, dtype); return NB200_ERR_ARG; }
    if (rows < 0) { set_error("%s: negative row count", what); return NB200_ERR_ARG; }
    if (ncols <= 0) { set_error("%s: Neptune requires positive last-dimension width", what); return NB200_ERR_ARG; }
    if (rows > 0 && (x == nullptr || out == nullptr)) { set_error("%s: null data pointer", what); return NB200_ERR_ARG; }
    return NB200_OK;
}

int check_launch(const nb200_launch* L) {
    if (!L) return NB200_OK;
    if (L->variant < 0 || L->variant > NB200_VARIANT_CLUSTER) { set_error("unknown launch variant %d", L->variant); return NB200_ERR_ARG; }
    if (L->threads && (L->threads < 64 || L->threads > 512 || L->threads % 32)) {
        set_error("launch threads must be a multiple of 32 in [64, 512]"); return NB200_ERR_ARG;
    }
    if (L->ctas_per_sm < 0 || L->ctas_per_sm > 32) { set_error("ctas_per_sm must be in [0, 32]"); return NB200_ERR_ARG; }
    if (L->variant == NB200_VARIANT_CLUSTER) {
        if (L->stages != 0 && (L->stages < 2 || L->stages > 16)) {
            set_error("cluster launches take 2..16 CTAs per row (stages field), or 0 to choose");
            return NB200_ERR_ARG;
        }
    } else if (L->stages < 0 || L->stages > 8) { set_error("stages must be in [0, 8]"); return NB200_ERR_ARG; }
    return NB200_OK;
}

}  // namespace

extern "C" {

const char* nb200_last_error(void) { return g_error; }
const char* nb200_version(void) { return "neptune_b200 0.1 (sm_100a)"; }
uint64_t nb200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int nb200_stream_fault(uint32_t* bits) {
    if (!bits) { set_error("nb200_stream_fault: null pointer"); return NB200_ERR_ARG; }
    unsigned int v = 0, w = 0, x = 0;
    int rc = stream_fault_take(&v);
    if (rc == NB200_OK) rc = attn_fault_take(&w);
    if (rc == NB200_OK) rc = peer_fault_take(&x);
    *bits = v | w | x;
    return rc;
}

int nb200_fold(int skeleton, const nb200_params* params, const void* x, int dtype, int64_t rows,
               int64_t ncols, int64_t stride_row, int64_t stride_col, void* out,
               const nb200_launch* launch, void* stream) {
    nb200_params q;
    int rc = check_params(skeleton, params, &q);
    if (rc) return rc;
    if ((rc = check_rows(x, dtype, rows, ncols, out, "nb200_fold"))) return rc;
    if ((rc = check_launch(launch))) return rc;
    if (rows == 0) return NB200_OK;
    return launch_fold(skeleton, make_params(q, ncols), x, dtype, rows, ncols, stride_row, stride_col,
                       out, launch, (cudaStream_t)stream);
}

int nb200_softmax(int mode, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t stride_row,
                  int64_t stride_col, void* y, void* lse, const nb200_launch* launch, void* stream) {
    if (mode != 0 && mode != 1) { set_error("nb200_softmax: mode must be 0 (softmax) or 1 (log_softmax)"); return NB200_ERR_ARG; }
    int rc = check_rows(x, dtype, rows, ncols, y, "nb200_softmax");
    if (rc) return rc;
    if ((rc = check_launch(launch))) return rc;
    if (rows == 0) return NB200_OK;
    return launch_softmax(mode, x, dtype, rows, ncols, stride_row, stride_col, y, lse, launch,
                          (cudaStream_t)stream);
}

int nb200_l2_normalize(const void* x, int dtype, int64_t rows, int64_t ncols, int64_t stride_row,
                       int64_t stride_col, void* y, void* norm, const nb200_launch* launch, void* stream) {
    int rc = check_rows(x, dtype, rows, ncols, y, "nb200_l2_normalize");
    if (rc) return rc;
    if ((rc = check_launch(launch))) return rc;
    if (rows == 0) return NB200_OK;
    return launch_l2(x, dtype, rows, ncols, stride_row, stride_col, y, norm, launch, (cudaStream_t)stream);
}

int64_t nb200_fold_split_scratch_bytes(int64_t rows, int64_t nparts) {
    if (rows < 0 || nparts < 0) return -1;
    return rows * nparts * (int64_t)sizeof(nb200_state);
}

int nb200_fold_partial(int skeleton, const nb200_params* params, const void* x, int dtype, int64_t rows,
                       int64_t ncols_total, int64_t col_begin, int64_t ncols_shard, int64_t stride_row,
                       int64_t stride_col, int64_t chunk_cols, nb200_state* states, const nb200_launch* launch,
                       void* stream) {
    nb200_params q;
    int rc = check_params(skeleton, params, &q);
    if (rc) return rc;
    if ((rc = check_rows(x, dtype, rows, ncols_total, states, "nb200_fold_partial"))) return rc;
    if (col_begin < 0 || ncols_shard <= 0 || col_begin + ncols_shard > ncols_total) {
        set_error("nb200_fold_partial: column shard [%lld, %lld) outside [0, %lld)", (long long)col_begin,
                  (long long)(col_begin + ncols_shard), (long long)ncols_total);
        return NB200_ERR_ARG;
    }
    if (chunk_cols <= 0) { set_error("nb200_fold_partial: chunk_cols must be positive"); return NB200_ERR_ARG; }
    if ((rc = check_launch(launch))) return rc;
    if (rows > 0 && !aligned16(states)) { set_error("nb200_fold_partial: states must be 16-byte aligned"); return NB200_ERR_ARG; }
    if (rows == 0) return NB200_OK;
    const int64_t nparts = (ncols_shard + chunk_cols - 1) / chunk_cols;
    return launch_partial(skeleton, make_params(q, ncols_total), x, dtype, rows, col_begin, ncols_shard,
                          stride_row, stride_col, chunk_cols, nparts, states, launch, (cudaStream_t)stream);
}

int nb200_fold_merge(int skeleton, const nb200_params* params, const nb200_state* states, int64_t rows,
                     int64_t nparts, int64_t row_stride, int64_t part_stride, void* out, int dtype,
                     void* stream) {
    nb200_params q;
    int rc = check_params(skeleton, params, &q);
    if (rc) return rc;
    if (!valid_dtype(dtype)) { set_error("nb200_fold_merge: unsupported dtype %d", dtype); return NB200_ERR_ARG; }
    if (rows < 0 || nparts <= 0) { set_error("nb200_fold_merge: need rows >= 0 and nparts > 0"); return NB200_ERR_ARG; }
    if (rows == 0) return NB200_OK;
    if (!states || !out) { set_error("nb200_fold_merge: null pointer"); return NB200_ERR_ARG; }
    return launch_merge(skeleton, make_params(q, 0), states, rows, nparts, row_stride, part_stride, out,
                        dtype, (cudaStream_t)stream);
}

int nb200_fold_split(int skeleton, const nb200_params* params, const void* x, int dtype, int64_t rows,
                     int64_t ncols, int64_t stride_row, int64_t stride_col, int64_t chunk_cols,
                     void* scratch, int64_t scratch_bytes, void* out, const nb200_launch* launch, void* stream) {
    nb200_params q;
    int rc = check_params(skeleton, params, &q);
    if (rc) return rc;
    if ((rc = check_rows(x, dtype, rows, ncols, out, "nb200_fold_split"))) return rc;
    if (skeleton == NB200_VARIANCE || skeleton == NB200_STD) {
        set_error("two_pass needs extended carried state; split refused");
        return NB200_ERR_UNSUPPORTED;
    }
    if (chunk_cols <= 0) { set_error("nb200_fold_split: chunk_cols must be positive"); return NB200_ERR_ARG; }
    if ((rc = check_launch(launch))) return rc;
    const int64_t nparts = (ncols + chunk_cols - 1) / chunk_cols;
    if (nparts > 4096) {
        set_error("split needs %lld partials, exceeding capacity 4096; use serial", (long long)nparts);
        return NB200_ERR_CAPACITY;
    }
    if (rows == 0) return NB200_OK;
    const int64_t need = nb200_fold_split_scratch_bytes(rows, nparts);
    if (!scratch || scratch_bytes < need || !aligned16(scratch)) {
        set_error("nb200_fold_split: scratch needs %lld bytes, 16-byte aligned (got %lld)", (long long)need,
                  (long long)scratch_bytes);
        return NB200_ERR_ARG;
    }
    nb200_state* states = (nb200_state*)scratch;
    const Params p = make_params(q, ncols);
    rc = launch_partial(skeleton, p, x, dtype, rows, 0, ncols, stride_row, stride_col, chunk_cols, nparts,
                        states, launch, (cudaStream_t)stream);
    if (rc) return rc;
    return launch_merge(skeleton, p, states, rows, nparts, nparts, 1, out, dtype, (cudaStream_t)stream);
}

int nb200_rms_norm(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols,
                   int64_t stride_row, int64_t stride_col, int64_t stride_gamma, double eps, void* out,
                   const nb200_launch* launch, void* stream) {
    int rc = check_rows(x, dtype, rows, ncols, out, "nb200_rms_norm");
    if (rc) return rc;
    if ((rc = check_launch(launch))) return rc;
    if (!std::isfinite(eps) || eps <= 0) { set_error("RMSNorm requires an explicit finite positive eps"); return NB200_ERR_ARG; }
    if (rows == 0) return NB200_OK;
    if (!gamma) { set_error("nb200_rms_norm: null gamma"); return NB200_ERR_ARG; }
    return launch_rms(x, gamma, dtype, rows, ncols, stride_row, stride_col, stride_gamma, (float)eps, out,
                      launch, (cudaStream_t)stream);
}

int nb200_segment_spans(const void* lengths, int index_dtype, int64_t nsegments, int64_t length_stride,
                        int unsafe, int64_t nrows, int64_t* spans, uint32_t* status, void* stream) {
    if (index_dtype != NB200_I32 && index_dtype != NB200_I64) {
        set_error("segment index dtype must be int32/int64"); return NB200_ERR_ARG;
    }
    if (nsegments < 0 || nrows < 0) { set_error("nb200_segment_spans: negative size"); return NB200_ERR_ARG; }
    if (!spans || (nsegments > 0 && !lengths)) { set_error("nb200_segment_spans: null pointer"); return NB200_ERR_ARG; }
    return launch_spans(lengths, index_dtype, nsegments, length_stride, unsafe, nrows, spans, status,
                        (cudaStream_t)stream);
}

int nb200_segment_pool(const void* data, int dtype, int64_t nrows, int64_t channels, int64_t stride_row,
                       int64_t stride_channel, const void* bounds, int index_dtype, int64_t bound_stride,
                       int64_t nsegments, int reduce, int has_initial, uint32_t initial_bits, void* out,
                       uint32_t* status, void* stream) {
    if (!valid_dtype(dtype)) { set_error("segment data dtype must be float16/bfloat16/float32"); return NB200_ERR_ARG; }
    if (index_dtype != NB200_I32 && index_dtype != NB200_I64) {
        set_error("segment index dtype must be int32/int64"); return NB200_ERR_ARG;
    }
    if (reduce != 0 && reduce != 1) { set_error("segment reduce must be 0 (sum) or 1 (mean)"); return NB200_ERR_ARG; }
    if (nrows < 0 || channels < 0 || nsegments < 0) { set_error("nb200_segment_pool: negative size"); return NB200_ERR_ARG; }
    if (nsegments == 0 || channels == 0) return NB200_OK;
    if (!bounds || !out || (nrows > 0 && !data)) { set_error("nb200_segment_pool: null pointer"); return NB200_ERR_ARG; }
    return launch_segment_pool(data, dtype, nrows, channels, stride_row, stride_channel, bounds, index_dtype,
                               bound_stride, nsegments, reduce, has_initial, initial_bits, out, status,
                               (cudaStream_t)stream);
}

int64_t nb200_peer_buffer_bytes(int64_t rows, int64_t world, int64_t nparts) {
    if (rows < 0 || world < 1 || world > peer_max_world() || nparts < 1) return -1;
    return peer_buffer_bytes(rows, world, nparts);
}

int nb200_peer_init(void* buffer, int64_t rows, int world, int64_t nparts, void* stream) {
    if (world < 1 || world > peer_max_world() || rows < 0 || nparts < 1) {
        set_error("nb200_peer_init: need 1 <= world <= %d, rows >= 0, nparts >= 1", peer_max_world());
        return NB200_ERR_ARG;
    }
    if (!buffer || (reinterpret_cast<uintptr_t>(buffer) & 255u)) {
        set_error("nb200_peer_init: null or unaligned buffer");
        return NB200_ERR_ARG;
    }
    return launch_peer_init(buffer, rows, nparts, world, (cudaStream_t)stream);
}

int nb200_peer_push(const nb200_state* states, int64_t rows, int64_t nlocal, int64_t nparts, void* const* peers,
                    int world, int rank, void* buffer, void* stream) {
    if (world < 1 || world > peer_max_world() || rank < 0 || rank >= world) {
        set_error("nb200_peer_push: need 1 <= world <= %d and 0 <= rank < world", peer_max_world());
        return NB200_ERR_ARG;
    }
    if (rows < 0 || nlocal < 0 || nparts < 1 || nlocal > nparts) {
        set_error("nb200_peer_push: need rows >= 0 and 0 <= nlocal <= nparts, nparts >= 1");
        return NB200_ERR_ARG;
    }
    if (!peers || !buffer || (rows > 0 && nlocal > 0 && !states)) {
        set_error("nb200_peer_push: null pointer");
        return NB200_ERR_ARG;
    }
    for (int r = 0; r < world; ++r)
        if (!peers[r] || (reinterpret_cast<uintptr_t>(peers[r]) & 255u)) {
            set_error("nb200_peer_push: exchange buffer of rank %d is null or not 256-byte aligned", r);
            return NB200_ERR_ARG;
        }
    if (peers[rank] != buffer) {
        set_error("nb200_peer_push: peers[rank] must be this rank's own buffer");
        return NB200_ERR_ARG;
    }
    return launch_peer_push(states, rows, nlocal, nparts, peers, world, rank, buffer, (cudaStream_t)stream);
}

int nb200_peer_fold(int skeleton, const nb200_params* params, const void* x, int dtype, int64_t rows,
                    int64_t ncols_total, int64_t ncols_shard, int64_t stride_row, int64_t chunk_cols, int64_t nparts,
                    void* const* peers, int world, int rank, void* buffer, void* out, void* stream) {
    nb200_params q;
    int rc = check_params(skeleton, params, &q);
    if (rc) return rc;
    if (!valid_dtype(dtype)) { set_error("nb200_peer_fold: unsupported dtype %d", dtype); return NB200_ERR_ARG; }
    if (world < 1 || world > peer_max_world() || rank < 0 || rank >= world) {
        set_error("nb200_peer_fold: need 1 <= world <= %d and 0 <= rank < world", peer_max_world());
        return NB200_ERR_ARG;
    }
    if (rows < 0 || ncols_shard < 1 || ncols_total < ncols_shard || chunk_cols < 1 || nparts < 1 || stride_row < 0) {
        set_error("nb200_peer_fold: need rows >= 0, 1 <= ncols_shard <= ncols_total, chunk_cols >= 1, nparts >= 1");
        return NB200_ERR_ARG;
    }
    if (!peers || !buffer || (rows > 0 && (!x || !out))) {
        set_error("nb200_peer_fold: null pointer");
        return NB200_ERR_ARG;
    }
    for (int r = 0; r < world; ++r)
        if (!peers[r] || (reinterpret_cast<uintptr_t>(peers[r]) & 255u)) {
            set_error("nb200_peer_fold: exchange buffer of rank %d is null or not 256-byte aligned", r);
            return NB200_ERR_ARG;
        }
    if (peers[rank] != buffer) {
        set_error("nb200_peer_fold: peers[rank] must be this rank's own buffer");
        return NB200_ERR_ARG;
    }
    if (rows == 0) return NB200_OK;
    return launch_peer_fold(skeleton, make_params(q, ncols_total), x, dtype, rows, ncols_shard, stride_row, chunk_cols,
                            nparts, peers, world, rank, buffer, out, (cudaStream_t)stream);
}

int nb200_peer_merge(int skeleton, const nb200_params* params, void* buffer, int64_t rows, int64_t nparts,
                     int world, void* out, int dtype, void* stream) {
    nb200_params q;
    int rc = check_params(skeleton, params, &q);
    if (rc) return rc;
    if (!valid_dtype(dtype)) { set_error("nb200_peer_merge: unsupported dtype %d", dtype); return NB200_ERR_ARG; }
    if (world < 1 || world > peer_max_world() || rows < 0 || nparts < 1) {
        set_error("nb200_peer_merge: need 1 <= world <= %d, rows >= 0, nparts >= 1", peer_max_world());
        return NB200_ERR_ARG;
    }
    if (!buffer || (rows > 0 && !out) || (reinterpret_cast<uintptr_t>(buffer) & 255u)) {
        set_error("nb200_peer_merge: null or unaligned pointer");
        return NB200_ERR_ARG;
    }
    return launch_peer_merge(skeleton, make_params(q, 0), buffer, rows, nparts, world, out, dtype,
                             (cudaStream_t)stream);
}

int nb200_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
    if (!ptr || !handle || !offset) { set_error("nb200_ipc_handle: null pointer"); return NB200_ERR_ARG; }
    static PFN_cuMemGetAddressRange_v3020 range = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
        cudaGetLastError();
    });
    CUdeviceptr base = 0;
    size_t size = 0;
    if (!range || range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        set_error("nb200_ipc_handle: %p is not device memory this process allocated", ptr);
        return NB200_ERR_ARG;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
        set_error("nb200_ipc_handle: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    std::memcpy(handle, &h, sizeof(h));
    *offset = (int64_t)(reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base);
    return NB200_OK;
}

int nb200_ipc_open(const void* handle, void** base) {
    if (!handle || !base) { set_error("nb200_ipc_open: null pointer"); return NB200_ERR_ARG; }
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    if (cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        set_error("nb200_ipc_open: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    return NB200_OK;
}

int nb200_ipc_close(void* base) {
    if (!base) { set_error("nb200_ipc_close: null pointer"); return NB200_ERR_ARG; }
    if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
        set_error("nb200_ipc_close: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    return NB200_OK;
}

int nb200_attention(const void* q, const void* k, const void* v, void* o, float* lse, int64_t batch,
                    int64_t heads, int64_t seq, int64_t head_dim, int causal, float scale, void* stream) {
    if (batch < 0 || heads < 0 || seq < 0) { set_error("nb200_attention: negative size"); return NB200_ERR_ARG; }
    if (batch * heads * seq == 0) return NB200_OK;
    if (!q || !k || !v || !o) { set_error("nb200_attention: null pointer"); return NB200_ERR_ARG; }
    if (!std::isfinite(scale)) { set_error("nb200_attention: scale must be finite"); return NB200_ERR_ARG; }
    return launch_attention(q, k, v, o, lse, batch, heads, seq, head_dim, causal, scale, (cudaStream_t)stream);
}

}  // extern "C"
