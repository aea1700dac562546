/*
 * neptune_b200.h -- C ABI of the B200 (sm_100a) backend for neptune-opt's fused
 * dependent-reduction hot path.
 *
 * Every entry point takes plain device pointers, element counts and element strides,
 * launches on the caller's CUDA stream and returns 0 (NB200_OK) or a negative
 * nb200_status. No C++ exception crosses this boundary. Inputs are never written.
 * Outputs and scratch are allocated by the caller; the library allocates no device
 * memory. nb200_last_error() returns a message for the last failing call on the
 * calling host thread.
 *
 * The entry points mirror the kernel launch signatures of the reference backend
 * (Defyli/neptune-opt, package neptune_codegen); each declaration names the launch it
 * replaces as file:line within that project.
 */
#ifndef NEPTUNE_B200_H
#define NEPTUNE_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status / types */
typedef enum {
    NB200_OK = 0,
    NB200_ERR_ARG = -1,         /* bad pointer, size, stride, dtype or parameter       */
    NB200_ERR_CAPACITY = -2,    /* request exceeds a documented capacity               */
    NB200_ERR_LAUNCH = -3,      /* the CUDA launch itself failed                       */
    NB200_ERR_TIMEOUT = -4,     /* a bounded device wait ran out                       */
    NB200_ERR_UNSUPPORTED = -5  /* valid request this build does not implement         */
} nb200_status;

/* Element types of row data (the reference accepts exactly these three:
 * neptune_codegen/template.py:346). */
typedef enum { NB200_F32 = 0, NB200_BF16 = 1, NB200_F16 = 2 } nb200_dtype;

/* Index types of segment descriptors (neptune_codegen/torch_op.py:358). */
typedef enum { NB200_I32 = 0, NB200_I64 = 1 } nb200_index_dtype;

/* The eleven scalar skeletons of neptune_codegen/library.py:19-177, compiled in. */
typedef enum {
    NB200_LOGSUMEXP = 0,    /* m + log(sum exp(x - m) + tiny)           library.py:19  */
    NB200_LSE_BIASED = 1,   /* logsumexp(x + alpha)                     library.py:100 */
    NB200_LSE_SCALED = 2,   /* logsumexp(x / T)                         library.py:157 */
    NB200_SOFTCAP_LSE = 3,  /* logsumexp(tanh(beta x))                  library.py:59  */
    NB200_STABLE_L2 = 4,    /* m sqrt(sum (x/m)^2), m = max|x|          library.py:32  */
    NB200_LINEAR_ATTN = 5,  /* sum x / max|x|                           library.py:40  */
    NB200_DECAY_RENORM = 6, /* sum x / (N + max|x|)                     library.py:49  */
    NB200_SUMSQ_DIV = 7,    /* sum x^2 / max|x|                         library.py:92  */
    NB200_RMSNORM_MAX = 8,  /* max x / sqrt(mean x^2 + eps)             library.py:72  */
    NB200_VARIANCE = 9,     /* two-pass mean((x - mean)^2)              library.py:114 */
    NB200_STD = 10,         /* two-pass sqrt(variance)                  library.py:143 */
    NB200_NUM_SKELETONS = 11
} nb200_skeleton;

/* Scalar parameters of a skeleton. Only the fields the skeleton declares are read
 * (library.py: tiny, alpha, T, beta, N, eps). Values arrive as binary64 exactly as the
 * reference bakes them into its source (emitters.py:300-327) and are narrowed to fp32
 * where the kernel computes. */
typedef struct {
    double tiny;
    double alpha;
    double T;
    double beta;
    double N;
    double eps;
} nb200_params;

/* Launch policy chosen by the host (neptune_codegen/autotune.py:222-250 picks Triton
 * (BLOCK, num_warps); here it picks a CUDA variant). Pass NULL for the library default. */
typedef enum {
    NB200_VARIANT_AUTO = 0,
    NB200_VARIANT_WARP_ROW = 1, /* one warp folds one row, register-resident chunks     */
    NB200_VARIANT_CTA_ROW = 2,  /* one CTA folds one row                                 */
    NB200_VARIANT_STREAM = 3,   /* bulk-copy staged rows (contiguous, 16-byte aligned)   */
    NB200_VARIANT_CLUSTER = 4   /* one thread-block cluster per row, CTA states merged   */
                                /* through distributed shared memory (contiguous,        */
                                /* 16-byte aligned rows; folds and RMSNorm)              */
} nb200_variant;

typedef struct {
    int32_t variant;        /* nb200_variant                                          */
    int32_t threads;        /* CTA size (64..512, x32); for NB200_VARIANT_STREAM the   */
                            /* number of warps, each owning its own ring of stages    */
    int32_t ctas_per_sm;    /* persistent grid = SMs * ctas_per_sm (0: default)       */
    int32_t stages;         /* NB200_VARIANT_STREAM: stages per warp ring (0: fit);   */
                            /* NB200_VARIANT_CLUSTER: CTAs per row, 2..16 (0: chosen) */
} nb200_launch;

/* One partial state of the repaired fold (emitters.py:436-519): raw producer value,
 * fp32 accumulator, "seen" flag and nonfinite status bits (bit 0 NaN, bit 1 +inf). */
typedef struct {
    float m;
    float acc;
    int32_t seen;
    int32_t status;
} nb200_state;

/* ------------------------------------------------------------------ library info */
const char* nb200_last_error(void);
const char* nb200_version(void);
/* Number of nb200 kernel launches issued by this process (for launch accounting). */
uint64_t nb200_launch_count(void);
/* Reads and clears the fault bits of the kernels with device-side waits or checks (bit 0: a
 * bounded wait on a bulk copy in a streaming kernel ran out and the kernel stopped early; bit 1: a
 * bounded wait in the attention kernel ran out and its output was left unwritten; bit 2: the peer
 * merge's bounded wait for the ranks' states ran out, those rows written as NaN; bit 3: a peer push or merge
 * found a buffer whose recorded layout differs from the call's, nothing stored or read).
 * Synchronous. No counterpart in the reference, whose Triton kernels have no device-side waits. */
int nb200_stream_fault(uint32_t* bits);

/* ------------------------------------------------------------------ a1: serial fold
 * Row-last repaired fold of one skeleton over a strided 2-D view x[rows, ncols]
 * (element strides stride_row, stride_col; any sign-free layout torch can express).
 * out[rows] is contiguous, in the input dtype. Replaces the serial launch
 * `kernel[(rows,)](x, out, rows, ncols, stride_row, stride_col, BLOCK=...)` of
 * neptune_codegen/template.py:376-378 (kernel body template.py:41-54 and the
 * two-pass body template.py:62-103). */
int nb200_fold(int skeleton, const nb200_params* params,
               const void* x, int dtype, int64_t rows, int64_t ncols,
               int64_t stride_row, int64_t stride_col,
               void* out, const nb200_launch* launch, void* stream);

/* Softmax-family readout fused into the log fold (the lowering of
 * neptune_recognize/lowering.py:80-99): mode 0 softmax exp(x - m) / s, mode 1
 * log_softmax (x - m) - log(s) with the reference's row-wide NaN for +inf rows.
 * y[rows, ncols] is contiguous in the input dtype; lse (nullable) receives the
 * logsumexp per row in the input dtype. */
int nb200_softmax(int mode, const void* x, int dtype, int64_t rows, int64_t ncols,
                  int64_t stride_row, int64_t stride_col,
                  void* y, void* lse, const nb200_launch* launch, void* stream);

/* Row L2 normalisation built on the stable_l2 fold (library.py:32-38): norm[rows]
 * (nullable) = m * sqrt(sum (x/m)^2) and y = x / norm, both in the input dtype. */
int nb200_l2_normalize(const void* x, int dtype, int64_t rows, int64_t ncols,
                       int64_t stride_row, int64_t stride_col,
                       void* y, void* norm, const nb200_launch* launch, void* stream);

/* ------------------------------------------------------------------ a2: split plan
 * Explicit split of each row into nparts column chunks of chunk_cols columns
 * (neptune_codegen/template.py:114-125, :137-165, launch :380-390). Chunk states go to
 * caller-owned scratch of nb200_fold_split_scratch_bytes(rows, nparts) bytes and are
 * merged in ascending chunk order. nparts = ceil(ncols / chunk_cols) <= 4096. */
int64_t nb200_fold_split_scratch_bytes(int64_t rows, int64_t nparts);
int nb200_fold_split(int skeleton, const nb200_params* params,
                     const void* x, int dtype, int64_t rows, int64_t ncols,
                     int64_t stride_row, int64_t stride_col, int64_t chunk_cols,
                     void* scratch, int64_t scratch_bytes, void* out,
                     const nb200_launch* launch, void* stream);

/* The split plan for callers that cannot allocate device memory (a host that hands over only its
 * input and output buffers, a fixed device-memory budget, a path where an allocation would
 * synchronise). Same arguments and result as nb200_fold_split minus the scratch: the chunk states
 * live in a 4 MiB array built into the library, which every GPU that loads the library holds until
 * exit. Limit: rows * ceil(ncols / chunk_cols) <= NB200_NOALLOC_MAX_STATES, else NB200_ERR_CAPACITY.
 * The first call on a device resolves the array's device address (make it before any stream
 * capture). Calls share the array: calls that overlap on the GPU race. Allocates nothing.
 * No counterpart in the reference, whose split plan always allocates its scratch with torch. */
#define NB200_NOALLOC_MAX_STATES 262144
int nb200_fold_split_noalloc(int skeleton, const nb200_params* params,
                             const void* x, int dtype, int64_t rows, int64_t ncols,
                             int64_t stride_row, int64_t stride_col, int64_t chunk_cols,
                             void* out, void* stream);

/* The two halves of the split plan, for callers that move states between devices.
 * nb200_fold_partial folds columns [col_begin, col_begin + ncols_shard) of every row in
 * chunk_cols chunks into states[rows * nparts] (nparts = ceil(ncols_shard / chunk_cols)).
 * nb200_fold_merge merges states laid out [rows][nparts] with element stride part_stride
 * between consecutive parts of a row and row_stride between rows, in ascending part
 * order, and finalises into out[rows] (input dtype). ncols_total is the full row width
 * (read by skeletons whose algebra uses N = ncols). */
int nb200_fold_partial(int skeleton, const nb200_params* params,
                       const void* x, int dtype, int64_t rows, int64_t ncols_total,
                       int64_t col_begin, int64_t ncols_shard,
                       int64_t stride_row, int64_t stride_col, int64_t chunk_cols,
                       nb200_state* states, const nb200_launch* launch, void* stream);
int nb200_fold_merge(int skeleton, const nb200_params* params,
                     const nb200_state* states, int64_t rows, int64_t nparts,
                     int64_t row_stride, int64_t part_stride,
                     void* out, int dtype, void* stream);

/* The split plan across GPUs without a collective (no counterpart in the reference, which has no
 * multi-GPU path): column shards' chunk states move through NVLink peer memory. Each rank owns an
 * exchange buffer of nb200_peer_buffer_bytes(rows, world, nparts) bytes (device memory, 256-byte
 * aligned, reused across calls), initialises it once with nb200_peer_init (which records the
 * (rows, world, nparts) layout in the buffer's header, clears its epoch and zeroes its slots), and maps
 * every other rank's buffer with nb200_ipc_handle / nb200_ipc_open (CUDA IPC; the library only
 * maps, it allocates nothing). Every rank initialises before any rank's first push (a barrier
 * between them). Per call, in this order on one stream:
 *   nb200_fold_partial  -> states[rows][nlocal] of this rank's shard;
 *   nb200_peer_push     -> writes them into slot `rank` (nparts wide, parts past nlocal empty) of
 *                          every rank's buffer (peers[r] = rank r's buffer as mapped here,
 *                          peers[rank] = buffer), each state tagged with the call's epoch inside
 *                          its 16 bytes (no fence, no flag);
 *   nb200_peer_merge    -> reads each state until it carries the call's epoch (bounded: about a
 *                          second, then bit 2 of nb200_stream_fault and the row reads NaN), merges
 *                          each row's world * nparts states in ascending (rank, part) order into
 *                          out[rows] -- the result of nb200_fold_merge on the gathered states.
 * Every rank makes the same calls in the same order with the same rows and nparts; a call's epoch
 * lives in the buffer, so the sequence may be captured in a CUDA graph and replayed. world <= 8.
 * Layout checks: before storing into a destination, the push kernel compares the call's
 * (rows, world, nparts) with the layout recorded in this rank's and the destination's header; the
 * merge compares its own. On a mismatch (or a buffer never initialised) nothing is stored or read,
 * bit 3 of nb200_stream_fault is set and the merge writes every row as NaN. After fault bit 2 or 3 the
 * ranks' epochs no longer agree: close the exchange on every rank and set it up again. */
int64_t nb200_peer_buffer_bytes(int64_t rows, int64_t world, int64_t nparts);
int nb200_peer_init(void* buffer, int64_t rows, int world, int64_t nparts, void* stream);
int nb200_peer_push(const nb200_state* states, int64_t rows, int64_t nlocal, int64_t nparts,
                    void* const* peers, int world, int rank, void* buffer, void* stream);
int nb200_peer_merge(int skeleton, const nb200_params* params, void* buffer, int64_t rows,
                     int64_t nparts, int world, void* out, int dtype, void* stream);
/* The same call in TWO launches (no counterpart in the reference): the partial fold of this rank's
 * column shard x[rows, ncols_shard] (contiguous rows, 16-byte aligned, row stride, width and
 * chunk_cols multiples of 16 bytes, chunks wider than 4 KB -- narrower ones return
 * NB200_ERR_UNSUPPORTED: use the push form) storing its tagged chunk states straight into every rank's
 * buffer (nb200_fold_partial + nb200_peer_push in one kernel), then the
 * merge of nb200_peer_merge. ncols_total (all ranks' columns) sets the skeletons' 1/N as in
 * nb200_fold_partial. Same buffers, layout checks, fault bits, epochs, parities and protocol as
 * the push/merge pair (the two forms may be mixed, across ranks and across calls), and the same
 * result bit for bit. */
int nb200_peer_fold(int skeleton, const nb200_params* params, const void* x, int dtype, int64_t rows,
                    int64_t ncols_total, int64_t ncols_shard, int64_t stride_row, int64_t chunk_cols, int64_t nparts,
                    void* const* peers, int world, int rank, void* buffer, void* out, void* stream);
/* CUDA IPC of a device allocation: handle (64 bytes) and the byte offset of ptr inside it; open
 * maps a peer's allocation (base; add the peer's offset), close unmaps it. */
int nb200_ipc_handle(const void* ptr, void* handle, int64_t* offset);
int nb200_ipc_open(const void* handle, void** base);
int nb200_ipc_close(void* base);

/* ------------------------------------------------------------------ a3: RMSNorm
 * out = round_in(x * rsqrt_rn(div_rn(sum x^2, ncols) + eps)) * gamma, rounded to the
 * input dtype; fp32 stages with no contraction (neptune_codegen/emitters.py:549-627,
 * launch template.py:294-319). out is contiguous [rows, ncols]. */
int nb200_rms_norm(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols,
                   int64_t stride_row, int64_t stride_col, int64_t stride_gamma,
                   double eps, void* out, const nb200_launch* launch, void* stream);

/* RMSNorm over rows held in HOST memory (no counterpart in the reference, whose ops take device
 * tensors): x[rows, ncols] and gamma[ncols] contiguous host buffers (page-locked for the copies to
 * overlap), y[rows, ncols] a host buffer. Rows move through the device in chunks of chunk_rows
 * (0: about 16 MiB per chunk): while chunk k runs on `stream`, chunk k+1 is copied in and chunk
 * k-1 copied back on two helper streams, so both PCIe directions are busy at once. The rows of y
 * equal nb200_rms_norm's on the same rows. work: device memory, 256-byte aligned, of
 * nb200_rms_norm_host_work_bytes(dtype, ncols, chunk_rows) bytes (gamma plus two input and two
 * output chunks). The copies wait for earlier work on `stream`, and `stream` waits for the last
 * copy back: y is complete once `stream` is. Calls on one device serialise their enqueueing. */
int64_t nb200_rms_norm_host_work_bytes(int dtype, int64_t ncols, int64_t chunk_rows);
int nb200_rms_norm_host(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols,
                        double eps, void* y, int64_t chunk_rows, void* work, int64_t work_bytes,
                        void* stream);

/* ------------------------------------------------------------------ a4/a5: segments
 * Descriptor status bits, ORed into a caller-owned device word (never a device assert):
 * 1 a length is negative or > nrows, 2 lengths do not cover nrows (checked unless unsafe),
 * 4 a boundary lies outside [0, nrows], 8 boundaries decrease. The word is sticky: the library
 * only sets bits, the caller clears it. */

/* Span construction from lengths (neptune_codegen/torch_op.py:370-387: cat(0, cumsum(lengths))
 * and its assertions): int64 spans[nsegments + 1] from lengths with element stride length_stride.
 * Offsets need no construction: nb200_segment_pool reads them directly. */
int nb200_segment_spans(const void* lengths, int index_dtype, int64_t nsegments, int64_t length_stride,
                        int unsafe, int64_t nrows, int64_t* spans, uint32_t* status, void* stream);

/* Ordered storage-dtype pooling (neptune_codegen/torch_op.py:254-306, launch :390-410): for each
 * segment s and channel c, acc = initial, then for every row r in [bounds[s], bounds[s+1]) in order
 * acc = round_storage(acc + data[r, c]); reduce 0 sum, 1 mean = div_rn(acc,
 * float(round_storage(count))). Empty mean without initial and malformed boundaries give NaN.
 * bounds are nsegments + 1 CSR boundaries (int32 or int64, element stride bound_stride), validated
 * in the kernel into *status (nullable). initial_bits is the fp32 bit pattern of `initial`. out is
 * contiguous [nsegments, channels]. */
int nb200_segment_pool(const void* data, int dtype, int64_t nrows, int64_t channels,
                       int64_t stride_row, int64_t stride_channel,
                       const void* bounds, int index_dtype, int64_t bound_stride, int64_t nsegments,
                       int reduce, int has_initial, uint32_t initial_bits, void* out,
                       uint32_t* status, void* stream);

/* ------------------------------------------------------------------ a9: attention
 * O = softmax(scale * Q K^T [+ causal mask]) V per (batch, head), bf16 in/out with
 * fp32 online max/sum repair; lse (nullable) receives fp32 natural log-sum-exp of the scaled
 * scores per query row, [B, H, S]. Q, K, V, O are contiguous [B, H, S, D], 16-byte aligned;
 * head_dim must be 128 (else NB200_ERR_UNSUPPORTED) and scale > 0. causal != 0 masks key > query.
 * No counterpart in the reference (its roadmap declares attention out of scope:
 * docs/roadmap.md:28-31). */
int nb200_attention(const void* q, const void* k, const void* v, void* o, float* lse,
                    int64_t batch, int64_t heads, int64_t seq, int64_t head_dim,
                    int causal, float scale, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NEPTUNE_B200_H */
