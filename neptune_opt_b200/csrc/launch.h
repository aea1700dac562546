// Internal host-side launchers shared by the kernel files and the C ABI (capi.cu). All return an
// nb200_status and record a message on failure.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/neptune_b200.h"

namespace nb200 {

struct Params;
Params make_params(const nb200_params& q, int64_t ncols);

int launch_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols,
                int64_t srow, int64_t scol, void* out, const nb200_launch* L, cudaStream_t st);
int launch_softmax(int mode, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow,
                   int64_t scol, void* y, void* lse, const nb200_launch* L, cudaStream_t st);
int launch_l2(const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
              void* y, void* norm, const nb200_launch* L, cudaStream_t st);
int launch_partial(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t cb,
                   int64_t ns, int64_t srow, int64_t scol, int64_t cc, int64_t nparts,
                   nb200_state* states, const nb200_launch* L, cudaStream_t st);
int launch_merge(int sk, const Params& p, const nb200_state* states, int64_t rows, int64_t nparts,
                 int64_t rs, int64_t ps, void* out, int dtype, cudaStream_t st);

// Few, very wide rows in one launch: a thread-block cluster of csize CTAs per row whose states
// (fold) or partial sums of squares (RMSNorm) meet through distributed shared memory
// (rows_ldg.cu). x, gamma, y 16-byte aligned, contiguous rows whose byte length and stride are
// 16-byte multiples. csize 0 picks the cluster size. Return 1 when launched, 0 when not taken,
// negative on error.
template <typename T>
int launch_cluster_fold(int sk, const Params& p, const T* x, int64_t rows, int64_t ncols, int64_t srow, T* out,
                        int csize, cudaStream_t st);
template <typename T>
int launch_cluster_rms(const T* x, const T* gamma, int64_t rows, int64_t ncols, int64_t srow, float eps, T* y,
                       int csize, cudaStream_t st);

// Column-sharded split plan across GPUs: chunk states exchanged through peer memory (fold.cu).
int64_t peer_buffer_bytes(int64_t rows, int64_t world, int64_t nparts);
int peer_max_world();
int launch_peer_init(void* buffer, int64_t rows, int64_t nparts, int world, cudaStream_t st);
int launch_peer_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols_shard,
                     int64_t srow, int64_t chunk, int64_t nparts, void* const* peers, int world, int rank, void* own,
                     void* out, cudaStream_t st);
int launch_peer_push(const nb200_state* states, int64_t rows, int64_t nlocal, int64_t nparts, void* const* peers,
                     int world, int rank, void* own, cudaStream_t st);
int launch_peer_merge(int sk, const Params& p, void* own, int64_t rows, int64_t nparts, int world, void* out,
                      int dtype, cudaStream_t st);
int peer_fault_take(unsigned int* bits);

int launch_rms(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols,
               int64_t srow, int64_t scol, int64_t sg, float eps, void* out,
               const nb200_launch* L, cudaStream_t st);

int launch_spans(const void* seg, int idt, int64_t nseg, int64_t sstride, int unsafe, int64_t nrows,
                 int64_t* spans, uint32_t* status, cudaStream_t st);
int launch_segment_pool(const void* data, int dtype, int64_t nrows, int64_t channels, int64_t srow, int64_t sch,
                        const void* bounds, int idt, int64_t bs, int64_t nseg, int reduce, int has_initial,
                        uint32_t initial_bits, void* out, uint32_t* status, cudaStream_t st);

// Streaming (bulk-copy staged) paths: return 1 when launched, 0 when the input is not eligible
// (the caller then uses the register-tiled kernels), negative on error.
int stream_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow,
                int64_t scol, void* out, const nb200_launch* L, cudaStream_t st);
int stream_softmax(int mode, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
                   void* y, void* lse, const nb200_launch* L, cudaStream_t st);
int stream_l2(const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol, void* y, void* norm,
              const nb200_launch* L, cudaStream_t st);
int stream_rms(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
               int64_t sg, float eps, void* y, const nb200_launch* L, cudaStream_t st);
int stream_span(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t cb, int64_t ns,
                int64_t srow, int64_t scol, int64_t cc, int64_t nparts, nb200_state* states, void* out,
                int finalize, const nb200_launch* L, cudaStream_t st);
int stream_fault_take(unsigned int* bits);
int attn_fault_take(unsigned int* bits);

int launch_attention(const void* q, const void* k, const void* v, void* o, float* lse,
                     int64_t B, int64_t H, int64_t S, int64_t D, int causal, float scale,
                     cudaStream_t st);

}  // namespace nb200
