// Register-row kernel for contiguous rows of 1-8 KB on sm_100a.
//
// One warp per row: all of the row's 16-byte vectors are loaded with plain vector loads at once
// (NV per lane, every load in flight together), then the fused Op (row_ops.cuh) runs on the
// registers -- both passes of the fold and the readout store -- so the row is read from HBM
// once with nothing staged. Rows go to warps round-robin, so the rows being read at any moment
// form one contiguous band of the tensor. Read-heavy rows of this size reach more of HBM's
// bandwidth this way than with per-warp bulk copies into shared memory (measured on B200: a
// plain-load reader sustains ~5.8 TB/s on a 67 MB read, the bulk-copy ring ~4.1 TB/s).
#include "launch.h"
#include "row_ops.cuh"

namespace nb200 {

constexpr int kLdgThreads = 128;

template <typename T, class Op, int NV>
__global__ void __launch_bounds__(kLdgThreads) ldg_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t srow,
                                                               Op op) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) unsigned char smem[];
    op.prologue(smem);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int64_t gw = (int64_t)blockIdx.x * (kLdgThreads / 32) + (threadIdx.x >> 5);
    const int64_t GW = (int64_t)gridDim.x * (kLdgThreads / 32);
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
    auto k = ldg_rows_kernel<T, Op, NV>;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kLdgThreads, smem) != cudaSuccess || occ < 1) occ = 1;
    const int64_t need = (rows + kLdgThreads / 32 - 1) / (kLdgThreads / 32);
    const int g = (int)std::min<int64_t>(need, (int64_t)sm_count() * occ);
    launch_pdl(k, (unsigned)std::max(g, 1), kLdgThreads, smem, st, x, rows, srow, op);
    count_launch();
    return finish_launch(what);
}

template <typename T, class Op>
int launch_ldg_rows(const T* x, int64_t rows, int64_t srow, const Op& op, uint32_t smem, cudaStream_t st,
                    const char* what) {
    if (op.nv <= 32 * 4) return launch_ldg_nv<T, Op, 4>(x, rows, srow, op, smem, st, what);
    return launch_ldg_nv<T, Op, 16>(x, rows, srow, op, smem, st, what);
}

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
