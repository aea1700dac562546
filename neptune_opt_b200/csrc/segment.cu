// Ordered storage-dtype segment pooling over CSR spans, and the span construction in front of it.
//
// Reference: the generated segment kernel neptune_codegen/torch_op.py:254-306 (launch :390-410)
// and the ATen span prefix with its four asynchronous assertions torch_op.py:370-387.
//
// Numeric contract (skeleton.py:218-221): per segment and channel, acc starts at the storage-dtype
// value of `initial` (0 when absent) and every row of the segment, in row order, is added in fp32
// and rounded to the storage dtype (round to nearest even) before the next add. fp32 holds at least
// 2p + 2 bits of a 16-bit format's p-bit significand, so this single rounding of the fp32 sum equals
// the correctly rounded storage-dtype sum. Mean divides the pooled value by the row count converted
// to the storage dtype, with IEEE division. Parallelism is only across segments and channels.
//
// Validation never traps the GPU: violations are reported as bits in a status word, and spans that
// are malformed make their segment NaN without issuing a data load.
#include "common.cuh"
#include "launch.h"

namespace nb200 {

// ------------------------------------------------------------------ spans (a single CTA)
__device__ __forceinline__ int64_t warp_incl_scan(int64_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int64_t u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    return v;
}

template <typename I>
__global__ void __launch_bounds__(1024)
spans_kernel(const I* __restrict__ seg, int64_t nseg, int64_t ss, int is_offsets, int unsafe,
             int64_t nrows, int64_t* __restrict__ spans, uint32_t* __restrict__ status) {
    __shared__ int64_t warp_tot[32];
    __shared__ unsigned int st_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    if (tid == 0) st_s = 0u;
    __syncthreads();
    unsigned int st = 0u;
    if (is_offsets) {
        for (int64_t i = tid; i <= nseg; i += blockDim.x) {
            const int64_t o = (int64_t)seg[i * ss];
            spans[i] = o;
            if (o < 0 || o > nrows) st |= 4u;
            if (i > 0 && (int64_t)seg[(i - 1) * ss] > o) st |= 8u;
        }
    } else {
        constexpr int ITEMS = 8;
        const int64_t tile = (int64_t)blockDim.x * ITEMS;
        int64_t carry = 0;
        for (int64_t base = 0; base < nseg; base += tile) {
            int64_t v[ITEMS];
            int64_t local = 0;
#pragma unroll
            for (int it = 0; it < ITEMS; ++it) {
                const int64_t idx = base + (int64_t)tid * ITEMS + it;
                v[it] = idx < nseg ? (int64_t)seg[idx * ss] : 0;
                if (idx < nseg && (v[it] < 0 || v[it] > nrows)) st |= 1u;
                local += v[it];
            }
            const int64_t incl = warp_incl_scan(local);
            if (lane == 31) warp_tot[warp] = incl;
            __syncthreads();
            int64_t before = 0, total = 0;
            for (int w = 0; w < nw; ++w) {
                if (w < warp) before += warp_tot[w];
                total += warp_tot[w];
            }
            int64_t run = carry + before + (incl - local);
#pragma unroll
            for (int it = 0; it < ITEMS; ++it) {
                const int64_t idx = base + (int64_t)tid * ITEMS + it;
                if (idx < nseg) {
                    spans[idx] = run;
                    if (run < 0 || run > nrows) st |= 4u;
                    if (v[it] < 0) st |= 8u;
                }
                run += v[it];
            }
            carry += total;
            __syncthreads();  // warp_tot is rewritten by the next tile
        }
        if (tid == 0) {
            spans[nseg] = carry;
            if (carry < 0 || carry > nrows) st |= 4u;
            if (!unsafe && carry != nrows) st |= 2u;
        }
    }
    if (st) atomicOr(&st_s, st);
    __syncthreads();
    if (tid == 0) *status = st_s;
}

// ------------------------------------------------------------------ pooling
template <typename T, int CV> struct ChanVec;
template <> struct ChanVec<float, 4> {
    using raw = uint4;
    __device__ __forceinline__ static raw load(const float* p) { return __ldcs(reinterpret_cast<const uint4*>(p)); }
    __device__ __forceinline__ static float get(const raw& r, int j) { return Elem<float>::lane(r, j); }
};
template <> struct ChanVec<__nv_bfloat16, 4> {
    using raw = uint2;
    __device__ __forceinline__ static raw load(const __nv_bfloat16* p) { return __ldcs(reinterpret_cast<const uint2*>(p)); }
    __device__ __forceinline__ static float get(const raw& r, int j) {
        const uint32_t w = (j >> 1) ? r.y : r.x;
        return __uint_as_float((j & 1) ? (w & 0xffff0000u) : (w << 16));
    }
};
template <> struct ChanVec<__half, 4> {
    using raw = uint2;
    __device__ __forceinline__ static raw load(const __half* p) { return __ldcs(reinterpret_cast<const uint2*>(p)); }
    __device__ __forceinline__ static float get(const raw& r, int j) {
        const uint32_t w = (j >> 1) ? r.y : r.x;
        return __half2float(__ushort_as_half((unsigned short)((j & 1) ? (w >> 16) : (w & 0xffffu))));
    }
};

// Round an fp32 value to the storage dtype and back (identity for fp32 storage).
template <typename T>
__device__ __forceinline__ float rs(float v) { return Elem<T>::to_f(Elem<T>::from_f(v)); }

// One warp per (segment, channel tile of 32 * CV channels). Rows are folded strictly in order;
// UNROLL rows are loaded ahead so the dependent adds overlap the loads.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256)
pool_kernel(const T* __restrict__ data, const int64_t* __restrict__ spans, T* __restrict__ out,
            int64_t nrows, int64_t channels, int64_t srow, int64_t sch, int64_t nseg, int reduce,
            int has_initial, uint32_t initial_bits) {
    constexpr int CV = 4;
    constexpr int UNROLL = 8;
    using CVec = ChanVec<T, CV>;
    const int lane = threadIdx.x & 31;
    const int64_t gid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t ng = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t ntiles = (channels + 32 * CV - 1) / (32 * CV);
    const float init = has_initial ? rs<T>(__uint_as_float(initial_bits)) : 0.f;
    for (int64_t w = gid; w < nseg * ntiles; w += ng) {
        const int64_t s = w / ntiles, tile = w - s * ntiles;
        const int64_t start = spans[s], end = spans[s + 1];
        const bool valid = start >= 0 && end >= start && end <= nrows;
        const int64_t c_base = tile * 32 * CV + (int64_t)lane * CV;
        float acc[CV];
#pragma unroll
        for (int j = 0; j < CV; ++j) acc[j] = init;
        if (valid) {
            for (int64_t tok = start; tok < end; tok += UNROLL) {
                float vals[UNROLL][CV];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    const int64_t rr = tok + u;
                    if (VEC) {
                        typename CVec::raw raw{};
                        if (rr < end && c_base < channels) raw = CVec::load(data + rr * srow + c_base);
#pragma unroll
                        for (int j = 0; j < CV; ++j) vals[u][j] = CVec::get(raw, j);
                    } else {
#pragma unroll
                        for (int j = 0; j < CV; ++j) {
                            const int64_t c = c_base + j;
                            vals[u][j] = (rr < end && c < channels) ? Elem<T>::to_f(data[rr * srow + c * sch]) : 0.f;
                        }
                    }
                }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                    if (tok + u < end) {
#pragma unroll
                        for (int j = 0; j < CV; ++j) acc[j] = rs<T>(__fadd_rn(acc[j], vals[u][j]));
                    }
            }
        }
        const int64_t n = end - start;
        const float den = rs<T>(__ll2float_rn(n));
#pragma unroll
        for (int j = 0; j < CV; ++j) {
            const int64_t c = c_base + j;
            if (c >= channels) continue;
            float res = acc[j];
            if (reduce == 1) {
                res = __fdiv_rn(acc[j], den);
                if (n == 0) res = has_initial ? acc[j] : NB200_NAN;
            }
            if (!valid) res = NB200_NAN;
            out[s * channels + c] = Elem<T>::from_f(res);
        }
    }
}

namespace {

template <typename T>
int pool_t(const T* data, int64_t nrows, int64_t channels, int64_t srow, int64_t sch,
           const int64_t* spans, int64_t nseg, int reduce, int has_initial, uint32_t bits, T* out,
           cudaStream_t st) {
    constexpr int CV = 4;
    const int64_t vbytes = CV * (int64_t)sizeof(T);
    const bool vec = sch == 1 && channels % CV == 0 &&
                     (reinterpret_cast<uintptr_t>(data) % (uintptr_t)vbytes) == 0 &&
                     (nrows <= 1 || (srow * (int64_t)sizeof(T)) % vbytes == 0);
    auto k = vec ? pool_kernel<T, true> : pool_kernel<T, false>;
    const int64_t ntiles = (channels + 32 * CV - 1) / (32 * CV);
    const int g = persistent_grid(k, 256, 0, (nseg * ntiles + 7) / 8, 0);
    k<<<g, 256, 0, st>>>(data, spans, out, nrows, channels, srow, sch, nseg, reduce, has_initial, bits);
    count_launch();
    return finish_launch("nb200_segment_pool");
}

}  // namespace

int launch_spans(const void* seg, int idt, int64_t nseg, int64_t sstride, int is_offsets,
                 int unsafe, int64_t nrows, int64_t* spans, uint32_t* status, cudaStream_t st) {
    if (idt == NB200_I32)
        spans_kernel<int32_t><<<1, 1024, 0, st>>>((const int32_t*)seg, nseg, sstride, is_offsets, unsafe,
                                                   nrows, spans, status);
    else
        spans_kernel<int64_t><<<1, 1024, 0, st>>>((const int64_t*)seg, nseg, sstride, is_offsets, unsafe,
                                                   nrows, spans, status);
    count_launch();
    return finish_launch("nb200_segment_spans");
}

int launch_segment_pool(const void* data, int dtype, int64_t nrows, int64_t channels,
                        int64_t srow, int64_t sch, const int64_t* spans, int64_t nseg, int reduce,
                        int has_initial, uint32_t initial_bits, void* out, cudaStream_t st) {
    switch (dtype) {
        case NB200_F32:
            return pool_t<float>((const float*)data, nrows, channels, srow, sch, spans, nseg, reduce,
                                 has_initial, initial_bits, (float*)out, st);
        case NB200_BF16:
            return pool_t<__nv_bfloat16>((const __nv_bfloat16*)data, nrows, channels, srow, sch, spans, nseg,
                                         reduce, has_initial, initial_bits, (__nv_bfloat16*)out, st);
        case NB200_F16:
            return pool_t<__half>((const __half*)data, nrows, channels, srow, sch, spans, nseg, reduce,
                                  has_initial, initial_bits, (__half*)out, st);
    }
    set_error("unknown dtype %d", dtype);
    return NB200_ERR_ARG;
}

}  // namespace nb200
