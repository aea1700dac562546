// Ordered storage-dtype segment pooling over CSR boundaries, and the span construction from lengths.
//
// Reference: the generated segment kernel neptune_codegen/torch_op.py:254-306 (launch :390-410)
// and the ATen span prefix with its four asynchronous assertions torch_op.py:370-387.
//
// Numeric contract (skeleton.py:218-221): per segment and channel, acc starts at the storage-dtype
// value of `initial` (0 when absent) and every row of the segment, in row order, is added in fp32
// and rounded to the storage dtype (round to nearest even) before the next add. fp32 carries at
// least 2p + 2 significand bits of a p-bit storage format (p = 11 for fp16, 8 for bf16), so that
// double rounding is innocuous: the fp32 sum rounded once to the storage dtype equals the
// correctly rounded storage-dtype sum. The kernel therefore adds in the storage dtype directly,
// two channels per instruction (add.rn.f16x2 / add.rn.bf16x2), which is bit-identical. Mean
// divides the pooled value by the row count converted to the storage dtype, with IEEE division.
// Parallelism is only across segments and channels; rows of a segment are folded in order.
//
// Validation never traps the GPU: descriptor violations are ORed into a caller-owned status word
// (1 length negative or > nrows, 2 lengths do not cover nrows, 4 boundary outside [0, nrows],
// 8 boundaries decreasing), and a segment whose boundaries are malformed pools to NaN without
// reading data.
#include "common.cuh"
#include "launch.h"

namespace nb200 {

// ------------------------------------------------------------------ spans from lengths (one CTA)
// Each of the 1024 threads owns a contiguous run of lengths: pass 1 sums the run, one block scan
// turns the run sums into run offsets, pass 2 writes the exclusive prefix of every element.
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
spans_kernel(const I* __restrict__ seg, int64_t nseg, int64_t ss, int unsafe, int64_t nrows,
             int64_t* __restrict__ spans, uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t warp_tot[32];
    __shared__ unsigned int st_s;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    if (tid == 0) st_s = 0u;
    const int64_t per = (nseg + blockDim.x - 1) / blockDim.x;
    const int64_t lo = min((int64_t)tid * per, nseg), hi = min(lo + per, nseg);
    unsigned int st = 0u;
    int64_t local = 0;
    for (int64_t i = lo; i < hi; ++i) {
        const int64_t v = (int64_t)seg[i * ss];
        if (v < 0 || v > nrows) st |= 1u;
        if (v < 0) st |= 8u;
        local += v;
    }
    const int64_t incl = warp_incl_scan(local);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int64_t before = 0, total = 0;
    for (int w = 0; w < nw; ++w) {
        if (w < warp) before += warp_tot[w];
        total += warp_tot[w];
    }
    int64_t run = before + (incl - local);
    for (int64_t i = lo; i < hi; ++i) {
        spans[i] = run;
        if (run < 0 || run > nrows) st |= 4u;
        run += (int64_t)seg[i * ss];
    }
    if (tid == 0) {
        spans[nseg] = total;
        if (total < 0 || total > nrows) st |= 4u;
        if (!unsafe && total != nrows) st |= 2u;
    }
    if (st) atomicOr(&st_s, st);
    __syncthreads();
    if (tid == 0 && st_s && status) atomicOr(status, st_s);
}

// ------------------------------------------------------------------ spans, many CTAs
// For long length vectors the single-CTA scan above would leave one SM streaming the whole vector.
// Three launches split it without scratch memory or waits between CTAs: blocks of kSpanChunk
// lengths each own spans[b*kSpanChunk + 1 .. (b+1)*kSpanChunk], and the first slot of that range
// carries the block's sum (K1), then its exclusive offset (K2), before K3 -- which reads only its
// own slot -- overwrites the range with the final boundaries. Status bits as spans_kernel.
constexpr int kSpanChunkThreads = 256;
constexpr int kSpanPerThread = 16;
constexpr int64_t kSpanChunk = (int64_t)kSpanChunkThreads * kSpanPerThread;

__device__ __forceinline__ int64_t block_excl_scan(int64_t v, int64_t* warp_tot, int64_t& total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    const int64_t incl = warp_incl_scan(v);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int64_t before = 0;
    total = 0;
    for (int w = 0; w < nw; ++w) {
        if (w < warp) before += warp_tot[w];
        total += warp_tot[w];
    }
    __syncthreads();
    return before + incl - v;
}

template <typename I>
__global__ void __launch_bounds__(kSpanChunkThreads)
spans_sum_kernel(const I* __restrict__ seg, int64_t nseg, int64_t ss, int64_t nrows, int64_t* __restrict__ spans,
                 uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t warp_tot[32];
    const int64_t b0 = (int64_t)blockIdx.x * kSpanChunk;
    const int64_t lo = b0 + (int64_t)threadIdx.x * kSpanPerThread, hi = min(lo + kSpanPerThread, nseg);
    unsigned int st = 0u;
    int64_t local = 0;
    for (int64_t i = lo; i < hi; ++i) {
        const int64_t v = (int64_t)seg[i * ss];
        if (v < 0 || v > nrows) st |= 1u;
        if (v < 0) st |= 8u;
        local += v;
    }
    int64_t total;
    block_excl_scan(local, warp_tot, total);
    if (threadIdx.x == 0) spans[b0 + 1] = total;
    st = __reduce_or_sync(0xffffffffu, st);
    if ((threadIdx.x & 31) == 0 && st && status) atomicOr(status, st);
}

__global__ void __launch_bounds__(1024)
spans_offsets_kernel(int64_t nseg, int64_t nblocks, int unsafe, int64_t nrows, int64_t* __restrict__ spans,
                     uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t warp_tot[32];
    const int64_t per = (nblocks + blockDim.x - 1) / blockDim.x;
    const int64_t lo = min((int64_t)threadIdx.x * per, nblocks), hi = min(lo + per, nblocks);
    int64_t local = 0;
    for (int64_t b = lo; b < hi; ++b) local += spans[b * kSpanChunk + 1];
    int64_t total;
    int64_t run = block_excl_scan(local, warp_tot, total);
    for (int64_t b = lo; b < hi; ++b) {
        const int64_t sum = spans[b * kSpanChunk + 1];
        spans[b * kSpanChunk + 1] = run;
        run += sum;
    }
    if (threadIdx.x == 0) {
        spans[0] = 0;
        unsigned int st = 0u;
        if (total < 0 || total > nrows) st |= 4u;
        if (!unsafe && total != nrows) st |= 2u;
        if (st && status) atomicOr(status, st);
    }
}

template <typename I>
__global__ void __launch_bounds__(kSpanChunkThreads)
spans_write_kernel(const I* __restrict__ seg, int64_t nseg, int64_t ss, int64_t nrows, int64_t* __restrict__ spans,
                   uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    __shared__ int64_t warp_tot[32];
    __shared__ int64_t offset;
    const int64_t b0 = (int64_t)blockIdx.x * kSpanChunk;
    if (threadIdx.x == 0) offset = spans[b0 + 1];
    const int64_t lo = b0 + (int64_t)threadIdx.x * kSpanPerThread, hi = min(lo + kSpanPerThread, nseg);
    int64_t v[kSpanPerThread];
    int64_t local = 0;
#pragma unroll
    for (int k = 0; k < kSpanPerThread; ++k) {
        v[k] = lo + k < hi ? (int64_t)seg[(lo + k) * ss] : 0;
        local += v[k];
    }
    int64_t total;
    int64_t run = block_excl_scan(local, warp_tot, total);  // its barriers also publish `offset`
    run += offset;
    unsigned int st = 0u;
#pragma unroll
    for (int k = 0; k < kSpanPerThread; ++k) {
        if (lo + k < hi) {
            run += v[k];
            spans[lo + k + 1] = run;
            if (run < 0 || run > nrows) st |= 4u;
        }
    }
    st = __reduce_or_sync(0xffffffffu, st);
    if ((threadIdx.x & 31) == 0 && st && status) atomicOr(status, st);
}

// ------------------------------------------------------------------ pooling
template <typename T> struct Pack;
template <> struct Pack<__half> {
    __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t splat(float v) {
        __half2 h = __float2half2_rn(v);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <> struct Pack<__nv_bfloat16> {
    __device__ __forceinline__ static uint32_t add(uint32_t a, uint32_t b) {
        uint32_t d;
        asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
        return d;
    }
    __device__ __forceinline__ static uint32_t splat(float v) {
        __nv_bfloat162 h = __float2bfloat162_rn(v);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

// Round an fp32 value to the storage dtype and back (identity for fp32 storage).
template <typename T>
__device__ __forceinline__ float rs(float v) { return Elem<T>::to_f(Elem<T>::from_f(v)); }

template <typename I>
__device__ __forceinline__ void segment_bounds(const I* b, int64_t bs, int64_t s, int64_t nrows, int64_t& start,
                                               int64_t& end, unsigned int& st) {
    start = (int64_t)b[s * bs];
    end = (int64_t)b[(s + 1) * bs];
    if (start < 0 || start > nrows || end < 0 || end > nrows) st |= 4u;
    if (end < start) st |= 8u;
}

// Readout of one pooled fp32 value (already a storage-dtype value).
template <typename T>
__device__ __forceinline__ float pool_readout(float acc, int64_t n, bool valid, int reduce, int has_initial) {
    float res = acc;
    if (reduce == 1) {
        res = __fdiv_rn(acc, rs<T>(__ll2float_rn(n)));
        if (n == 0) res = has_initial ? acc : NB200_NAN;
    }
    return valid ? res : NB200_NAN;
}

// 16-bit storage, channels a multiple of 8 and 16-byte-aligned rows: each lane owns 8 channels
// (one 16-byte vector per row), LPS lanes cover a row tile of 8 * LPS channels, and one warp
// folds 32 / LPS (segment, channel tile) items at once.
template <typename T, typename I, int LPS>
__global__ void __launch_bounds__(256)
pool16_kernel(const T* __restrict__ data, const I* __restrict__ bounds, int64_t bs, T* __restrict__ out,
              int64_t nrows, int64_t channels, int64_t srow, int64_t nseg, int reduce, int has_initial,
              uint32_t initial_bits, uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    constexpr int G = 32 / LPS, UNROLL = 8;
    const int lane = threadIdx.x & 31, sub = lane / LPS, sl = lane % LPS;
    const int64_t ntiles = (channels + 8 * LPS - 1) / (8 * LPS);
    const int64_t nitems = nseg * ntiles;
    const int64_t gw = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t GW = (int64_t)gridDim.x * (blockDim.x >> 5);
    const float init = has_initial ? rs<T>(__uint_as_float(initial_bits)) : 0.f;
    const uint32_t init2 = Pack<T>::splat(init);
    unsigned int st = 0u;
    for (int64_t base = gw * G; base < nitems; base += GW * G) {
        const int64_t w = base + sub;
        if (w >= nitems) continue;
        const int64_t s = w / ntiles, tile = w - s * ntiles;
        int64_t start, end;
        segment_bounds(bounds, bs, s, nrows, start, end, st);
        const bool valid = start >= 0 && end >= start && end <= nrows;
        const int64_t c = tile * 8 * LPS + (int64_t)sl * 8;
        const bool active = c < channels;
        uint32_t acc[4] = {init2, init2, init2, init2};
        if (valid && active) {
            const T* p = data + start * srow + c;
            for (int64_t tok = start; tok < end; tok += UNROLL, p += UNROLL * srow) {
                uint4 v[UNROLL];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) v[u] = (tok + u < end) ? ld_stream(p + u * srow) : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int u = 0; u < UNROLL; ++u) {
                    if (tok + u < end) {
                        acc[0] = Pack<T>::add(acc[0], v[u].x);
                        acc[1] = Pack<T>::add(acc[1], v[u].y);
                        acc[2] = Pack<T>::add(acc[2], v[u].z);
                        acc[3] = Pack<T>::add(acc[3], v[u].w);
                    }
                }
            }
        }
        if (!active) continue;
        const uint4 a = make_uint4(acc[0], acc[1], acc[2], acc[3]);
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) f[e] = pool_readout<T>(Elem<T>::lane(a, e), end - start, valid, reduce, has_initial);
        T* o = out + s * channels + c;
        if ((reinterpret_cast<uintptr_t>(o) & 15u) == 0) {
            st_stream(o, Elem<T>::pack(f));
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = Elem<T>::from_f(f[e]);
        }
    }
    if (st && status) atomicOr(status, st);
}

// General layout (any strides, fp32 or unaligned 16-bit): one warp per (segment, 128-channel
// tile), four channels per lane, scalar loads, fp32 adds rounded to the storage dtype.
template <typename T, typename I>
__global__ void __launch_bounds__(256)
pool_kernel(const T* __restrict__ data, const I* __restrict__ bounds, int64_t bs, T* __restrict__ out,
            int64_t nrows, int64_t channels, int64_t srow, int64_t sch, int64_t nseg, int reduce, int has_initial,
            uint32_t initial_bits, uint32_t* __restrict__ status) {
    pdl_wait();
    pdl_trigger();
    constexpr int CV = 4, UNROLL = 8;
    const int lane = threadIdx.x & 31;
    const int64_t gid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t ng = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int64_t ntiles = (channels + 32 * CV - 1) / (32 * CV);
    const float init = has_initial ? rs<T>(__uint_as_float(initial_bits)) : 0.f;
    unsigned int st = 0u;
    for (int64_t w = gid; w < nseg * ntiles; w += ng) {
        const int64_t s = w / ntiles, tile = w - s * ntiles;
        int64_t start, end;
        segment_bounds(bounds, bs, s, nrows, start, end, st);
        const bool valid = start >= 0 && end >= start && end <= nrows;
        const int64_t c_base = tile * 32 * CV + (int64_t)lane * CV;
        float acc[CV];
#pragma unroll
        for (int j = 0; j < CV; ++j) acc[j] = init;
        if (valid) {
            for (int64_t tok = start; tok < end; tok += UNROLL) {
                float vals[UNROLL][CV];
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
#pragma unroll
                    for (int j = 0; j < CV; ++j) {
                        const int64_t c = c_base + j;
                        vals[u][j] = (tok + u < end && c < channels) ? Elem<T>::to_f(data[(tok + u) * srow + c * sch]) : 0.f;
                    }
#pragma unroll
                for (int u = 0; u < UNROLL; ++u)
                    if (tok + u < end) {
#pragma unroll
                        for (int j = 0; j < CV; ++j) acc[j] = rs<T>(__fadd_rn(acc[j], vals[u][j]));
                    }
            }
        }
#pragma unroll
        for (int j = 0; j < CV; ++j) {
            const int64_t c = c_base + j;
            if (c < channels) out[s * channels + c] = Elem<T>::from_f(pool_readout<T>(acc[j], end - start, valid, reduce, has_initial));
        }
    }
    if (st && status) atomicOr(status, st);
}

namespace {

template <typename T, typename I>
int pool_t(const T* data, int64_t nrows, int64_t channels, int64_t srow, int64_t sch, const I* bounds, int64_t bs,
           int64_t nseg, int reduce, int has_initial, uint32_t bits, T* out, uint32_t* status, cudaStream_t st) {
    const bool vec16 = sizeof(T) == 2 && sch == 1 && channels % 8 == 0 && aligned16(data) &&
                       (nrows <= 1 || (srow * (int64_t)sizeof(T)) % 16 == 0);
    if constexpr (sizeof(T) == 2) {
        if (vec16) {
            const int64_t lanes_needed = channels / 8;  // lanes to cover a row with 16-byte vectors
            auto go = [&](auto k, int lps) {
                const int64_t ntiles = (channels + 8 * lps - 1) / (8 * lps);
                const int64_t per_warp = 32 / lps;
                const int g = persistent_grid(k, 256, 0, (nseg * ntiles / per_warp + 8) / 8, 0);
                launch_pdl(k, g, 256, 0, st, data, bounds, bs, out, nrows, channels, srow, nseg, reduce, has_initial, bits, status);
                count_launch();
                return finish_launch("nb200_segment_pool");
            };
            if (lanes_needed <= 4) return go(pool16_kernel<T, I, 4>, 4);
            if (lanes_needed <= 8) return go(pool16_kernel<T, I, 8>, 8);
            if (lanes_needed <= 16) return go(pool16_kernel<T, I, 16>, 16);
            return go(pool16_kernel<T, I, 32>, 32);
        }
    }
    auto k = pool_kernel<T, I>;
    const int64_t ntiles = (channels + 127) / 128;
    const int g = persistent_grid(k, 256, 0, (nseg * ntiles + 7) / 8, 0);
    launch_pdl(k, g, 256, 0, st, data, bounds, bs, out, nrows, channels, srow, sch, nseg, reduce, has_initial, bits, status);
    count_launch();
    return finish_launch("nb200_segment_pool");
}

template <typename T>
int pool_idx(const T* data, int64_t nrows, int64_t channels, int64_t srow, int64_t sch, const void* bounds, int idt,
             int64_t bs, int64_t nseg, int reduce, int has_initial, uint32_t bits, T* out, uint32_t* status,
             cudaStream_t st) {
    if (idt == NB200_I32)
        return pool_t<T, int32_t>(data, nrows, channels, srow, sch, (const int32_t*)bounds, bs, nseg, reduce,
                                  has_initial, bits, out, status, st);
    return pool_t<T, int64_t>(data, nrows, channels, srow, sch, (const int64_t*)bounds, bs, nseg, reduce, has_initial,
                              bits, out, status, st);
}

}  // namespace

int launch_spans(const void* seg, int idt, int64_t nseg, int64_t sstride, int unsafe, int64_t nrows,
                 int64_t* spans, uint32_t* status, cudaStream_t st) {
    if (nseg > 4 * kSpanChunk) {  // long vectors: three launches over many CTAs
        const int64_t nb = (nseg + kSpanChunk - 1) / kSpanChunk;
        if (idt == NB200_I32)
            launch_pdl(spans_sum_kernel<int32_t>, (unsigned)nb, kSpanChunkThreads, 0, st, (const int32_t*)seg, nseg,
                       sstride, nrows, spans, status);
        else
            launch_pdl(spans_sum_kernel<int64_t>, (unsigned)nb, kSpanChunkThreads, 0, st, (const int64_t*)seg, nseg,
                       sstride, nrows, spans, status);
        launch_pdl(spans_offsets_kernel, 1, 1024, 0, st, nseg, nb, unsafe, nrows, spans, status);
        if (idt == NB200_I32)
            launch_pdl(spans_write_kernel<int32_t>, (unsigned)nb, kSpanChunkThreads, 0, st, (const int32_t*)seg, nseg,
                       sstride, nrows, spans, status);
        else
            launch_pdl(spans_write_kernel<int64_t>, (unsigned)nb, kSpanChunkThreads, 0, st, (const int64_t*)seg, nseg,
                       sstride, nrows, spans, status);
        count_launch(3);
        return finish_launch("nb200_segment_spans");
    }
    if (idt == NB200_I32)
        launch_pdl(spans_kernel<int32_t>, 1, 1024, 0, st, (const int32_t*)seg, nseg, sstride, unsafe, nrows, spans, status);
    else
        launch_pdl(spans_kernel<int64_t>, 1, 1024, 0, st, (const int64_t*)seg, nseg, sstride, unsafe, nrows, spans, status);
    count_launch();
    return finish_launch("nb200_segment_spans");
}

int launch_segment_pool(const void* data, int dtype, int64_t nrows, int64_t channels, int64_t srow, int64_t sch,
                        const void* bounds, int idt, int64_t bs, int64_t nseg, int reduce, int has_initial,
                        uint32_t initial_bits, void* out, uint32_t* status, cudaStream_t st) {
    switch (dtype) {
        case NB200_F32:
            return pool_idx<float>((const float*)data, nrows, channels, srow, sch, bounds, idt, bs, nseg, reduce,
                                   has_initial, initial_bits, (float*)out, status, st);
        case NB200_BF16:
            return pool_idx<__nv_bfloat16>((const __nv_bfloat16*)data, nrows, channels, srow, sch, bounds, idt, bs,
                                           nseg, reduce, has_initial, initial_bits, (__nv_bfloat16*)out, status, st);
        case NB200_F16:
            return pool_idx<__half>((const __half*)data, nrows, channels, srow, sch, bounds, idt, bs, nseg, reduce,
                                    has_initial, initial_bits, (__half*)out, status, st);
    }
    set_error("unknown dtype %d", dtype);
    return NB200_ERR_ARG;
}

}  // namespace nb200
