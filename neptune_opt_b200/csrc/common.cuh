// Shared device/host helpers for the neptune-opt B200 backend (sm_100a).
//
// Row data arrive as a strided 2-D view [rows, ncols] of fp32 / bf16 / fp16. Every kernel
// computes in fp32 and converts back to the storage type only where the reference's numeric
// contract rounds (neptune_codegen/torch_op.py:91-97 narrows only the result).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <atomic>

#include "../../include/neptune_b200.h"

#define NB200_INF __int_as_float(0x7f800000)
#define NB200_NAN __int_as_float(0x7fc00000)

namespace nb200 {

// ------------------------------------------------------------------ host bookkeeping
void set_error(const char* fmt, ...);
int sm_count();
void count_launch(int n = 1);
int finish_launch(const char* what);  // checks cudaGetLastError, returns nb200_status

// ------------------------------------------------------------------ programmatic dependent launch
// Kernels launched with launch_pdl may be scheduled while the previous kernel on the stream is
// still draining, so the launch and CTA start-up overlap its tail. Each such kernel calls
// pdl_wait() before its first global-memory access (read or write): it returns once the previous
// kernel has completed and its writes are visible, so results are exactly those of plain stream
// order. pdl_trigger() allows the next PDL kernel to be scheduled; it can start only after every
// CTA of this grid has triggered or exited, so a grid never waits on a dependent for resources.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem, cudaStream_t st,
                       Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

inline size_t dtype_size(int dtype) { return dtype == NB200_F32 ? 4 : 2; }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ------------------------------------------------------------------ element traits
// V = elements per 16-byte vector. unpack/pack convert a 16-byte vector to/from fp32 lanes.
template <typename T> struct Elem;

template <> struct Elem<float> {
    static constexpr int V = 4;
    __device__ __forceinline__ static float to_f(float v) { return v; }
    __device__ __forceinline__ static float from_f(float v) { return v; }
    __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
        f[0] = __uint_as_float(u.x); f[1] = __uint_as_float(u.y);
        f[2] = __uint_as_float(u.z); f[3] = __uint_as_float(u.w);
    }
    __device__ __forceinline__ static uint4 pack(const float* f) {
        return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                          __float_as_uint(f[2]), __float_as_uint(f[3]));
    }
    __device__ __forceinline__ static float lane(const uint4& u, int j) {
        return __uint_as_float(j == 0 ? u.x : j == 1 ? u.y : j == 2 ? u.z : u.w);
    }
};

template <> struct Elem<__nv_bfloat16> {
    static constexpr int V = 8;
    __device__ __forceinline__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    __device__ __forceinline__ static __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
    __device__ __forceinline__ static void unpack_word(uint32_t w, float* f) {
        f[0] = __uint_as_float(w << 16);
        f[1] = __uint_as_float(w & 0xffff0000u);
    }
    __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
        unpack_word(u.x, f); unpack_word(u.y, f + 2); unpack_word(u.z, f + 4); unpack_word(u.w, f + 6);
    }
    __device__ __forceinline__ static uint32_t pack_word(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static uint4 pack(const float* f) {
        return make_uint4(pack_word(f[0], f[1]), pack_word(f[2], f[3]),
                          pack_word(f[4], f[5]), pack_word(f[6], f[7]));
    }
    __device__ __forceinline__ static float lane(const uint4& u, int j) {
        const uint32_t w = (j >> 1) == 0 ? u.x : (j >> 1) == 1 ? u.y : (j >> 1) == 2 ? u.z : u.w;
        return __uint_as_float((j & 1) ? (w & 0xffff0000u) : (w << 16));
    }
};

template <> struct Elem<__half> {
    static constexpr int V = 8;
    __device__ __forceinline__ static float to_f(__half v) { return __half2float(v); }
    __device__ __forceinline__ static __half from_f(float v) { return __float2half_rn(v); }
    __device__ __forceinline__ static void unpack_word(uint32_t w, float* f) {
        __half2 h = *reinterpret_cast<__half2*>(&w);
        float2 g = __half22float2(h);
        f[0] = g.x; f[1] = g.y;
    }
    __device__ __forceinline__ static void unpack(const uint4& u, float* f) {
        unpack_word(u.x, f); unpack_word(u.y, f + 2); unpack_word(u.z, f + 4); unpack_word(u.w, f + 6);
    }
    __device__ __forceinline__ static uint32_t pack_word(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    __device__ __forceinline__ static uint4 pack(const float* f) {
        return make_uint4(pack_word(f[0], f[1]), pack_word(f[2], f[3]),
                          pack_word(f[4], f[5]), pack_word(f[6], f[7]));
    }
    __device__ __forceinline__ static float lane(const uint4& u, int j) {
        const uint32_t w = (j >> 1) == 0 ? u.x : (j >> 1) == 1 ? u.y : (j >> 1) == 2 ? u.z : u.w;
        return __half2float(__ushort_as_half((unsigned short)((j & 1) ? (w >> 16) : (w & 0xffffu))));
    }
};

// [v0, v1): part i of n items cut into k contiguous, nearly equal parts.
__device__ __forceinline__ void split_range(int64_t n, int64_t k, int64_t i, int64_t& v0, int64_t& v1) {
    v0 = n * i / k;
    v1 = n * (i + 1) / k;
}

// Streaming 16-byte load/store: data read once should not displace reused lines.
__device__ __forceinline__ uint4 ld_stream(const void* p) {
    return __ldcs(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ uint4 ld_keep(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
    __stcs(reinterpret_cast<uint4*>(p), v);
}

// ------------------------------------------------------------------ warp / group reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_or(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

enum RedOp { RED_SUM = 0, RED_MAX = 1 };

// A row "group" is one warp (CTA == false) or the whole CTA (CTA == true). Group reductions
// return the result in every thread. The CTA form alternates two shared-memory buffers so one
// __syncthreads per reduction suffices. Cross-warp order is fixed (warp 0, 1, ...), so results
// are deterministic.
template <bool CTA>
struct Group {
    float* buf;   // 2 * 32 floats of shared memory when CTA
    int phase;

    __device__ __forceinline__ float reduce(float v, RedOp op) {
        v = (op == RED_SUM) ? warp_sum(v) : warp_max(v);
        if (!CTA) return v;
        float* slot = buf + (phase & 1) * 32;
        phase++;
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
        if (lane == 0) slot[warp] = v;
        __syncthreads();
        float r = slot[0];
        for (int w = 1; w < nw; ++w) r = (op == RED_SUM) ? r + slot[w] : fmaxf(r, slot[w]);
        return r;
    }
    __device__ __forceinline__ int reduce_or(int v) {
        v = warp_or(v);
        if (!CTA) return v;
        int* slot = reinterpret_cast<int*>(buf + (phase & 1) * 32);
        phase++;
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
        if (lane == 0) slot[warp] = v;
        __syncthreads();
        int r = 0;
        for (int w = 0; w < nw; ++w) r |= slot[w];
        return r;
    }
};

// ------------------------------------------------------------------ chunk loader
// A chunk is G * NV * V consecutive columns of one row starting at column c0. Thread t of the
// group holds NV vectors of V elements. With VEC, vector k of thread t covers columns
// (c0 / V + t + k * G) * V .. + V (16-byte loads, coalesced across the group) and stays packed
// in registers (16-bit data costs half the registers of fp32); without VEC, element (k, j) is
// column c0 + t + (k * V + j) * G (scalar strided loads) held as fp32. col_of gives the column
// of element i = k * V + j for either layout; get(i) returns it as fp32.
template <typename T, int NV, bool VEC>
struct Chunk {
    static constexpr int V = Elem<T>::V;
    static constexpr int E = NV * V;
    uint4 raw[VEC ? NV : 1];
    float v[VEC ? 1 : E];

    __device__ __forceinline__ static int64_t col_of(int64_t c0, int t, int G, int i) {
        const int k = i / V, j = i % V;
        if (VEC) return c0 + ((int64_t)t + (int64_t)k * G) * V + j;
        return c0 + t + ((int64_t)k * V + j) * G;
    }
    __device__ __forceinline__ static bool valid(int64_t c0, int64_t c_hi, int t, int G, int i) {
        return col_of(c0, t, G, i) < c_hi;
    }

    __device__ __forceinline__ float get(int i) const {
        if constexpr (VEC) return Elem<T>::lane(raw[i / V], i % V);
        else return v[i];
    }

    // Loads columns < c_hi; others read as 0. `stream` selects evict-first loads.
    __device__ __forceinline__ void load(const T* row, int64_t stride_col, int64_t c0, int64_t c_hi,
                                         int t, int G, bool stream) {
        if constexpr (VEC) {
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                const int64_t c = col_of(c0, t, G, k * V);
                if (c < c_hi) raw[k] = stream ? ld_stream(row + c) : ld_keep(row + c);
                else raw[k] = make_uint4(0u, 0u, 0u, 0u);
            }
        } else {
#pragma unroll
            for (int i = 0; i < E; ++i) {
                const int64_t c = col_of(c0, t, G, i);
                v[i] = (c < c_hi) ? Elem<T>::to_f(row[c * stride_col]) : 0.f;
            }
        }
    }
};

// Vectors per thread of the scalar (strided) path: 16 elements per thread for every dtype.
template <typename T>
constexpr int kScalarNV = 16 / Elem<T>::V;

// Writes the V fp32 values of vector k of a Chunk-shaped tile to a contiguous output row (one
// 16-byte store when the chunk is vectorised and the output row is 16-byte aligned).
template <typename T, int NV, bool VEC>
__device__ __forceinline__ void store_vec(T* out_row, const float* f, int k, int64_t c0, int64_t c_hi,
                                          int t, int G, bool out_vec) {
    using CH = Chunk<T, NV, VEC>;
    constexpr int V = CH::V;
    if (VEC && out_vec) {
        const int64_t c = CH::col_of(c0, t, G, k * V);
        if (c < c_hi) st_stream(out_row + c, Elem<T>::pack(f));
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int64_t c = CH::col_of(c0, t, G, k * V + j);
            if (c < c_hi) out_row[c] = Elem<T>::from_f(f[j]);
        }
    }
}

// Persistent grid: enough CTAs to fill every SM at the occupancy the kernel reaches.
template <typename K>
inline int persistent_grid(K kernel, int threads, size_t smem, int64_t work_ctas, int ctas_per_sm) {
    int occ = ctas_per_sm;
    if (occ <= 0) {
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem) != cudaSuccess || occ < 1)
            occ = 1;
    }
    int64_t g = (int64_t)sm_count() * occ;
    if (work_ctas < g) g = work_ctas;
    if (g < 1) g = 1;
    return (int)g;
}

}  // namespace nb200
