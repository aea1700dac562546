// RMSNorm with fp32 accumulation on sm_100a.
//
// Numeric contract of the reference's structured backend (neptune_codegen/skeleton.py:213-217,
// emitters.py:576-595): total = sum x^2 in fp32, count = ncols, mean = div_rn(total, count),
// scale = rsqrt_rn(mean + eps), normalized = x * scale rounded to the input dtype BEFORE gamma,
// result = normalized * gamma rounded to the output dtype. The reference compiles with
// enable_fp_fusion=False (template.py:308), so every product and sum here is an explicit
// round-to-nearest operation and nothing contracts into an FMA.
#include "common.cuh"
#include "launch.h"

namespace nb200 {

template <typename T, int NV, bool VEC, bool CTA>
__global__ void __launch_bounds__(CTA ? 512 : 256)
rms_kernel(const T* __restrict__ x, const T* __restrict__ gamma, T* __restrict__ y, int64_t rows,
           int64_t ncols, int64_t srow, int64_t scol, int64_t sg, float eps, int gvec, int out_vec) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[64];
    Group<CTA> grp{red, 0};
    const int G = CTA ? (int)blockDim.x : 32;
    const int t = CTA ? (int)threadIdx.x : (int)(threadIdx.x & 31);
    const int64_t gid = CTA ? (int64_t)blockIdx.x
                            : (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t ng = CTA ? (int64_t)gridDim.x : (int64_t)gridDim.x * (blockDim.x >> 5);
    using CH = Chunk<T, NV, VEC>;
    constexpr int V = CH::V;
    const int64_t span = (int64_t)G * CH::E;
    const bool resident = span >= ncols;
    const float count = __ll2float_rn(ncols);
    for (int64_t r = gid; r < rows; r += ng) {
        const T* row = x + r * srow;
        CH ch;
        float total = 0.f;
        for (int64_t c0 = 0; c0 < ncols; c0 += span) {
            ch.load(row, scol, c0, ncols, t, G, resident);
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < CH::E; ++i) {
                const float v = ch.get(i);  // 0 beyond the row: contributes exactly 0
                s = __fadd_rn(s, __fmul_rn(v, v));
            }
            total = __fadd_rn(total, grp.reduce(s, RED_SUM));
        }
        const float mean = __fdiv_rn(total, count);
        const float scale = __frsqrt_rn(__fadd_rn(mean, eps));
        T* yrow = y + r * ncols;
        for (int64_t c0 = 0; c0 < ncols; c0 += span) {
            if (!resident) ch.load(row, scol, c0, ncols, t, G, false);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                float g[V];
                if (VEC && gvec) {
                    const int64_t c = CH::col_of(c0, t, G, k * V);
                    if (c < ncols) Elem<T>::unpack(ld_keep(gamma + c), g);
                    else {
#pragma unroll
                        for (int j = 0; j < V; ++j) g[j] = 0.f;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < V; ++j) {
                        const int64_t c = CH::col_of(c0, t, G, k * V + j);
                        g[j] = c < ncols ? Elem<T>::to_f(gamma[c * sg]) : 0.f;
                    }
                }
                float f[V];
#pragma unroll
                for (int j = 0; j < V; ++j) {
                    const float normalized = Elem<T>::to_f(Elem<T>::from_f(__fmul_rn(ch.get(k * V + j), scale)));
                    f[j] = __fmul_rn(normalized, g[j]);
                }
                store_vec<T, NV, VEC>(yrow, f, k, c0, ncols, t, G, out_vec != 0);
            }
        }
    }
}

namespace {

template <typename T>
int rms_t(const T* x, const T* gamma, T* y, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
          int64_t sg, float eps, const nb200_launch* L, cudaStream_t st) {
    constexpr int V = Elem<T>::V;
    const bool vec = scol == 1 && aligned16(x) && (rows <= 1 || (srow * (int64_t)sizeof(T)) % 16 == 0) &&
                     ncols % V == 0;
    const int gvec = sg == 1 && aligned16(gamma);
    const int out_vec = aligned16(y) && (ncols * (int64_t)sizeof(T)) % 16 == 0;
    const int cps = L ? L->ctas_per_sm : 0;
    const int64_t vecs = (ncols + V - 1) / V;
    const int variant = (L && L->variant) ? L->variant
                                          : (vecs <= 32 * 16 ? NB200_VARIANT_WARP_ROW : NB200_VARIANT_CTA_ROW);
    auto go = [&](auto k, int threads, int64_t work) {
        const int g = persistent_grid(k, threads, 0, work, cps);
        launch_pdl(k, g, threads, 0, st, x, gamma, y, rows, ncols, srow, scol, sg, eps, gvec, out_vec);
        count_launch();
        return finish_launch("nb200_rms_norm");
    };
    if (!vec) {
        if (variant == NB200_VARIANT_WARP_ROW) return go(rms_kernel<T, kScalarNV<T>, false, false>, 256, (rows + 7) / 8);
        return go(rms_kernel<T, kScalarNV<T>, false, true>, (L && L->threads) ? L->threads : 256, rows);
    }
    if (variant == NB200_VARIANT_WARP_ROW) {
        const int64_t per_lane = (vecs + 31) / 32;
        if (per_lane <= 1) return go(rms_kernel<T, 1, true, false>, 256, (rows + 7) / 8);
        if (per_lane <= 2) return go(rms_kernel<T, 2, true, false>, 256, (rows + 7) / 8);
        if (per_lane <= 4) return go(rms_kernel<T, 4, true, false>, 256, (rows + 7) / 8);
        if (per_lane <= 8) return go(rms_kernel<T, 8, true, false>, 256, (rows + 7) / 8);
        return go(rms_kernel<T, 16, true, false>, 256, (rows + 7) / 8);
    }
    const int threads = (L && L->threads) ? L->threads : 256;
    const int64_t per_thread = (vecs + threads - 1) / threads;
    if (per_thread <= 4) return go(rms_kernel<T, 4, true, true>, threads, rows);
    if (per_thread <= 8) return go(rms_kernel<T, 8, true, true>, threads, rows);
    return go(rms_kernel<T, 16, true, true>, threads, rows);
}

}  // namespace

// Few rows wider than 32 KB go to one thread-block cluster per row when x, gamma and y are
// contiguous and 16-byte aligned (and the CTA ranges fit the kernel's registers).
static int cluster_rms(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols, int64_t srow,
                       int64_t scol, int64_t sg, float eps, void* out, int csize, cudaStream_t st) {
    const int64_t es = dtype_size(dtype);
    if (scol != 1 || sg != 1 || !aligned16(x) || !aligned16(gamma) || !aligned16(out) || (ncols * es) % 16 != 0 ||
        (srow * es) % 16 != 0)
        return 0;
    switch (dtype) {
        case NB200_F32:
            return launch_cluster_rms<float>((const float*)x, (const float*)gamma, rows, ncols, srow, eps, (float*)out,
                                             csize, st);
        case NB200_BF16:
            return launch_cluster_rms<__nv_bfloat16>((const __nv_bfloat16*)x, (const __nv_bfloat16*)gamma, rows, ncols,
                                                     srow, eps, (__nv_bfloat16*)out, csize, st);
        case NB200_F16:
            return launch_cluster_rms<__half>((const __half*)x, (const __half*)gamma, rows, ncols, srow, eps,
                                              (__half*)out, csize, st);
    }
    return 0;
}

int launch_rms(const void* x, const void* gamma, int dtype, int64_t rows, int64_t ncols,
               int64_t srow, int64_t scol, int64_t sg, float eps, void* out,
               const nb200_launch* L, cudaStream_t st) {
    const bool auto_cluster = rows >= 1 && rows <= 2 * (int64_t)sm_count() && ncols * (int64_t)dtype_size(dtype) > 32768;
    if ((L && L->variant == NB200_VARIANT_CLUSTER) || ((!L || L->variant == NB200_VARIANT_AUTO) && auto_cluster)) {
        const int rc = cluster_rms(x, gamma, dtype, rows, ncols, srow, scol, sg, eps, out, L ? L->stages : 0, st);
        if (rc != 0) return rc < 0 ? rc : NB200_OK;
        if (L && L->variant == NB200_VARIANT_CLUSTER) {
            set_error("nb200_rms_norm: the cluster variant needs contiguous 16-byte-aligned x, gamma, y whose row "
                      "ranges fit the kernel (at most 16 x 256 x 8 vectors per row)");
            return NB200_ERR_ARG;
        }
    }
    if (!L || L->variant == NB200_VARIANT_AUTO || L->variant == NB200_VARIANT_STREAM) {
        const int rc = stream_rms(x, gamma, dtype, rows, ncols, srow, scol, sg, eps, out, L, st);
        if (rc != 0) return rc < 0 ? rc : NB200_OK;
        if (L && L->variant == NB200_VARIANT_STREAM) {
            set_error("nb200_rms_norm: the streaming variant needs contiguous 16-byte-aligned rows of <= 32 KB");
            return NB200_ERR_ARG;
        }
    }
    switch (dtype) {
        case NB200_F32:
            return rms_t<float>((const float*)x, (const float*)gamma, (float*)out, rows, ncols, srow, scol, sg, eps, L, st);
        case NB200_BF16:
            return rms_t<__nv_bfloat16>((const __nv_bfloat16*)x, (const __nv_bfloat16*)gamma,
                                        (__nv_bfloat16*)out, rows, ncols, srow, scol, sg, eps, L, st);
        case NB200_F16:
            return rms_t<__half>((const __half*)x, (const __half*)gamma, (__half*)out, rows, ncols, srow, scol, sg, eps, L, st);
    }
    set_error("unknown dtype %d", dtype);
    return NB200_ERR_ARG;
}

}  // namespace nb200
