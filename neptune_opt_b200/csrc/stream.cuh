// Bulk-copy (TMA) staging primitives for sm_100a and the per-lane fold algebra that consumes
// staged data from shared memory.
//
// Each warp of a streaming kernel owns a ring of shared-memory stages. Lane 0 fills a stage with
// `cp.async.bulk` (global -> shared, completion counted in bytes on the stage's mbarrier); all
// lanes wait on the mbarrier's phase, read the stage, and lane 0 refills it once the warp has
// finished reading. No load uses cluster multicast. Every wait is bounded: after about a second
// the kernel records a fault bit and stops instead of spinning.
#pragma once

#include "fold.cuh"

namespace nb200 {

// Set (bitwise OR) by streaming kernels whose bounded wait ran out; read and cleared by the host
// (stream.cu, the one translation unit that includes this header).
static __device__ unsigned int g_stream_fault = 0u;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier generic-proxy shared-memory accesses before later async-proxy ones.
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Global -> shared bulk copy; dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait for the phase with `parity` to complete: false after ~2^31 SM cycles.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (int i = 0; i < (1 << 26); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (clock64() - t0 > (1ll << 31)) break;
    }
    atomicOr(&g_stream_fault, 1u);
    return false;
}

// 2^x on the special-function unit (ex2.approx, max relative error about 2 ulp).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// e^d for the fold's terms and repairs: exp(d) = 2^(d log2 e).
__device__ __forceinline__ float fexp(float d) { return ex2(d * kLog2e); }

// Per-lane state of the elements this lane holds in a staged block of `nv` 16-byte vectors
// (vectors lane, lane + 32, ...). Same algebra as chunk_state, with the reductions lane-local.
// Every reduction keeps V independent partials (one per position inside a 16-byte vector) so the
// element loop is V dependency chains instead of one; the partials combine at the end.
template <int V>
__device__ __forceinline__ float combine_sum(const float* a) {
    float s = a[0];
#pragma unroll
    for (int e = 1; e < V; ++e) s += a[e];
    return s;
}
template <int V>
__device__ __forceinline__ float combine_max(const float* a) {
    float s = a[0];
#pragma unroll
    for (int e = 1; e < V; ++e) s = fmaxf(s, a[e]);
    return s;
}

// ------------------------------------------------------------------ row sources
// The vectors of a row one lane holds: 16-byte vector j (V elements) for j = lane, lane + 32, ...
// below nv. for_each(f) calls f(u, j) for each of them in ascending j.
struct SmemRow {  // staged in shared memory
    const uint4* v;
    int nv, lane;
    template <class F>
    __device__ __forceinline__ void for_each(F&& f) const {
        for (int j = lane; j < nv; j += 32) f(v[j], j);
    }
};
template <int NV>
struct RegRow {  // held in registers, vector lane + 32 k in r[k] (a row of at most 32 NV vectors)
    uint4 r[NV];
    int nv, lane;
    template <class F>
    __device__ __forceinline__ void for_each(F&& f) const {
#pragma unroll
        for (int k = 0; k < NV; ++k)
            if (lane + 32 * k < nv) f(r[k], lane + 32 * k);
    }
};

template <int S, typename T, class Src>
__device__ __forceinline__ St lane_state(const Src& src, const Params& p) {
    using K = Sk<S>;
    constexpr int V = Elem<T>::V;
    const bool any = src.lane < src.nv;
    if constexpr (K::kind == K_LOG) {
        // Fast path: one max and one finiteness probe per element (phi * 0 is 0 for finite phi and
        // NaN for +-inf or NaN); when every element is finite the status is 0 and the max is the
        // max over finite terms, so the sum pass needs no per-element test.
        float mv[V], probe[V];
#pragma unroll
        for (int e = 0; e < V; ++e) { mv[e] = -NB200_INF; probe[e] = 0.f; }
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float ph = K::phi(Elem<T>::lane(u, e), p);
                mv[e] = fmaxf(mv[e], ph);
                probe[e] = fmaf(ph, 0.f, probe[e]);
            }
        });
        const float mall = combine_max<V>(mv);
        if (combine_sum<V>(probe) == 0.f) {
            const bool seen = mall != -NB200_INF;
            float a = 0.f;
            if (seen) {
                const float nm = -mall * kLog2e;
                float av[V];
#pragma unroll
                for (int e = 0; e < V; ++e) av[e] = 0.f;
                src.for_each([&](const uint4& u, int) {
#pragma unroll
                    for (int e = 0; e < V; ++e) av[e] += ex2(fmaf(K::phi(Elem<T>::lane(u, e), p), kLog2e, nm));
                });
                a = combine_sum<V>(av);
            }
            return St{mall, a, seen ? 1 : 0, 0};
        }
        // A non-finite element is present: exact NaN / +inf status and the max over finite terms.
        float m = -NB200_INF;
        int st = 0;
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float ph = K::phi(Elem<T>::lane(u, e), p);
                if (ph != ph) st |= 1;
                else if (ph == NB200_INF) st |= 2;
                else m = fmaxf(m, ph);
            }
        });
        const bool seen = m != -NB200_INF;
        const float den = seen ? m : 0.f;
        float a = 0.f;
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float ph = K::phi(Elem<T>::lane(u, e), p);
                if (fabsf(ph) < NB200_INF) a += fexp(ph - den);
            }
        });
        return St{m, a, seen ? 1 : 0, st};
    } else if constexpr (K::kind == K_MAXABS) {
        float mv[V], av[V];
#pragma unroll
        for (int e = 0; e < V; ++e) { mv[e] = 0.f; av[e] = 0.f; }
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) mv[e] = fmaxf(mv[e], fabsf(Elem<T>::lane(u, e)));
        });
        const float m = combine_max<V>(mv);
        const float c = K::prep(K::floor ? fmaxf(m, 1e-30f) : m, p);
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) av[e] += K::term_r(Elem<T>::lane(u, e), c);
        });
        return St{m, combine_sum<V>(av), any ? 1 : 0, 0};
    } else {  // K_SUMMAX
        float sv[V], av[V];
#pragma unroll
        for (int e = 0; e < V; ++e) { sv[e] = 0.f; av[e] = -NB200_INF; }
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) sv[e] += K::operand(Elem<T>::lane(u, e), p);
        });
        const float m = combine_sum<V>(sv);
        const float r = K::term_scale(m, p);
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) av[e] = fmaxf(av[e], Elem<T>::lane(u, e) * r);
        });
        return St{m, combine_max<V>(av), any ? 1 : 0, 0};
    }
}

// merge for the streaming path: identical algebra to merge<S>, with the log family's repair
// exponentials on the special-function unit.
template <int S>
__device__ __forceinline__ St merge_fast(const St& A, const St& B, const Params& p) {
    if constexpr (Sk<S>::kind == K_LOG) {
        const int status = A.status | B.status;
        if (!B.seen) return St{A.m, A.acc, A.seen, status};
        if (!A.seen) return St{B.m, B.acc, 1, status};
        const float m = fmaxf(A.m, B.m);
        return St{m, A.acc * fexp(A.m - m) + B.acc * fexp(B.m - m), 1, status};
    } else {
        return merge<S>(A, B, p);
    }
}

__device__ __forceinline__ St shfl_xor_state(const St& s, int o) {
    St r;
    r.m = __shfl_xor_sync(0xffffffffu, s.m, o);
    r.acc = __shfl_xor_sync(0xffffffffu, s.acc, o);
    r.seen = __shfl_xor_sync(0xffffffffu, s.seen, o);
    r.status = __shfl_xor_sync(0xffffffffu, s.status, o);
    return r;
}

// Merge the 32 lane states in a fixed balanced tree, lower lane on the left; every lane ends
// with the same state.
template <int S>
__device__ __forceinline__ St warp_merge(St s, int lane, const Params& p) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const St other = shfl_xor_state(s, o);
        s = (lane & o) ? merge_fast<S>(other, s, p) : merge_fast<S>(s, other, p);
    }
    return s;
}

// State of a whole resident row, computed the way the reference computes one chunk
// (emitters.py:459-488): the producer is reduced across the warp first, then every lane forms its
// terms against the row's producer and the consumer is reduced across the warp. No repair is
// needed inside a row, so this costs two warp reductions instead of a 32-state merge tree.
template <int S, typename T, class Src>
__device__ __forceinline__ St row_state(const Src& src, const Params& p) {
    using K = Sk<S>;
    constexpr int V = Elem<T>::V;
    if constexpr (K::kind == K_LOG) {
        float mv[V], probe[V];
#pragma unroll
        for (int e = 0; e < V; ++e) { mv[e] = -NB200_INF; probe[e] = 0.f; }
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const float ph = K::phi(Elem<T>::lane(u, e), p);
                mv[e] = fmaxf(mv[e], ph);
                probe[e] = fmaf(ph, 0.f, probe[e]);
            }
        });
        const float mall = warp_max(combine_max<V>(mv));
        const bool finite = __all_sync(0xffffffffu, combine_sum<V>(probe) == 0.f);
        if (finite) {
            const bool seen = mall != -NB200_INF;
            float av[V];
#pragma unroll
            for (int e = 0; e < V; ++e) av[e] = 0.f;
            if (seen) {
                const float nm = -mall * kLog2e;
                src.for_each([&](const uint4& u, int) {
#pragma unroll
                    for (int e = 0; e < V; ++e) av[e] += ex2(fmaf(K::phi(Elem<T>::lane(u, e), p), kLog2e, nm));
                });
            }
            return St{mall, warp_sum(combine_sum<V>(av)), seen ? 1 : 0, 0};
        }
        // a non-finite element: lane states with exact status, merged (rare path)
        return warp_merge<S>(lane_state<S, T>(src, p), src.lane, p);
    } else if constexpr (K::kind == K_MAXABS) {
        float mv[V], av[V];
#pragma unroll
        for (int e = 0; e < V; ++e) { mv[e] = 0.f; av[e] = 0.f; }
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) mv[e] = fmaxf(mv[e], fabsf(Elem<T>::lane(u, e)));
        });
        const float m = warp_max(combine_max<V>(mv));
        const float c = K::prep(K::floor ? fmaxf(m, 1e-30f) : m, p);
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) av[e] += K::term_r(Elem<T>::lane(u, e), c);
        });
        return St{m, warp_sum(combine_sum<V>(av)), 1, 0};
    } else {  // K_SUMMAX
        float sv[V], av[V];
#pragma unroll
        for (int e = 0; e < V; ++e) { sv[e] = 0.f; av[e] = -NB200_INF; }
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) sv[e] += K::operand(Elem<T>::lane(u, e), p);
        });
        const float m = warp_sum(combine_sum<V>(sv));
        const float r = K::term_scale(m, p);
        src.for_each([&](const uint4& u, int) {
#pragma unroll
            for (int e = 0; e < V; ++e) av[e] = fmaxf(av[e], Elem<T>::lane(u, e) * r);
        });
        return St{m, warp_max(combine_max<V>(av)), 1, 0};
    }
}


}  // namespace nb200
