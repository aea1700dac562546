// Row-last repaired folds on sm_100a: the serial plan (one warp or one CTA per row), the
// softmax / log_softmax / L2-normalize readouts fused into the same single pass, and the explicit
// split plan (chunk states + ordered merge).
//
// Reference kernels replaced: the serial template neptune_codegen/template.py:41-54 with its
// helpers emitters.py:436-532, the two-pass template template.py:62-103 and the split pair
// template.py:137-165 (launch template.py:368-390).
#include "fold.cuh"
#include "launch.h"
#include "span.cuh"

namespace nb200 {

// ------------------------------------------------------------------ serial fold
template <int S, typename T, int NV, bool VEC, bool CTA>
__global__ void __launch_bounds__(CTA ? 512 : 256)
fold_kernel(const T* __restrict__ x, T* __restrict__ out, int64_t rows, int64_t ncols,
            int64_t srow, int64_t scol, Params p) {
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
    const int64_t span = (int64_t)G * CH::E;
    for (int64_t r = gid; r < rows; r += ng) {
        const T* row = x + r * srow;
        float res;
        if constexpr (Sk<S>::kind == K_TWOPASS) {
            // pass 1: the producer (mean as sum of c / N); pass 2: the centred term with the
            // producer held constant. A resident row is not read twice.
            const bool resident = span >= ncols;
            CH ch;
            float mean = 0.f;
            for (int64_t c0 = 0; c0 < ncols; c0 += span) {
                ch.load(row, scol, c0, ncols, t, G, false);
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < CH::E; ++i)
                    if (CH::valid(c0, ncols, t, G, i)) s += ch.get(i) * p.invN;
                mean = mean + grp.reduce(s, RED_SUM);
            }
            float acc = 0.f;
            for (int64_t c0 = 0; c0 < ncols; c0 += span) {
                if (!resident) ch.load(row, scol, c0, ncols, t, G, true);
                float s = 0.f;
#pragma unroll
                for (int i = 0; i < CH::E; ++i) {
                    if (CH::valid(c0, ncols, t, G, i)) {
                        const float d = ch.get(i) - mean;
                        s += p.invN * (d * d);
                    }
                }
                acc = acc + grp.reduce(s, RED_SUM);
            }
            res = Sk<S>::fin(acc);
        } else {
            St run = empty_state();
            for (int64_t c0 = 0; c0 < ncols; c0 += span) {
                CH ch;
                ch.load(row, scol, c0, ncols, t, G, true);
                run = merge<S>(run, chunk_state<S>(ch, c0, ncols, t, G, grp, p), p);
            }
            res = finalize<S>(run, p);
        }
        if (t == 0) out[r] = Elem<T>::from_f(res);
    }
}

// ------------------------------------------------------------------ softmax-family readout
// mode 0: softmax = exp(x - m) / s; mode 1: log_softmax = (x - m) - log(s). A row with NaN, +inf
// or no finite element reads out as NaN everywhere, as the reference's lowering does
// (neptune_recognize/lowering.py:91-99). Rows that fit the chunk are read from HBM once.
template <typename T, int NV, bool VEC, bool CTA>
__global__ void __launch_bounds__(CTA ? 512 : 256)
softmax_kernel(const T* __restrict__ x, T* __restrict__ y, T* __restrict__ lse, int64_t rows,
               int64_t ncols, int64_t srow, int64_t scol, int mode, int out_vec) {
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
    const int64_t span = (int64_t)G * CH::E;
    const bool resident = span >= ncols;
    const Params p{0.f, 0.f, 1.f, 1.f, 0.f, 0.f, 0.f};
    for (int64_t r = gid; r < rows; r += ng) {
        const T* row = x + r * srow;
        CH ch;
        St run = empty_state();
        for (int64_t c0 = 0; c0 < ncols; c0 += span) {
            ch.load(row, scol, c0, ncols, t, G, resident);
            run = merge<NB200_LOGSUMEXP>(run, chunk_state<NB200_LOGSUMEXP>(ch, c0, ncols, t, G, grp, p), p);
        }
        const bool bad = run.status != 0 || !run.seen;
        const float m = run.m, inv = 1.0f / run.acc, lg = logf(run.acc);
        T* yrow = y + r * ncols;
        for (int64_t c0 = 0; c0 < ncols; c0 += span) {
            if (!resident) ch.load(row, scol, c0, ncols, t, G, false);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                float f[CH::V];
#pragma unroll
                for (int j = 0; j < CH::V; ++j) {
                    const float v = ch.get(k * CH::V + j);
                    f[j] = bad ? NB200_NAN : (mode == 0 ? expf(v - m) * inv : (v - m) - lg);
                }
                store_vec<T, NV, VEC>(yrow, f, k, c0, ncols, t, G, out_vec != 0);
            }
        }
        if (lse != nullptr && t == 0) lse[r] = Elem<T>::from_f(finalize<NB200_LOGSUMEXP>(run, p));
    }
}

// ------------------------------------------------------------------ L2 normalize readout
template <typename T, int NV, bool VEC, bool CTA>
__global__ void __launch_bounds__(CTA ? 512 : 256)
l2norm_kernel(const T* __restrict__ x, T* __restrict__ y, T* __restrict__ norm, int64_t rows,
              int64_t ncols, int64_t srow, int64_t scol, int out_vec) {
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
    const int64_t span = (int64_t)G * CH::E;
    const bool resident = span >= ncols;
    const Params p{0.f, 0.f, 1.f, 1.f, 0.f, 0.f, 0.f};
    for (int64_t r = gid; r < rows; r += ng) {
        const T* row = x + r * srow;
        CH ch;
        St run = empty_state();
        for (int64_t c0 = 0; c0 < ncols; c0 += span) {
            ch.load(row, scol, c0, ncols, t, G, resident);
            run = merge<NB200_STABLE_L2>(run, chunk_state<NB200_STABLE_L2>(ch, c0, ncols, t, G, grp, p), p);
        }
        const float nrm = finalize<NB200_STABLE_L2>(run, p);
        T* yrow = y + r * ncols;
        for (int64_t c0 = 0; c0 < ncols; c0 += span) {
            if (!resident) ch.load(row, scol, c0, ncols, t, G, false);
#pragma unroll
            for (int k = 0; k < NV; ++k) {
                float f[CH::V];
#pragma unroll
                for (int j = 0; j < CH::V; ++j) f[j] = __fdiv_rn(ch.get(k * CH::V + j), nrm);
                store_vec<T, NV, VEC>(yrow, f, k, c0, ncols, t, G, out_vec != 0);
            }
        }
        if (norm != nullptr && t == 0) norm[r] = Elem<T>::from_f(nrm);
    }
}

// ------------------------------------------------------------------ split plan
// One CTA per (row, part): the state of columns [cb + part * cc, min(cb + (part+1) * cc, cb + ns)).
template <int S, typename T, bool VEC>
__global__ void __launch_bounds__(256)
partial_kernel(const T* __restrict__ x, nb200_state* __restrict__ states, int64_t rows, int64_t cb,
               int64_t ns, int64_t srow, int64_t scol, int64_t cc, int64_t nparts, Params p) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[64];
    Group<true> grp{red, 0};
    const int G = (int)blockDim.x, t = (int)threadIdx.x;
    using CH = Chunk<T, 4, VEC>;
    const int64_t span = (int64_t)G * CH::E;
    const int64_t work = rows * nparts;
    for (int64_t w = blockIdx.x; w < work; w += gridDim.x) {
        const int64_t r = w / nparts, part = w - r * nparts;
        const T* row = x + r * srow;
        const int64_t lo = cb + part * cc;
        const int64_t hi = min(lo + cc, cb + ns);
        St run = empty_state();
        for (int64_t c0 = lo; c0 < hi; c0 += span) {
            CH ch;
            ch.load(row, scol, c0, hi, t, G, true);
            run = merge<S>(run, chunk_state<S>(ch, c0, hi, t, G, grp, p), p);
        }
        if (t == 0)
            reinterpret_cast<float4*>(states)[w] =
                make_float4(run.m, run.acc, __int_as_float(run.seen), __int_as_float(run.status));
    }
}

__device__ __forceinline__ St shfl_state(const St& s, int o) {
    St r;
    r.m = __shfl_xor_sync(0xffffffffu, s.m, o);
    r.acc = __shfl_xor_sync(0xffffffffu, s.acc, o);
    r.seen = __shfl_xor_sync(0xffffffffu, s.seen, o);
    r.status = __shfl_xor_sync(0xffffffffu, s.status, o);
    return r;
}

// One row's states merged by a warp. Lane l folds the contiguous run of parts [l*k, (l+1)*k) left
// to right; the 32 runs then combine in a fixed balanced tree, always with the lower-indexed run on
// the left. The order depends only on nparts, so the result is deterministic. kL2 reads the states
// at L2 (states another GPU wrote into this one's memory).
template <int S, bool kL2>
__device__ __forceinline__ St merge_row(const nb200_state* row, int64_t nparts, int64_t pstride, int lane,
                                        const Params& p) {
    const int64_t k = (nparts + 31) / 32;
    St s = empty_state();
    const int64_t lo = (int64_t)lane * k;
    const int64_t hi = min(lo + k, nparts);
    constexpr int kBatch = 8;  // a lane's states are loaded kBatch at a time, then merged in order
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;  // else 4-byte loads (caller's layout)
    for (int64_t j0 = lo; j0 < hi; j0 += kBatch) {
        float4 b[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            if (j0 + u >= hi) continue;
            const nb200_state* q = row + (j0 + u) * pstride;
            if (vec) {
                b[u] = kL2 ? __ldcg(reinterpret_cast<const float4*>(q)) : __ldg(reinterpret_cast<const float4*>(q));
            } else {
                const float* f = reinterpret_cast<const float*>(q);
                b[u] = kL2 ? make_float4(__ldcg(f), __ldcg(f + 1), __ldcg(f + 2), __ldcg(f + 3))
                           : make_float4(__ldg(f), __ldg(f + 1), __ldg(f + 2), __ldg(f + 3));
            }
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            if (j0 + u < hi) s = merge<S>(s, St{b[u].x, b[u].y, __float_as_int(b[u].z), __float_as_int(b[u].w)}, p);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const St other = shfl_state(s, o);
        s = (lane & o) ? merge<S>(other, s, p) : merge<S>(s, other, p);
    }
    return s;
}

// One warp per row, two rows per CTA: the few hundred rows of a split plan spread over every SM.
constexpr int kMergeThreads = 64;
template <int S, typename T>
__global__ void __launch_bounds__(256)
merge_kernel(const nb200_state* __restrict__ states, T* __restrict__ out, int64_t rows,
             int64_t nparts, int64_t rstride, int64_t pstride, Params p) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int64_t gid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t ng = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = gid; r < rows; r += ng) {
        const St s = merge_row<S, false>(states + r * rstride, nparts, pstride, lane, p);
        if (lane == 0) out[r] = Elem<T>::from_f(finalize<S>(s, p));
    }
}

// ------------------------------------------------------------------ split plan across GPUs
// The column-sharded split plan exchanges its chunk states through peer memory instead of a
// collective. Each rank owns an exchange buffer, mapped into every other rank's address space:
//   header   epoch of the last completed exchange, a completion counter, the recorded layout;
//   slots    two parities x [rows][world][nparts] tagged states; call e uses parity e & 1.
// A slot carries its epoch inside the data (the split plan's states are 16 bytes): two 8-byte
// words {m, e} and {acc, e << 5 | status << 1 | seen}, written with one 16-byte store whose two
// 8-byte halves are each single-copy atomic. Call e: the fold (peer_span_kernel, or the partial
// fold + peer_push_kernel) writes this rank's states into slot `rank` of parity e & 1 in every
// rank's buffer (stores over NVLink, no fence, no flag); peer_merge_kernel reads each state until
// both its words carry epoch e (bounded), merges each row's world * nparts states in ascending
// (rank, part) order -- the order of the single-GPU split plan -- and its last CTA records e as
// completed. Rows it cannot produce (a state that never arrived, a layout that differs) read NaN. A rank can be at most one call ahead of another (its next stores follow its own
// merge, which needs everyone's states), so two parities keep a fast rank from overwriting states
// a slow one is still merging, and a slot still holding call e - 2's words never passes for call
// e's. The epoch lives in device memory, so a captured CUDA graph replays correctly.
static __device__ unsigned int g_peer_fault = 0u;
constexpr int kMaxPeers = 8;
constexpr int64_t kPeerHeaderBytes = 256;
constexpr long long kPeerWaitCycles = 1ll << 31;
constexpr unsigned int kPeerMagic = 0x4e425045u;  // "NBPE": written by peer_init_kernel
struct PeerHeader {
    unsigned int ep;          // epoch of the last completed exchange on this rank
    unsigned int merge_done;  // CTAs of the merge that have finished reading the slots
    unsigned int pad[2 + kMaxPeers];
    // The layout this buffer was sized and initialised for (nb200_peer_init). Every push checks the
    // destination's layout and every merge its own before touching the slots: a call whose
    // (rows, world, nparts) differ, or a buffer never initialised, stores nothing.
    long long rows;
    long long nparts;
    int world;
    unsigned int magic;
};
static_assert(sizeof(PeerHeader) <= kPeerHeaderBytes, "peer header");
struct PeerPtrs {
    unsigned char* p[kMaxPeers];  // every rank's exchange buffer as mapped in this process
};
// peers.p[i] for a thread-dependent i without indexing the parameter array (which would copy it to
// local memory): an unrolled select.
__device__ __forceinline__ unsigned char* peer_at(const PeerPtrs& peers, int i) {
    unsigned char* q = nullptr;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
        if (i == r) q = peers.p[r];
    return q;
}

__device__ __forceinline__ bool peer_layout_ok(const unsigned char* buf, int64_t rows, int64_t nparts, int world) {
    const volatile PeerHeader* h = reinterpret_cast<const volatile PeerHeader*>(buf);
    return h->magic == kPeerMagic && h->rows == rows && h->nparts == nparts && h->world == world;
}

// A tagged slot: state v (m, acc, seen, status as in the float4 state layout) of call e.
__device__ __forceinline__ void peer_slot_store(void* slot, const float4& v, unsigned int e) {
    const unsigned int tag = (e << 5) | ((unsigned int)(__float_as_int(v.w) & 15) << 1) |
                             (unsigned int)(__float_as_int(v.z) & 1);
    const unsigned long long a = (unsigned long long)__float_as_uint(v.x) | ((unsigned long long)e << 32);
    const unsigned long long b = (unsigned long long)__float_as_uint(v.y) | ((unsigned long long)tag << 32);
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(slot), "l"(a), "l"(b) : "memory");
}
// The two words of a tagged slot, and whether they carry epoch e (then v holds the state).
__device__ __forceinline__ void peer_slot_raw(const void* slot, unsigned long long& a, unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(slot) : "memory");
}
__device__ __forceinline__ bool peer_slot_ready(unsigned long long a, unsigned long long b, unsigned int e, float4& v) {
    const unsigned int tag = (unsigned int)(b >> 32);
    if ((unsigned int)(a >> 32) != e || (tag >> 5) != (e & 0x07ffffffu)) return false;
    v = make_float4(__uint_as_float((unsigned int)a), __uint_as_float((unsigned int)b), __int_as_float((int)(tag & 1u)),
                    __int_as_float((int)((tag >> 1) & 15u)));
    return true;
}

// Records the layout in a buffer's header, clears its epoch and counter (CTA 0, thread 0) and
// zeroes every slot (no slot then carries an epoch of a call to come).
__global__ void peer_init_kernel(unsigned char* buf, int64_t rows, int64_t nparts, int world) {
    pdl_wait();
    pdl_trigger();
    const int64_t nslots = 2 * rows * world * nparts;
    uint4* slots = reinterpret_cast<uint4*>(buf + kPeerHeaderBytes);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nslots; i += (int64_t)gridDim.x * blockDim.x)
        slots[i] = make_uint4(0u, 0u, 0u, 0u);
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        PeerHeader* h = reinterpret_cast<PeerHeader*>(buf);
        h->ep = 0u;
        h->merge_done = 0u;
        for (int r = 0; r < 2 + kMaxPeers; ++r) h->pad[r] = 0u;
        h->rows = rows;
        h->nparts = nparts;
        h->world = world;
        __threadfence_system();
        h->magic = kPeerMagic;
        __threadfence_system();
    }
}

// One CTA per destination rank: CTA r checks rank r's recorded layout and writes this rank's
// states, tagged with the call's epoch, into rank r's buffer. A destination whose layout differs
// gets nothing (fault bit 3).
constexpr int kPushThreads = 512;
__global__ void __launch_bounds__(kPushThreads)
peer_push_kernel(const nb200_state* __restrict__ states, int64_t rows, int64_t nlocal, int64_t nparts,
                 PeerPtrs peers, int world, int rank, unsigned char* own) {
    pdl_wait();
    pdl_trigger();
    const PeerHeader* h = reinterpret_cast<const PeerHeader*>(own);
    const unsigned int e = *reinterpret_cast<const volatile unsigned int*>(&h->ep) + 1u;
    const int64_t par = e & 1u, n = rows * nparts;
    unsigned char* dst = peer_at(peers, blockIdx.x);
    __shared__ int layout_ok;
    if (threadIdx.x == 0) {
        layout_ok = peer_layout_ok(own, rows, nparts, world) && peer_layout_ok(dst, rows, nparts, world);
        if (!layout_ok) atomicOr(&g_peer_fault, 8u);
    }
    __syncthreads();
    if (!layout_ok) return;
    float4* slots = reinterpret_cast<float4*>(dst + kPeerHeaderBytes);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t row = i / nparts, part = i - row * nparts;
        // parts past this rank's own count are empty states (unequal shard widths)
        const float4 v = part < nlocal ? reinterpret_cast<const float4*>(states)[row * nlocal + part]
                                       : make_float4(-NB200_INF, 0.f, 0.f, 0.f);
        peer_slot_store(&slots[((par * rows + row) * world + rank) * nparts + part], v, e);
    }
}

// One warp per row, as merge_row: lane l reads the contiguous run of states [l*k, (l+1)*k) of the
// row's world * nparts, eight slots at a time (all eight loads issued before any is tested), each
// until it carries epoch e -- bounded: about a second of SM cycles, then the caller writes the row
// as NaN and sets fault bit 2 -- merges its run left to right, then the 32 runs combine in
// merge_row's tree.
template <int S>
__device__ __forceinline__ bool peer_merge_row(const float4* row, int64_t total, unsigned int e, int lane,
                                               const Params& p, St& out, long long t0) {
    constexpr int kBatch = 8;
    const int64_t k = (total + 31) / 32;
    const int64_t lo = (int64_t)lane * k, hi = min(lo + k, total);
    St s = empty_state();
    bool ok = true;
    for (int64_t j0 = lo; j0 < hi && ok; j0 += kBatch) {
        float4 v[kBatch];
        unsigned int pending = 0u;  // bit u: slot j0 + u not yet carrying epoch e
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            if (j0 + u < hi) pending |= 1u << u;
        for (unsigned int it = 0; pending; ++it) {
            unsigned long long a[kBatch], b[kBatch];
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
                if ((pending >> u) & 1u) peer_slot_raw(row + j0 + u, a[u], b[u]);
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
                if (((pending >> u) & 1u) && peer_slot_ready(a[u], b[u], e, v[u])) pending &= ~(1u << u);
            if (pending && (it & 63u) == 63u && clock64() - t0 > kPeerWaitCycles) {
                ok = false;
                break;
            }
        }
        if (!ok) break;
#pragma unroll
        for (int u = 0; u < kBatch; ++u)
            if (j0 + u < hi) s = merge<S>(s, St{v[u].x, v[u].y, __float_as_int(v[u].z), __float_as_int(v[u].w)}, p);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const St other = shfl_state(s, o);
        s = (lane & o) ? merge<S>(other, s, p) : merge<S>(s, other, p);
    }
    out = s;
    return __all_sync(0xffffffffu, ok);
}

template <int S, typename T>
__global__ void __launch_bounds__(256)
peer_merge_kernel(unsigned char* own, T* __restrict__ out, int64_t rows, int64_t nparts, int world, Params p) {
    pdl_wait();
    pdl_trigger();
    PeerHeader* h = reinterpret_cast<PeerHeader*>(own);
    if (!peer_layout_ok(own, rows, nparts, world)) {  // nothing read, every row NaN, epoch kept
        if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&g_peer_fault, 8u);
        for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += (int64_t)gridDim.x * blockDim.x)
            out[r] = Elem<T>::from_f(NB200_NAN);
        return;
    }
    const unsigned int e = *reinterpret_cast<volatile unsigned int*>(&h->ep) + 1u;
    const int lane = threadIdx.x & 31;
    const int64_t total = (int64_t)world * nparts;
    const float4* slots = reinterpret_cast<const float4*>(own + kPeerHeaderBytes) + (int64_t)(e & 1u) * rows * total;
    const int64_t gid = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t ng = (int64_t)gridDim.x * (blockDim.x >> 5);
    const long long t0 = clock64();
    for (int64_t r = gid; r < rows; r += ng) {
        St s;
        if (peer_merge_row<S>(slots + r * total, total, e, lane, p, s, t0)) {
            if (lane == 0) out[r] = Elem<T>::from_f(finalize<S>(s, p));
        } else if (lane == 0) {  // a state never arrived: the row reads NaN
            atomicOr(&g_peer_fault, 4u);
            out[r] = Elem<T>::from_f(NB200_NAN);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(&h->merge_done, 1u) == gridDim.x - 1) {
        atomicExch(&h->merge_done, 0u);
        atomicExch(&h->ep, e);
    }
}

// Two launches per call of the column-sharded split (nb200_peer_fold): the partial fold storing
// its states straight into every rank's buffer, then peer_merge_kernel above. Each warp folds span
// items of this rank's shard (the split plan's span fold, so the states are bit-identical to
// nb200_fold_partial's) and lanes 0..world-1 store the item's tagged state into slot `rank` of
// every rank's buffer (parts past this rank's chunk count are stored empty). Nothing waits here;
// layouts are checked before any store (fault bit 3: nothing stored).
template <int S, typename T, int W>
__global__ void __launch_bounds__(kLdgThreads, 7)
peer_span_kernel(const T* __restrict__ x, LdgSpan pl, int64_t slot_parts, Params p, PeerPtrs peers, int world,
                 int rank, unsigned char* own) {
    pdl_wait();
    pdl_trigger();
    PeerHeader* h = reinterpret_cast<PeerHeader*>(own);
    const int64_t rows = pl.rows;
    __shared__ int layout_ok;
    if (threadIdx.x == 0) layout_ok = 1;
    __syncthreads();
    if (threadIdx.x < world && !peer_layout_ok(peer_at(peers, threadIdx.x), rows, slot_parts, world)) layout_ok = 0;
    __syncthreads();
    if (!layout_ok) {
        if (threadIdx.x == 0) atomicOr(&g_peer_fault, 8u);
        return;
    }
    const unsigned int e = *reinterpret_cast<volatile unsigned int*>(&h->ep) + 1u;
    const int64_t par = e & 1u;
    const int lane = threadIdx.x & 31;
    // slot of (row, part) in slot `rank` of any rank's buffer
    auto slot = [&](unsigned char* buf, int64_t row, int64_t part) {
        return reinterpret_cast<float4*>(buf + kPeerHeaderBytes) + ((par * rows + row) * world + rank) * slot_parts + part;
    };
    if constexpr (W == 1) {
        // lane r < world stores into rank r's buffer
        unsigned char* mine = lane < world ? peer_at(peers, lane) : nullptr;
        const int64_t gw = (int64_t)blockIdx.x * (kLdgThreads / 32) + (threadIdx.x >> 5);
        const int64_t GW = (int64_t)gridDim.x * (kLdgThreads / 32);
        for (int64_t item = gw; item < pl.nitems; item += GW) {
            const St w = span_item_state<S, T>(x, pl, item, lane, p);
            const int64_t row = item / pl.nparts, part = item - row * pl.nparts;
            if (mine)
                peer_slot_store(slot(mine, row, part), make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status)), e);
        }
    } else {
        span_items_shared<S, T, W>(x, pl, p, [&](int64_t item, const St& w) {
            const int64_t row = item / pl.nparts, part = item - row * pl.nparts;
            const float4 v = make_float4(w.m, w.acc, __int_as_float(w.seen), __int_as_float(w.status));
#pragma unroll
            for (int r = 0; r < kMaxPeers; ++r)
                if (r < world) peer_slot_store(slot(peers.p[r], row, part), v, e);
        });
    }
    // parts past this shard's chunk count (unequal shard widths): empty states
    const int64_t extra = slot_parts - pl.nparts;
    if (extra > 0) {
        const float4 v = make_float4(-NB200_INF, 0.f, 0.f, 0.f);
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows * extra * world;
             i += (int64_t)gridDim.x * blockDim.x) {
            const int r = (int)(i % world);
            const int64_t j = i / world, row = j / extra, part = pl.nparts + (j - row * extra);
            peer_slot_store(slot(peer_at(peers, r), row, part), v, e);
        }
    }
}

// ================================================================== host side
Params make_params(const nb200_params& q, int64_t ncols) {
    Params p;
    p.tiny = (float)q.tiny;
    p.alpha = (float)q.alpha;
    p.invT = q.T != 0.0 ? (float)(1.0 / q.T) : 0.f;
    p.beta = (float)q.beta;
    p.N = (float)q.N;
    p.eps = (float)q.eps;
    p.invN = ncols > 0 ? (float)(1.0 / (double)ncols) : 0.f;
    return p;
}

namespace {

constexpr int kWarpThreads = 256;

template <typename T>
bool rows_vectorizable(const T* x, int64_t rows, int64_t ncols, int64_t srow, int64_t scol) {
    constexpr int V = Elem<T>::V;
    return scol == 1 && aligned16(x) && (rows <= 1 || (srow * (int64_t)sizeof(T)) % 16 == 0) &&
           ncols % V == 0;
}

template <int S, typename T>
int fold_t(const T* x, T* out, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
           const Params& p, const nb200_launch* L, cudaStream_t st) {
    const bool vec = rows_vectorizable(x, rows, ncols, srow, scol);
    const int64_t bytes = ncols * (int64_t)sizeof(T);
    int variant = (L && L->variant) ? L->variant : (bytes <= 16384 ? NB200_VARIANT_WARP_ROW : NB200_VARIANT_CTA_ROW);
    const int cps = L ? L->ctas_per_sm : 0;
    if (variant == NB200_VARIANT_WARP_ROW) {
        auto k = vec ? fold_kernel<S, T, 4, true, false> : fold_kernel<S, T, kScalarNV<T>, false, false>;
        const int g = persistent_grid(k, kWarpThreads, 0, (rows + 7) / 8, cps);
        launch_pdl(k, g, kWarpThreads, 0, st, x, out, rows, ncols, srow, scol, p);
    } else {
        int threads = (L && L->threads) ? L->threads : (bytes >= 65536 ? 512 : 256);
        auto k = vec ? fold_kernel<S, T, 4, true, true> : fold_kernel<S, T, kScalarNV<T>, false, true>;
        const int g = persistent_grid(k, threads, 0, rows, cps);
        launch_pdl(k, g, threads, 0, st, x, out, rows, ncols, srow, scol, p);
    }
    count_launch();
    return finish_launch("nb200_fold");
}

template <typename T>
int fold_dispatch(int sk, const T* x, T* out, int64_t rows, int64_t ncols, int64_t srow,
                  int64_t scol, const Params& p, const nb200_launch* L, cudaStream_t st) {
    switch (sk) {
        case NB200_LOGSUMEXP: return fold_t<NB200_LOGSUMEXP, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_LSE_BIASED: return fold_t<NB200_LSE_BIASED, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_LSE_SCALED: return fold_t<NB200_LSE_SCALED, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_SOFTCAP_LSE: return fold_t<NB200_SOFTCAP_LSE, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_STABLE_L2: return fold_t<NB200_STABLE_L2, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_LINEAR_ATTN: return fold_t<NB200_LINEAR_ATTN, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_DECAY_RENORM: return fold_t<NB200_DECAY_RENORM, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_SUMSQ_DIV: return fold_t<NB200_SUMSQ_DIV, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_RMSNORM_MAX: return fold_t<NB200_RMSNORM_MAX, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_VARIANCE: return fold_t<NB200_VARIANCE, T>(x, out, rows, ncols, srow, scol, p, L, st);
        case NB200_STD: return fold_t<NB200_STD, T>(x, out, rows, ncols, srow, scol, p, L, st);
    }
    set_error("unknown skeleton %d", sk);
    return NB200_ERR_ARG;
}

// Chooses the register tile so that a row fits one chunk whenever it can: a warp per row up to
// 16 vectors per lane, then a CTA per row, then chunked (two reads of the row).
template <typename T, template <typename, int, bool, bool> class KS>
struct ReadoutPlan {
    template <typename F>
    static int run(const T* x, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
                   const nb200_launch* L, cudaStream_t st, F&& launch) {
        constexpr int V = Elem<T>::V;
        const bool vec = rows_vectorizable(x, rows, ncols, srow, scol);
        const int cps = L ? L->ctas_per_sm : 0;
        const int64_t vecs = (ncols + V - 1) / V;  // 16-byte vectors per row
        int variant = (L && L->variant) ? L->variant : (vecs <= 32 * 16 ? NB200_VARIANT_WARP_ROW : NB200_VARIANT_CTA_ROW);
        if (!vec) {
            if (variant == NB200_VARIANT_WARP_ROW) {
                auto k = KS<T, kScalarNV<T>, false, false>::get();
                return launch(k, persistent_grid(k, kWarpThreads, 0, (rows + 7) / 8, cps), kWarpThreads);
            }
            const int threads = (L && L->threads) ? L->threads : 256;
            auto k = KS<T, kScalarNV<T>, false, true>::get();
            return launch(k, persistent_grid(k, threads, 0, rows, cps), threads);
        }
        if (variant == NB200_VARIANT_WARP_ROW) {
            const int64_t per_lane = (vecs + 31) / 32;
            auto pick = [&]() {
                if (per_lane <= 1) return KS<T, 1, true, false>::get();
                if (per_lane <= 2) return KS<T, 2, true, false>::get();
                if (per_lane <= 4) return KS<T, 4, true, false>::get();
                if (per_lane <= 8) return KS<T, 8, true, false>::get();
                return KS<T, 16, true, false>::get();
            };
            auto k = pick();
            return launch(k, persistent_grid(k, kWarpThreads, 0, (rows + 7) / 8, cps), kWarpThreads);
        }
        const int threads = (L && L->threads) ? L->threads : 256;
        const int64_t per_thread = (vecs + threads - 1) / threads;
        auto pick = [&]() {
            if (per_thread <= 4) return KS<T, 4, true, true>::get();
            if (per_thread <= 8) return KS<T, 8, true, true>::get();
            return KS<T, 16, true, true>::get();
        };
        auto k = pick();
        return launch(k, persistent_grid(k, threads, 0, rows, cps), threads);
    }
};

template <typename T, int NV, bool VEC, bool CTA>
struct SoftmaxK {
    static auto get() { return softmax_kernel<T, NV, VEC, CTA>; }
};
template <typename T, int NV, bool VEC, bool CTA>
struct L2K {
    static auto get() { return l2norm_kernel<T, NV, VEC, CTA>; }
};

template <typename T>
int softmax_t(int mode, const T* x, T* y, T* lse, int64_t rows, int64_t ncols, int64_t srow,
              int64_t scol, const nb200_launch* L, cudaStream_t st) {
    const int out_vec = aligned16(y) && (ncols * (int64_t)sizeof(T)) % 16 == 0;
    return ReadoutPlan<T, SoftmaxK>::run(x, rows, ncols, srow, scol, L, st, [&](auto k, int g, int th) {
        launch_pdl(k, g, th, 0, st, x, y, lse, rows, ncols, srow, scol, mode, out_vec);
        count_launch();
        return finish_launch("nb200_softmax");
    });
}

template <typename T>
int l2_t(const T* x, T* y, T* norm, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
         const nb200_launch* L, cudaStream_t st) {
    const int out_vec = aligned16(y) && (ncols * (int64_t)sizeof(T)) % 16 == 0;
    return ReadoutPlan<T, L2K>::run(x, rows, ncols, srow, scol, L, st, [&](auto k, int g, int th) {
        launch_pdl(k, g, th, 0, st, x, y, norm, rows, ncols, srow, scol, out_vec);
        count_launch();
        return finish_launch("nb200_l2_normalize");
    });
}

template <int S, typename T>
int partial_t(const T* x, nb200_state* states, int64_t rows, int64_t cb, int64_t ns, int64_t srow,
              int64_t scol, int64_t cc, int64_t nparts, const Params& p, cudaStream_t st) {
    constexpr int V = Elem<T>::V;
    const bool vec = rows_vectorizable(x, rows, cb + ns, srow, scol) && cb % V == 0 && cc % V == 0;
    auto k = vec ? partial_kernel<S, T, true> : partial_kernel<S, T, false>;
    const int g = persistent_grid(k, 256, 0, rows * nparts, 0);
    launch_pdl(k, g, 256, 0, st, x, states, rows, cb, ns, srow, scol, cc, nparts, p);
    count_launch();
    return finish_launch("nb200_fold_partial");
}

template <int S, typename T>
int merge_t(const nb200_state* states, T* out, int64_t rows, int64_t nparts, int64_t rs, int64_t ps,
            const Params& p, cudaStream_t st) {
    auto k = merge_kernel<S, T>;
    const int g = persistent_grid(k, kMergeThreads, 0, (rows + kMergeThreads / 32 - 1) / (kMergeThreads / 32), 0);
    launch_pdl(k, g, kMergeThreads, 0, st, states, out, rows, nparts, rs, ps, p);
    count_launch();
    return finish_launch("nb200_fold_merge");
}

#define NB200_SPLIT_SKELETONS(X)                                                              \
    X(NB200_LOGSUMEXP) X(NB200_LSE_BIASED) X(NB200_LSE_SCALED) X(NB200_SOFTCAP_LSE)           \
    X(NB200_STABLE_L2) X(NB200_LINEAR_ATTN) X(NB200_DECAY_RENORM) X(NB200_SUMSQ_DIV)          \
    X(NB200_RMSNORM_MAX)

template <typename T>
int partial_dispatch(int sk, const T* x, nb200_state* states, int64_t rows, int64_t cb, int64_t ns,
                     int64_t srow, int64_t scol, int64_t cc, int64_t nparts, const Params& p,
                     cudaStream_t st) {
    switch (sk) {
#define X(S) case S: return partial_t<S, T>(x, states, rows, cb, ns, srow, scol, cc, nparts, p, st);
        NB200_SPLIT_SKELETONS(X)
#undef X
    }
    set_error("skeleton %d has no split plan (two-pass skeletons need extended carried state)", sk);
    return NB200_ERR_UNSUPPORTED;
}

template <typename T>
int peer_merge_dispatch(int sk, unsigned char* own, T* out, int64_t rows, int64_t nparts, int world,
                        const Params& p, cudaStream_t st) {
    switch (sk) {
#define X(S)                                                                       \
    case S: {                                                                      \
        auto k = peer_merge_kernel<S, T>;                                          \
        const int g = persistent_grid(k, 256, 0, (rows + 7) / 8, 0);               \
        launch_pdl(k, g, 256, 0, st, own, out, rows, nparts, world, p);            \
        count_launch();                                                            \
        return finish_launch("nb200_peer_merge");                                  \
    }
        NB200_SPLIT_SKELETONS(X)
#undef X
    }
    set_error("skeleton %d has no split plan (two-pass skeletons need extended carried state)", sk);
    return NB200_ERR_UNSUPPORTED;
}

template <typename T>
int peer_fold_dispatch(int sk, const T* x, const LdgSpan& pl, int64_t slot_parts, const PeerPtrs& pp, int world,
                       int rank, unsigned char* own, T* out, const Params& p, cudaStream_t st) {
    // the items' decomposition of the partial fold (span_item_warps), so the states match it bit for bit
    const int W = span_item_warps(pl.nitems, pl.cc / Elem<T>::V, sm_count());
    auto go = [&](auto k) {
        int occ = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, kLdgThreads, 0) != cudaSuccess || occ < 1) occ = 1;
        const int64_t warps = std::max<int64_t>(pl.nitems * W, 1);
        const int g = (int)std::max<int64_t>(1, std::min<int64_t>((warps + 3) / 4, (int64_t)sm_count() * occ));
        launch_pdl(k, (unsigned)g, kLdgThreads, 0, st, x, pl, slot_parts, p, pp, world, rank, own);
        count_launch();
        const int rc = finish_launch("nb200_peer_fold");
        return rc ? rc : peer_merge_dispatch<T>(sk, own, out, pl.rows, slot_parts, world, p, st);
    };
    switch (sk) {
#define X(S)                                                   \
    case S:                                                    \
        if (W == 4) return go(peer_span_kernel<S, T, 4>);      \
        return go(peer_span_kernel<S, T, 1>);
        NB200_SPLIT_SKELETONS(X)
#undef X
    }
    set_error("skeleton %d has no split plan (two-pass skeletons need extended carried state)", sk);
    return NB200_ERR_UNSUPPORTED;
}

template <typename T>
int merge_dispatch(int sk, const nb200_state* states, T* out, int64_t rows, int64_t nparts,
                   int64_t rs, int64_t ps, const Params& p, cudaStream_t st) {
    switch (sk) {
#define X(S) case S: return merge_t<S, T>(states, out, rows, nparts, rs, ps, p, st);
        NB200_SPLIT_SKELETONS(X)
#undef X
    }
    set_error("skeleton %d has no split plan (two-pass skeletons need extended carried state)", sk);
    return NB200_ERR_UNSUPPORTED;
}

}  // namespace

#define NB200_DTYPE_CASES(dtype, CALL)                                                  \
    switch (dtype) {                                                                  \
        case NB200_F32: { using T = float; return CALL; }                              \
        case NB200_BF16: { using T = __nv_bfloat16; return CALL; }                     \
        case NB200_F16: { using T = __half; return CALL; }                             \
    }                                                                                 \
    set_error("unknown dtype %d", dtype);                                             \
    return NB200_ERR_ARG;

// The library's own choice for a fold with no launch given (or variant AUTO), from the launch
// campaign measured on B200 (autotune.measure_shapes, logsumexp fp32 and bf16, device time):
// rows under 1 KB fold fastest one per warp from registers (1.2-1.9x over the bulk-copy ring),
// and fewer rows than SMs of 8-32 KB fastest one per CTA of 8 (<= 16 KB) or 16 warps (1.2-1.7x);
// the register-row and bulk-copy paths win everywhere else. Returns false to keep the default.
static bool fold_auto_override(int dtype, int64_t rows, int64_t ncols, nb200_launch& out) {
    const int64_t rb = ncols * (int64_t)dtype_size(dtype);
    if (rb < 1024) {
        out = nb200_launch{NB200_VARIANT_WARP_ROW, 0, 0, 0};
        return true;
    }
    if (rb > 8192 && rb <= 32768 && rows < (int64_t)sm_count()) {
        out = nb200_launch{NB200_VARIANT_CTA_ROW, rb <= 16384 ? 256 : 512, 0, 0};
        return true;
    }
    return false;
}

// Rows a thread-block cluster per row folds in one launch: contiguous, 16-byte aligned, one-pass
// skeletons.
static bool cluster_rows_ok(int sk, const void* x, int dtype, int64_t ncols, int64_t srow, int64_t scol) {
    const int64_t es = dtype_size(dtype);
    return sk != NB200_VARIANCE && sk != NB200_STD && scol == 1 && aligned16(x) && (ncols * es) % 16 == 0 &&
           (srow * es) % 16 == 0;
}

// Up to two rows per SM wider than 32 KB: one cluster of CTAs per row (measured on B200: fp32
// [1, 262144] 6.8 us against 24.9 us for the two-launch split and 110 us for one CTA per row;
// fp32 [256, 16384] 9.5 us against 11.3 us for the default path).
static bool cluster_auto(int sk, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol) {
    return rows >= 1 && rows <= 2 * (int64_t)sm_count() && ncols * (int64_t)dtype_size(dtype) > 32768 &&
           cluster_rows_ok(sk, x, dtype, ncols, srow, scol);
}

static int cluster_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow,
                        void* out, int csize, cudaStream_t st) {
    NB200_DTYPE_CASES(dtype, launch_cluster_fold<T>(sk, p, (const T*)x, rows, ncols, srow, (T*)out, csize, st))
}

int launch_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols,
                int64_t srow, int64_t scol, void* out, const nb200_launch* L, cudaStream_t st) {
    const bool want_cluster = L ? L->variant == NB200_VARIANT_CLUSTER
                                : cluster_auto(sk, x, dtype, rows, ncols, srow, scol);
    if (want_cluster || (L && L->variant == NB200_VARIANT_AUTO && cluster_auto(sk, x, dtype, rows, ncols, srow, scol))) {
        const int rc = cluster_rows_ok(sk, x, dtype, ncols, srow, scol)
                           ? cluster_fold(sk, p, x, dtype, rows, ncols, srow, out, L ? L->stages : 0, st)
                           : 0;
        if (rc != 0) return rc < 0 ? rc : NB200_OK;
        if (L && L->variant == NB200_VARIANT_CLUSTER) {
            set_error("nb200_fold: the cluster variant needs contiguous 16-byte-aligned rows and a one-pass skeleton");
            return NB200_ERR_ARG;
        }
    }
    nb200_launch chosen;
    if ((!L || L->variant == NB200_VARIANT_AUTO) && fold_auto_override(dtype, rows, ncols, chosen)) L = &chosen;
    if (!L || L->variant == NB200_VARIANT_AUTO || L->variant == NB200_VARIANT_STREAM) {
        int rc = stream_fold(sk, p, x, dtype, rows, ncols, srow, scol, out, L, st);
        // rows too wide for a stage: one warp streams each row, when there are enough rows to
        // occupy every warp slot; otherwise the CTA-per-row register kernel spreads a row wider
        if (rc == 0 && rows >= (int64_t)sm_count() * 8)
            rc = stream_span(sk, p, x, dtype, rows, 0, ncols, srow, scol, ncols, 1, nullptr, out, 1, L, st);
        if (rc != 0) return rc < 0 ? rc : NB200_OK;
        if (L && L->variant == NB200_VARIANT_STREAM) {
            set_error("nb200_fold: the streaming variant needs contiguous 16-byte-aligned rows");
            return NB200_ERR_ARG;
        }
    }
    NB200_DTYPE_CASES(dtype, fold_dispatch<T>(sk, (const T*)x, (T*)out, rows, ncols, srow, scol, p, L, st))
}

int launch_softmax(int mode, const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow,
                   int64_t scol, void* y, void* lse, const nb200_launch* L, cudaStream_t st) {
    if (!L || L->variant == NB200_VARIANT_AUTO || L->variant == NB200_VARIANT_STREAM) {
        const int rc = stream_softmax(mode, x, dtype, rows, ncols, srow, scol, y, lse, L, st);
        if (rc != 0) return rc < 0 ? rc : NB200_OK;
        if (L && L->variant == NB200_VARIANT_STREAM) {
            set_error("nb200_softmax: the streaming variant needs contiguous 16-byte-aligned rows of <= 32 KB");
            return NB200_ERR_ARG;
        }
    }
    NB200_DTYPE_CASES(dtype, softmax_t<T>(mode, (const T*)x, (T*)y, (T*)lse, rows, ncols, srow, scol, L, st))
}

int launch_l2(const void* x, int dtype, int64_t rows, int64_t ncols, int64_t srow, int64_t scol,
              void* y, void* norm, const nb200_launch* L, cudaStream_t st) {
    if (!L || L->variant == NB200_VARIANT_AUTO || L->variant == NB200_VARIANT_STREAM) {
        const int rc = stream_l2(x, dtype, rows, ncols, srow, scol, y, norm, L, st);
        if (rc != 0) return rc < 0 ? rc : NB200_OK;
        if (L && L->variant == NB200_VARIANT_STREAM) {
            set_error("nb200_l2_normalize: the streaming variant needs contiguous 16-byte-aligned rows of <= 32 KB");
            return NB200_ERR_ARG;
        }
    }
    NB200_DTYPE_CASES(dtype, l2_t<T>((const T*)x, (T*)y, (T*)norm, rows, ncols, srow, scol, L, st))
}

int launch_partial(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t cb,
                   int64_t ns, int64_t srow, int64_t scol, int64_t cc, int64_t nparts,
                   nb200_state* states, const nb200_launch* L, cudaStream_t st) {
    const int rc = stream_span(sk, p, x, dtype, rows, cb, ns, srow, scol, cc, nparts, states, nullptr, 0, L, st);
    if (rc != 0) return rc < 0 ? rc : NB200_OK;
    NB200_DTYPE_CASES(dtype, partial_dispatch<T>(sk, (const T*)x, states, rows, cb, ns, srow, scol, cc, nparts, p, st))
}

int launch_merge(int sk, const Params& p, const nb200_state* states, int64_t rows, int64_t nparts,
                 int64_t rs, int64_t ps, void* out, int dtype, cudaStream_t st) {
    NB200_DTYPE_CASES(dtype, merge_dispatch<T>(sk, states, (T*)out, rows, nparts, rs, ps, p, st))
}

int64_t peer_buffer_bytes(int64_t rows, int64_t world, int64_t nparts) {
    return kPeerHeaderBytes + 2 * rows * world * nparts * (int64_t)sizeof(nb200_state);
}

int peer_max_world() { return kMaxPeers; }

int launch_peer_init(void* buffer, int64_t rows, int64_t nparts, int world, cudaStream_t st) {
    const int64_t nslots = 2 * rows * world * nparts;
    const int g = (int)std::min<int64_t>(std::max<int64_t>((nslots + 255) / 256, 1), 1024);
    launch_pdl(peer_init_kernel, g, 256, 0, st, static_cast<unsigned char*>(buffer), rows, nparts, world);
    count_launch();
    return finish_launch("nb200_peer_init");
}

int launch_peer_push(const nb200_state* states, int64_t rows, int64_t nlocal, int64_t nparts, void* const* peers,
                     int world, int rank, void* own, cudaStream_t st) {
    PeerPtrs pp{};
    for (int r = 0; r < world; ++r) pp.p[r] = static_cast<unsigned char*>(peers[r]);
    launch_pdl(peer_push_kernel, world, kPushThreads, 0, st, states, rows, nlocal, nparts, pp, world, rank,
               static_cast<unsigned char*>(own));
    count_launch();
    return finish_launch("nb200_peer_push");
}

int launch_peer_merge(int sk, const Params& p, void* own, int64_t rows, int64_t nparts, int world, void* out,
                      int dtype, cudaStream_t st) {
    NB200_DTYPE_CASES(dtype, peer_merge_dispatch<T>(sk, static_cast<unsigned char*>(own), (T*)out, rows, nparts,
                                                    world, p, st))
}

int launch_peer_fold(int sk, const Params& p, const void* x, int dtype, int64_t rows, int64_t ncols_shard,
                     int64_t srow, int64_t chunk, int64_t nparts, void* const* peers, int world, int rank, void* own,
                     void* out, cudaStream_t st) {
    const int64_t es = dtype_size(dtype), V = 16 / es;
    if (!aligned16(x) || (rows > 1 && (srow * es) % 16 != 0) || ncols_shard % V != 0 || chunk % V != 0) {
        set_error("nb200_peer_fold: needs a contiguous, 16-byte aligned shard whose width and chunk are multiples of "
                  "%lld elements", (long long)V);
        return NB200_ERR_ARG;
    }
    if (chunk / V <= 32 * kSpanNV) {  // the partial fold holds such chunks as resident rows instead
        set_error("nb200_peer_fold: chunks of at most %lld columns take the partial fold + nb200_peer_push form",
                  (long long)(32 * kSpanNV * V));
        return NB200_ERR_UNSUPPORTED;
    }
    const int64_t nlocal = (ncols_shard + chunk - 1) / chunk;
    if (nlocal > nparts) {
        set_error("nb200_peer_fold: the shard has %lld chunks, more than the exchange's %lld parts per rank",
                  (long long)nlocal, (long long)nparts);
        return NB200_ERR_ARG;
    }
    PeerPtrs pp{};
    for (int r = 0; r < world; ++r) pp.p[r] = static_cast<unsigned char*>(peers[r]);
    const LdgSpan pl{rows, srow, 0, ncols_shard, chunk, nlocal, rows * nlocal, 0};
    NB200_DTYPE_CASES(dtype, peer_fold_dispatch<T>(sk, (const T*)x, pl, nparts, pp, world, rank,
                                                   static_cast<unsigned char*>(own), (T*)out, p, st))
}

int peer_fault_take(unsigned int* bits) {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_peer_fault, sizeof(v)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_peer_fault, &zero, sizeof(zero)) != cudaSuccess) {
        set_error("cannot read the peer-exchange fault word: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    *bits = v;
    return NB200_OK;
}

}  // namespace nb200
