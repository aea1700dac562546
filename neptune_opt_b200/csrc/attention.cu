// Fused single-pass attention forward, O = softmax(scale * Q K^T [+ causal mask]) V, bf16 in and
// out, fp32 scores and online max/sum repair, on the sm_100a tensor cores.
//
// One CTA owns 256 query rows of one (batch, head): two query tiles of 128 rows, one tensor-memory
// lane per row. The K/V sequence streams through a ring of shared-memory stages filled by
// tensor-map (TMA) loads; one thread issues the tcgen05 MMAs; two softmax warpgroups, one per
// query tile, hold one query row per thread.
//
//   warp 9      producer: Q tiles once, then K_0, V_0, K_1, V_1, ... into the stage ring
//   warp 8      MMA: S_t = Q_t K_j^T (shared x shared -> TMEM, fp32)
//                    O_t += P_t V_j    (P from TMEM, V from shared -> TMEM, fp32)
//   warps 0-7   softmax for tile t = warp / 4: read S_t, update the running max (log2 domain),
//               rescale O_t in TMEM when the max grew by more than 2^8, write P_t = 2^(s - m)
//               as bf16 into the upper half of S_t's columns, accumulate the row sum;
//               at the end O_t / l -> bf16 -> shared -> TMA store, and the row's log-sum-exp.
//
// TMEM (512 columns x 128 lanes of 32 bits): S_0 [0,128), S_1 [128,256), O_0 [256,384),
// O_1 [384,512); P_t occupies columns [64,128) of S_t.
//
// MMA issue order per key tile j: PV_0(j), S_0(j+1), PV_1(j), S_1(j+1). tcgen05.commit arrives
// only when every earlier MMA of the issuing thread has finished, so the arrival of S_t(j+1)
// also means PV_t(j) is complete: the softmax warps may rescale O_t between reading S_t(j+1) and
// publishing P_t(j+1) without a separate barrier. S_t(j+1) overwrites the columns PV_t(j) reads
// P_t(j) from; the tensor pipe executes one thread's MMAs in issue order. Under a causal mask
// query tile 0 stops one key tile early: its rows end where tile 1's begin, so the unit's last key
// tile lies entirely above tile 0's diagonal.
//
// Every wait is bounded (about a second of SM clock). A wait that runs out sets bit 1 of the
// attention fault word and the CTA's abort flag; the other roles stop at their next wait, the
// producer waits for the copies it issued, the MMA thread waits for its MMAs, and the CTA frees
// its tensor memory and exits with the output unwritten.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "launch.h"
#include "fastmath.cuh"
#include "tcgen05.cuh"

namespace nb200 {
namespace {

static __device__ unsigned int g_attn_fault = 0u;

constexpr int kRows = 128;   // query rows per tile (= TMEM lanes)
constexpr int kQTiles = 2;   // query tiles per CTA
constexpr int kKeys = 128;   // keys per K/V tile
constexpr int kDim = 128;    // head dimension
constexpr int kStages = 5;   // K/V ring stages; each holds one K or one V tile
constexpr uint32_t kTileBytes = kRows * kDim * 2;  // 32 KB per Q, K or V tile
constexpr uint32_t kHalfBytes = kTileBytes / 2;    // one 64-column half: the TMA box
constexpr int kMmaWarp = 8;
constexpr int kLoadWarp = 9;
constexpr int kThreads = 384;  // warps 10-11 only complete the third warpgroup for the register split
// Register split (setmaxnreg, per warpgroup): the softmax warpgroups hold a 128-column score row
// per thread; the MMA/producer warpgroup needs little. The sum stays within what the block is
// launched with (kThreads x kLaunchRegs), so the increase never waits on registers that do not exist.
constexpr int kLaunchRegs = 168;
constexpr int kRegsSoftmax = 216;
constexpr int kRegsControl = 72;
static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsControl <= kThreads * kLaunchRegs, "register split");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS0 = 0, kColO0 = 256;  // tile t: S at kColS0 + 128 t, O at kColO0 + 128 t
constexpr uint32_t kColP = 64;                // P inside S's columns
// P is published in kPParts parts of 128 / kPParts keys; the MMA thread issues each part's P V
// steps as soon as that part is in TMEM. Two parts measured fastest (interleaved A/B on one box,
// non-causal: 2 parts 1059-1222, 4 parts 1001-1096, 8 parts 857-915 TFLOP/s): every further
// hand-off (store wait, fence, arrival, one more wait in the MMA thread) costs more than the extra
// overlap of the P V MMAs with the exponentials gains.
#ifndef NB200_ATTN_PPARTS
#define NB200_ATTN_PPARTS 2
#endif
constexpr int kPParts = NB200_ATTN_PPARTS;
constexpr int kPairsPerPart = 64 / kPParts;  // TMEM columns of P per part (two keys per column)
constexpr int kStepsPerPart = 8 / kPParts;   // K=16 P V MMA steps per part
static_assert(kPParts == 2 || kPParts == 4 || kPParts == 8, "P parts");
constexpr float kRescaleSlack = 8.f;          // keep a stale max while the new one is < 2^8 above it
constexpr uint32_t kIdescQK = tc::idesc_bf16(128, 128, false);
constexpr uint32_t kIdescPV = tc::idesc_bf16(128, 128, true);
constexpr long long kWaitCycles = 1ll << 31;

// Shared-memory layout (offsets from a 1024-byte aligned base).
constexpr uint32_t kOffQ = 0;                                // kQTiles tiles
constexpr uint32_t kOffKV = kOffQ + kQTiles * kTileBytes;    // kStages tiles
constexpr uint32_t kOffBar = kOffKV + kStages * kTileBytes;  // mbarriers
struct Bars {
    uint64_t q_full[kQTiles];
    uint64_t kv_full[kStages];
    uint64_t kv_empty[kStages];
    uint64_t s_full[kQTiles];
    uint64_t p_full[kQTiles][kPParts];  // per part of P (128 / kPParts keys each)
    uint64_t o_final;
    uint32_t tmem_base;
    int abort;
};
constexpr uint32_t kSmemBytes = kOffBar + sizeof(Bars) + 1024;  // + alignment slack

struct AttnArgs {
    int S;        // sequence length (queries = keys)
    int BH;       // batch * heads
    int nqb;      // query blocks of kQTiles * kRows rows per (batch, head)
    int causal;
    float sl2;    // scale * log2(e)
    float* lse;   // [BH, S] natural log-sum-exp, nullable
};

// Bounded wait on phase `parity` of `bar`. Gives up early when another role has aborted the CTA.
// (Inline on purpose: a called function would need one register budget for roles that run under
// different setmaxnreg limits.)
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t i = 1; i < (1u << 30); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort) return false;
            if (clock64() - t0 > kWaitCycles) break;
        }
    }
    atomicOr(&g_attn_fault, 2u);
    *abort = 1;
    return false;
}

// Position in the K/V stage ring: stage index and the parity of its current fill.
struct Ring {
    int s = 0;
    uint32_t ph = 0;
    __device__ __forceinline__ void next() {
        if (++s == kStages) {
            s = 0;
            ph ^= 1u;
        }
    }
};

// Bounded wait used while shutting down: ignores the abort flag (outstanding copies and MMAs
// must land before the CTA exits) but still gives up after the same limit.
__device__ __forceinline__ void drain_bar(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return;
    const long long t0 = clock64();
    for (uint32_t i = 1; i < (1u << 30); ++i) {
        if (mbar_try_wait(bar, parity)) return;
        if ((i & 255u) == 0 && clock64() - t0 > kWaitCycles) break;
    }
    atomicOr(&g_attn_fault, 2u);
}

// P for part qp of this row's keys: p = 2^(s * sl2 - m) on the special-function unit,
// rounded to bf16 into TMEM (one column per key pair, the lower key in the low half), fp32 p added
// to the row sums. (Computing a share of the exponentials with an FMA-pipe polynomial instead was
// measured slower at every share tried, 2/8 to 5/8 of the pairs: the softmax warps run out of
// issue slots before the special-function unit saturates.)
template <int kPairs = kPairsPerPart>
__device__ __forceinline__ void p_part(const float* s, int qp, uint64_t sl2, uint64_t nm, uint64_t& acc0,
                                       uint64_t& acc1, uint32_t tP) {
    uint32_t pk[kPairs];
#pragma unroll
    for (int i = 0; i < kPairs; ++i) {
        const int pi = kPairs * qp + i;
        const uint64_t x = fma2(f2(s[2 * pi], s[2 * pi + 1]), sl2, nm);
        const uint64_t p = f2(ex2_ftz(f2lo(x)), ex2_ftz(f2hi(x)));
        if (i & 1)
            acc1 = add2(acc1, p);
        else
            acc0 = add2(acc0, p);
        pk[i] = tc::pack_bf16(f2lo(p), f2hi(p));
    }
    const uint32_t col = tP + kPairs * qp;
    if constexpr (kPairs == 32) {
        tc::tmem_st16(col, pk);
        tc::tmem_st16(col + 16, pk + 16);
    } else if constexpr (kPairs == 16) {
        tc::tmem_st16(col, pk);
    } else {
        tc::tmem_st8(col, pk);
    }
}

__device__ __forceinline__ void producer(const CUtensorMap* mq, const CUtensorMap* mk, const CUtensorMap* mv,
                                         uint8_t* smem, Bars* b, int bh, int q0, int n) {
    volatile int* abort = &b->abort;
    tc::prefetch_map(mq);
    tc::prefetch_map(mk);
    tc::prefetch_map(mv);
    for (int t = 0; t < kQTiles; ++t) {
        uint8_t* dst = smem + kOffQ + t * kTileBytes;
        mbar_expect_tx(&b->q_full[t], kTileBytes);
        tc::tma_load_3d(dst, mq, 0, q0 + t * kRows, bh, &b->q_full[t]);
        tc::tma_load_3d(dst + kHalfBytes, mq, kDim / 2, q0 + t * kRows, bh, &b->q_full[t]);
    }
    int it = 0;
    Ring r;
    for (; it < 2 * n; ++it, r.next()) {
        const int s = r.s;
        if (!wait_bar(&b->kv_empty[s], r.ph ^ 1u, abort)) break;
        uint8_t* dst = smem + kOffKV + s * kTileBytes;
        const CUtensorMap* m = (it & 1) ? mv : mk;
        const int row = (it >> 1) * kKeys;
        mbar_expect_tx(&b->kv_full[s], kTileBytes);
        tc::tma_load_3d(dst, m, 0, row, bh, &b->kv_full[s]);
        tc::tma_load_3d(dst + kHalfBytes, m, kDim / 2, row, bh, &b->kv_full[s]);
    }
    // Every copy issued into this CTA's shared memory lands before the CTA may exit: wait for the
    // last phase filled in each stage (`it` tiles were issued, stage s got those with index = s
    // mod kStages).
    for (int t = 0; t < kQTiles; ++t) drain_bar(&b->q_full[t], 0);
    for (int s = 0; s < kStages && s < it; ++s) drain_bar(&b->kv_full[s], ((it - 1 - s) / kStages) & 1u);
}

// n K/V tiles in the unit; query tile 0 uses the first n0 of them (n0 = n, or n - 1 under a causal
// mask, where tile 0's rows end 128 keys before tile 1's).
__device__ __forceinline__ void mma_issuer(uint8_t* smem, Bars* b, uint32_t tmem, int n0, int n) {
    volatile int* abort = &b->abort;
    // Descriptors are built once; an operand step only adds its byte offset / 16 to the start-
    // address field (bits 0-13, which cannot carry: shared addresses stay below 2^18 bytes).
    const uint64_t q_desc = tc::sw128_desc(smem_u32(smem + kOffQ), 16, 1024);
    const uint64_t k_desc = tc::sw128_desc(smem_u32(smem + kOffKV), 16, 1024);
    const uint64_t v_desc = tc::sw128_desc(smem_u32(smem + kOffKV), kHalfBytes, 1024);
    // S_t = Q_t K^T: eight K=16 steps along the head dimension; 32 bytes per step inside a
    // 128-byte swizzled row, the second 64 columns in the other half tile.
    auto qk = [&](int t, int s) {
        const uint64_t qa = q_desc + ((t * kTileBytes) >> 4), ka = k_desc + ((s * kTileBytes) >> 4);
        const uint32_t d = tmem + kColS0 + 128 * t;
        constexpr uint32_t h = kHalfBytes >> 4;  // second 64 head columns
        tc::mma_ss_at<0>(d, qa, ka, kIdescQK, 0u);
        tc::mma_ss_at<2>(d, qa, ka, kIdescQK, 1u);
        tc::mma_ss_at<4>(d, qa, ka, kIdescQK, 1u);
        tc::mma_ss_at<6>(d, qa, ka, kIdescQK, 1u);
        tc::mma_ss_at<h + 0>(d, qa, ka, kIdescQK, 1u);
        tc::mma_ss_at<h + 2>(d, qa, ka, kIdescQK, 1u);
        tc::mma_ss_at<h + 4>(d, qa, ka, kIdescQK, 1u);
        tc::mma_ss_at<h + 6>(d, qa, ka, kIdescQK, 1u);
    };
    // O_t += P_t V: eight K=16 steps along the keys; P from TMEM (8 columns per step), V as an
    // MN-major operand (head dimension contiguous, 16 key rows = 2048 bytes per step, the second
    // 64 head columns 16 KB further).
    // One K=16 step k of O_t += P_t V (compile-time k after unrolling).
    auto pv_step = [&](int k, uint32_t d, uint32_t pa, uint64_t va, uint32_t acc) {
        switch (k) {
            case 0: tc::mma_ts_at<0, 0>(d, pa, va, kIdescPV, acc); break;
            case 1: tc::mma_ts_at<8, 128>(d, pa, va, kIdescPV, acc); break;
            case 2: tc::mma_ts_at<16, 256>(d, pa, va, kIdescPV, acc); break;
            case 3: tc::mma_ts_at<24, 384>(d, pa, va, kIdescPV, acc); break;
            case 4: tc::mma_ts_at<32, 512>(d, pa, va, kIdescPV, acc); break;
            case 5: tc::mma_ts_at<40, 640>(d, pa, va, kIdescPV, acc); break;
            case 6: tc::mma_ts_at<48, 768>(d, pa, va, kIdescPV, acc); break;
            default: tc::mma_ts_at<56, 896>(d, pa, va, kIdescPV, acc); break;
        }
    };
    // Issued part by part, each as soon as the softmax warps publish that part of P.
    auto pv_tile = [&](int t, int s, bool acc, uint32_t parity) {
        const uint64_t va = v_desc + ((s * kTileBytes) >> 4);
        const uint32_t d = tmem + kColO0 + 128 * t, pa = tmem + kColS0 + 128 * t + kColP;
#pragma unroll
        for (int qp = 0; qp < kPParts; ++qp) {
            if (!wait_bar(&b->p_full[t][qp], parity, abort)) return false;
            tc::fence_after();
#pragma unroll
            for (int kk = 0; kk < kStepsPerPart; ++kk) {
                const int k = qp * kStepsPerPart + kk;
                pv_step(k, d, pa, va, (acc || k > 0) ? 1u : 0u);
            }
        }
        return true;
    };
    // kr: the next K tile's stage, vr: the next V tile's stage (tiles alternate K_0, V_0, K_1, ...).
    Ring kr, vr;
    vr.next();
    bool ok = wait_bar(&b->q_full[0], 0, abort) && wait_bar(&b->q_full[1], 0, abort) &&
              wait_bar(&b->kv_full[kr.s], kr.ph, abort);
    if (ok) {
        tc::fence_after();
        qk(0, kr.s);
        tc::commit(&b->s_full[0]);
        qk(1, kr.s);
        tc::commit(&b->s_full[1]);
        tc::commit(&b->kv_empty[kr.s]);
        kr.next();
        kr.next();
    }
    for (int j = 0; ok && j < n; ++j) {
        const bool more = j + 1 < n;
        if (!(ok = wait_bar(&b->kv_full[vr.s], vr.ph, abort))) break;
        if (j < n0 && !(ok = pv_tile(0, vr.s, j > 0, j & 1u))) break;
        if (more) {
            if (!(ok = wait_bar(&b->kv_full[kr.s], kr.ph, abort))) break;
            tc::fence_after();
            if (j + 1 < n0) {
                qk(0, kr.s);
                tc::commit(&b->s_full[0]);
            }
        }
        if (!(ok = pv_tile(1, vr.s, j > 0, j & 1u))) break;
        tc::commit(&b->kv_empty[vr.s]);
        vr.next();
        vr.next();
        if (more) {
            qk(1, kr.s);
            tc::commit(&b->s_full[1]);
            tc::commit(&b->kv_empty[kr.s]);
            kr.next();
            kr.next();
        }
    }
    // Arrives when every MMA above has finished (at once if none was issued).
    tc::commit(&b->o_final);
    drain_bar(&b->o_final, 0);
}

__device__ __forceinline__ void softmax_tile(const CUtensorMap* mo, uint8_t* smem, Bars* b, uint32_t tmem,
                                             const AttnArgs& a, int bh, int q0, int n) {
    volatile int* abort = &b->abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = warp >> 2, wq = warp & 3;
    const int r = wq * 32 + lane;  // row inside the tile = TMEM lane
    const int qrow = q0 + t * kRows + r;
    const int lim = a.causal ? min(qrow, a.S - 1) : a.S - 1;  // last key this row attends to
    const uint32_t lanes = (uint32_t)(wq * 32) << 16;
    const uint32_t tS = tmem + lanes + kColS0 + 128 * t;
    const uint32_t tP = tS + kColP;
    const uint32_t tO = tmem + lanes + kColO0 + 128 * t;
    const float sl2 = a.sl2;
    float m = -NB200_INF, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
        // All lanes take the same branch: the TMEM accesses below are warp-collective.
        if (!(ok = __all_sync(0xffffffffu, wait_bar(&b->s_full[t], j & 1u, abort)))) break;
        tc::fence_after();
        uint32_t u[128];
        tc::tmem_ld128(tS, u);
        float s[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(u[c]);
        const int kb = j * kKeys;
        // Warp-uniform: the tile holds a key past some row's last (causal diagonal, ragged end).
        const bool masked = __any_sync(0xffffffffu, kb + kKeys - 1 > lim);
        if (masked) {
#pragma unroll
            for (int c = 0; c < 128; ++c)
                if (kb + c > lim) s[c] = -NB200_INF;
        }
        float a0 = s[0], a1 = s[1], a2 = s[2], a3 = s[3];
#pragma unroll
        for (int c = 4; c < 124; c += 8) {
            a0 = max3(a0, s[c], s[c + 1]);
            a1 = max3(a1, s[c + 2], s[c + 3]);
            a2 = max3(a2, s[c + 4], s[c + 5]);
            a3 = max3(a3, s[c + 6], s[c + 7]);
        }
        a0 = max3(a0, s[124], s[125]);
        a1 = max3(a1, s[126], s[127]);
        const float mnew = fmaxf(m, fmaxf(max3(a0, a1, a2), a3) * sl2);
        const bool grow = mnew > m + kRescaleSlack;
        if (__any_sync(0xffffffffu, grow)) {
            // Move the whole warp to the new maxima; rows whose max did not move keep factor 1.
            const float f = (mnew == m) ? 1.f : ex2(m - mnew);
            if (j > 0) {
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t v[32];
                    tc::tmem_ld32(tO + 32 * c, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __float_as_uint(__uint_as_float(v[i]) * f);
                    tc::tmem_st32(tO + 32 * c, v);
                }
            }
            l *= f;
            m = mnew;
        }
        const uint64_t sl2x2 = f2(sl2, sl2), nm = f2(-m, -m);
        uint64_t acc0 = 0, acc1 = 0;  // packed fp32 partial row sums (+0.0 bit patterns)
#pragma unroll
        for (int qp = 0; qp < kPParts; ++qp) {
            p_part(s, qp, sl2x2, nm, acc0, acc1, tP);
            tc::tmem_wait_st();
            tc::fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&b->p_full[t][qp]);
        }
        const uint64_t acc = add2(acc0, acc1);
        l += f2lo(acc) + f2hi(acc);
    }
    if (ok) ok = __all_sync(0xffffffffu, wait_bar(&b->o_final, 0, abort));
    if (!ok) return;
    tc::fence_after();
    // Epilogue: O / l in bf16, written into this tile's (now idle) Q buffer in the swizzled layout
    // the O tensor map expects, then one TMA store per warp for its 32 rows.
    uint8_t* stage = smem + kOffQ + t * kTileBytes;
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        uint32_t v[32];
        tc::tmem_ld32(tO + 32 * c, v);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
            pk[i] = tc::pack_bf16(__uint_as_float(v[2 * i]) * inv, __uint_as_float(v[2 * i + 1]) * inv);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int ch = 4 * c + q;  // 16-byte chunk of the 256-byte row
            uint8_t* dst = stage + (ch >> 3) * kHalfBytes + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
    }
    if (a.lse && qrow < a.S) a.lse[(size_t)bh * a.S + qrow] = (m + log2f(l)) * 0.69314718055994531f;
    fence_proxy_async();
    __syncwarp();
    const int row0 = q0 + t * kRows + wq * 32;
    if (lane == 0 && row0 < a.S) {
        tc::tma_store_3d(mo, stage + wq * 32 * 128, 0, row0, bh);
        tc::tma_store_3d(mo, stage + kHalfBytes + wq * 32 * 128, kDim / 2, row0, bh);
        tc::bulk_commit();
        tc::bulk_wait_read();
    }
    __syncwarp();
}

__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mo, AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* b = reinterpret_cast<Bars*>(smem + kOffBar);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Head-major order: the query blocks of one (batch, head) run side by side and share its K/V
    // through L2, so each head's K/V is read from HBM about once. Within a head the longest causal
    // blocks go first.
    const int bh = (int)(blockIdx.x / (unsigned)a.nqb);
    const int qb = a.nqb - 1 - (int)(blockIdx.x % (unsigned)a.nqb);
    const int q0 = qb * kQTiles * kRows;
    const int kv_end = a.causal ? min(q0 + kQTiles * kRows, a.S) : a.S;
    const int n = (kv_end + kKeys - 1) / kKeys;
    // Query tile 0 of a causal unit ends 128 rows earlier: its last K/V tile would be fully masked.
    const int n0 = a.causal ? (min(q0 + kRows, a.S) + kKeys - 1) / kKeys : n;

    if (threadIdx.x == 0) {
        for (int t = 0; t < kQTiles; ++t) {
            mbar_init(&b->q_full[t], 1);
            mbar_init(&b->s_full[t], 1);
            for (int qp = 0; qp < kPParts; ++qp) mbar_init(&b->p_full[t][qp], 4);  // one arrival per softmax warp
        }
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&b->kv_full[s], 1);
            mbar_init(&b->kv_empty[s], 1);
        }
        mbar_init(&b->o_final, 1);
        b->abort = 0;
        fence_barrier_init();
    }
    if (warp == kMmaWarp) {
        tc::tmem_alloc(&b->tmem_base, kTmemCols);
        tc::tmem_relinquish();
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    const uint32_t tmem = b->tmem_base;

    // Each role runs to the end of the kernel in its own branch (the register budget differs per
    // branch); both end at barrier 0, after which the MMA warp frees the tensor memory.
    if (warp < 8) {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsSoftmax));
        softmax_tile(&mo, smem, b, tmem, a, bh, q0, warp < 4 ? n0 : n);
        tc::fence_before();
        asm volatile("bar.sync 0;" ::: "memory");
    } else {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsControl));
        if (warp == kLoadWarp) {
            if (lane == 0) producer(&mq, &mk, &mv, smem, b, bh, q0, n);
            __syncwarp();
        } else if (warp == kMmaWarp) {
            if (lane == 0) mma_issuer(smem, b, tmem, n0, n);
            __syncwarp();
        }
        tc::fence_before();
        asm volatile("bar.sync 0;" ::: "memory");
        if (warp == kMmaWarp) {
            tc::fence_after();
            tc::tmem_dealloc(tmem, kTmemCols);
        }
    }
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
std::mutex g_attr_mutex;
bool g_attr_set[64] = {false};

int get_encoder() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        cudaGetLastError();
    });
    if (!g_encode) {
        set_error("nb200_attention: the driver does not provide cuTensorMapEncodeTiled");
        return NB200_ERR_LAUNCH;
    }
    return NB200_OK;
}

// [BH, S, D] bf16 viewed as a 3-D tensor map with a {64, box_rows, 1} box and 128-byte swizzle.
int encode_map(CUtensorMap* map, const void* base, int64_t BH, int64_t S, uint32_t box_rows, const char* what) {
    const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)S, (cuuint64_t)BH};
    const cuuint64_t strides[2] = {(cuuint64_t)kDim * 2, (cuuint64_t)S * kDim * 2};
    const cuuint32_t box[3] = {kDim / 2, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUresult rc = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                                 box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (rc != CUDA_SUCCESS) {
        set_error("nb200_attention: cannot describe %s as a tensor map (CUresult %d)", what, (int)rc);
        return NB200_ERR_ARG;
    }
    return NB200_OK;
}

}  // namespace

int attn_fault_take(unsigned int* bits) {
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_attn_fault, sizeof(v)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_attn_fault, &zero, sizeof(zero)) != cudaSuccess) {
        set_error("cannot read the attention fault word: %s", cudaGetErrorString(cudaGetLastError()));
        return NB200_ERR_LAUNCH;
    }
    *bits = v;
    return NB200_OK;
}

int launch_attention(const void* q, const void* k, const void* v, void* o, float* lse, int64_t B, int64_t H,
                     int64_t S, int64_t D, int causal, float scale, cudaStream_t st) {
    if (D != kDim) {
        set_error("nb200_attention: head_dim %lld is not supported (this kernel is built for %d)", (long long)D, kDim);
        return NB200_ERR_UNSUPPORTED;
    }
    if (!(scale > 0.f)) {
        set_error("nb200_attention: scale must be positive");
        return NB200_ERR_ARG;
    }
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) ||
        (lse && (reinterpret_cast<uintptr_t>(lse) & 3u))) {
        set_error("nb200_attention: q, k, v, o must be 16-byte aligned and lse 4-byte aligned");
        return NB200_ERR_ARG;
    }
    const int64_t BH = B * H;
    const int64_t nqb = (S + kQTiles * kRows - 1) / (kQTiles * kRows);
    if (S > (int64_t)1 << 30 || BH > (int64_t)1 << 30 || BH * nqb > 0x7fffffffLL) {
        set_error("nb200_attention: batch*heads=%lld, seq=%lld exceed the kernel's index range", (long long)BH,
                  (long long)S);
        return NB200_ERR_CAPACITY;
    }
    int rc = get_encoder();
    if (rc) return rc;
    CUtensorMap mq, mk, mv, mo;
    if ((rc = encode_map(&mq, q, BH, S, kRows, "q")) || (rc = encode_map(&mk, k, BH, S, kKeys, "k")) ||
        (rc = encode_map(&mv, v, BH, S, kKeys, "v")) || (rc = encode_map(&mo, o, BH, S, 32, "o")))
        return rc;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        set_error("nb200_attention: no usable current CUDA device");
        return NB200_ERR_LAUNCH;
    }
    {
        std::lock_guard<std::mutex> lock(g_attr_mutex);
        if (!g_attr_set[dev]) {
            if (cudaFuncSetAttribute(attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
                cudaSuccess) {
                set_error("nb200_attention: cannot reserve %u bytes of shared memory: %s", kSmemBytes,
                          cudaGetErrorString(cudaGetLastError()));
                return NB200_ERR_LAUNCH;
            }
            g_attr_set[dev] = true;
        }
    }
    AttnArgs a;
    a.S = (int)S;
    a.BH = (int)BH;
    a.nqb = (int)nqb;
    a.causal = causal ? 1 : 0;
    a.sl2 = scale * 1.4426950408889634f;
    a.lse = lse;
    attn_fwd_kernel<<<(unsigned)(BH * nqb), kThreads, kSmemBytes, st>>>(mq, mk, mv, mo, a);
    count_launch();
    return finish_launch("nb200_attention");
}

}  // namespace nb200
