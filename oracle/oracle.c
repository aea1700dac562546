/*
 * CPU ORACLE -- test infrastructure only. A plain-C restatement of the reference backend's
 * algorithms (Defyli/neptune-opt, package neptune_codegen), used by tests/ as the checker, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg. The product path never calls it.
 *
 * Parity pinning: tests/test_oracle_golden.py checks every function here against golden
 * vectors produced by the reference itself (tests/golden/make_golden.py runs the reference's own
 * generated kernels under Triton's CPU interpreter and its ATen graphs).
 *
 * Build: make -C oracle   (gcc -O2 -fopenmp -ffp-contract=off: no FMA contraction, no
 * reassociation; float arithmetic is IEEE binary32 with round-to-nearest-even). Sums are
 * accumulated in binary64 so the oracle sits closer to the exact value than any fp32 summation
 * order; storage-dtype rounding (segments, RMSNorm stages) is reproduced exactly.
 *
 * Functions and the reference code they restate:
 *   oracle_fold        serial repaired fold, template.py:41-54 + emitters.py:436-532
 *                      (chunk of `block` columns -> state; merge_state; finaliser)
 *   oracle_two_pass    two-pass variance/std, template.py:62-103
 *   oracle_split       split plan, template.py:137-165 (partials per chunk, then merge)
 *   oracle_softmax     log-family readout of the lowering, neptune_recognize/lowering.py:80-99
 *   oracle_l2_normalize stable_l2 fold (library.py:32-38) then x / norm
 *   oracle_rms_norm    RMSNorm numeric stages, emitters.py:576-595, skeleton.py:213-217
 *   oracle_rms_scale   the per-row fp32 scale of those stages (emitters.py:576-586)
 *   oracle_segment_spans  torch_op.py:370-387 (cumsum + the four assertions, as status bits)
 *   oracle_segment_pool   torch_op.py:286-306 (ordered storage-dtype fold)
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* Skeleton ids (the order of neptune_codegen/library.py's registrations as numbered by the
 * backend's C ABI). */
enum { SK_LOGSUMEXP, SK_LSE_BIASED, SK_LSE_SCALED, SK_SOFTCAP_LSE, SK_STABLE_L2, SK_LINEAR_ATTN,
       SK_DECAY_RENORM, SK_SUMSQ_DIV, SK_RMSNORM_MAX, SK_VARIANCE, SK_STD };
enum { DT_F32 = 0, DT_BF16 = 1, DT_F16 = 2 };

typedef struct { double tiny, alpha, T, beta, N, eps; } oparams;
typedef struct { float m, acc; int seen, status; } ostate;

/* ------------------------------------------------------------------ storage rounding */
/* Round-to-nearest-even of a binary32 value to bf16 / fp16, returned as binary32. Computed from
 * the definition (scale by the ulp, round to nearest even integer, scale back), all exact. */
static float round_dtype(float v, int dtype) {
    if (dtype == DT_F32 || isnan(v) || isinf(v) || v == 0.0f) return v;
    double d = v;
    int e;
    frexp(d, &e); /* d = m * 2^e, 0.5 <= |m| < 1 -> floor(log2|d|) = e - 1 */
    int p = dtype == DT_BF16 ? 8 : 11;             /* significand bits incl. the leading one */
    int emin = dtype == DT_BF16 ? -126 : -14;       /* smallest normal exponent */
    double maxv = dtype == DT_BF16 ? ldexp(2.0 - ldexp(1.0, -7), 127) : 65504.0;
    int ex = e - 1;
    if (ex < emin) ex = emin;                       /* subnormal: fixed quantum */
    double ulp = ldexp(1.0, ex - (p - 1));
    double r = nearbyint(d / ulp) * ulp;           /* default rounding mode: to nearest, even */
    if (fabs(r) > maxv) r = r > 0 ? INFINITY : -INFINITY;
    return (float)r;
}

float oracle_round(float v, int dtype) { return round_dtype(v, dtype); }

/* ------------------------------------------------------------------ skeleton algebra */
static int is_log(int sk) { return sk <= SK_SOFTCAP_LSE; }

static float phi(int sk, float v, const oparams* p) {
    switch (sk) {
        case SK_LSE_BIASED: return (float)p->alpha + v;
        case SK_LSE_SCALED: return v * (float)(1.0 / p->T);
        case SK_SOFTCAP_LSE: return tanhf((float)p->beta * v);
        default: return v;
    }
}

static int floors(int sk) { return sk == SK_STABLE_L2 || sk == SK_LINEAR_ATTN || sk == SK_SUMSQ_DIV; }

/* The `{sk}_chunk` helper (emitters.py:459-488) over n contiguous values. As a checker the oracle
 * evaluates every term and every sum in binary64 (the reference kernel sums fp32 terms in a tree;
 * a binary64 sum is closer to the exact value than any fp32 order), then stores the state in fp32. */
static ostate chunk_state(int sk, const float* v, int64_t n, int64_t ncols_total, const oparams* p) {
    ostate s = {-INFINITY, 0.0f, 0, 0};
    if (n <= 0) return s;
    if (is_log(sk)) {
        float m = -INFINITY;
        int st = 0, seen = 0;
        for (int64_t i = 0; i < n; ++i) {
            float ph = phi(sk, v[i], p);
            if (isnan(ph)) st |= 1;
            else if (ph == INFINITY) st |= 2;
            else if (ph != -INFINITY) { seen = 1; if (ph > m) m = ph; }
        }
        double den = seen ? m : 0.0, acc = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            float ph = phi(sk, v[i], p);
            if (isfinite(ph)) acc += exp((double)ph - den);
        }
        s.m = m; s.acc = (float)acc; s.seen = seen; s.status = st;
        return s;
    }
    if (sk == SK_RMSNORM_MAX) {
        double invn = 1.0 / (double)ncols_total, m = 0.0;
        for (int64_t i = 0; i < n; ++i) m += ((double)v[i] * v[i]) * invn;
        double r = 1.0 / sqrt(m + p->eps), acc = -INFINITY;
        for (int64_t i = 0; i < n; ++i) { double t = v[i] * r; if (t > acc) acc = t; }
        s.m = (float)m; s.acc = (float)acc; s.seen = 1;
        return s;
    }
    float m = 0.0f;
    for (int64_t i = 0; i < n; ++i) { float a = fabsf(v[i]); if (a > m) m = a; }
    double den = floors(sk) ? fmax(m, 1e-30) : m, acc = 0.0;
    for (int64_t i = 0; i < n; ++i) {
        double x = v[i];
        switch (sk) {
            case SK_STABLE_L2: acc += (x / den) * (x / den); break;
            case SK_LINEAR_ATTN: acc += x / den; break;
            case SK_DECAY_RENORM: acc += x / (den + p->N); break;
            case SK_SUMSQ_DIV: acc += x * x / den; break;
        }
    }
    s.m = m; s.acc = (float)acc; s.seen = 1;
    return s;
}

/* `{sk}_merge_state` (emitters.py:500-517): A is the left operand; repairs in binary64. */
static double factor_d(int sk, double q, double qn, const oparams* p) {
    switch (sk) {
        case SK_STABLE_L2: return (q / qn) * (q / qn);
        case SK_LINEAR_ATTN: case SK_SUMSQ_DIV: return q / qn;
        case SK_DECAY_RENORM: return (q + p->N) / (qn + p->N);
        case SK_RMSNORM_MAX: return sqrt(q + p->eps) / sqrt(qn + p->eps);
    }
    return 1.0;
}

static ostate merge_state(int sk, ostate A, ostate B, const oparams* p) {
    ostate r;
    r.status = A.status | B.status;
    if (!B.seen) { r.m = A.m; r.acc = A.acc; r.seen = A.seen; return r; }
    if (!A.seen) { r.m = B.m; r.acc = B.acc; r.seen = 1; return r; }
    r.seen = 1;
    if (is_log(sk)) {
        r.m = fmaxf(A.m, B.m);
        r.acc = (float)((double)A.acc * exp((double)A.m - r.m) + (double)B.acc * exp((double)B.m - r.m));
    } else if (sk == SK_RMSNORM_MAX) {
        double m = (double)A.m + (double)B.m;
        r.m = (float)m;
        r.acc = (float)fmax(A.acc * factor_d(sk, A.m, m, p), B.acc * factor_d(sk, B.m, m, p));
    } else {
        int f = floors(sk);
        r.m = fmaxf(A.m, B.m);
        double qa = f ? fmax(A.m, 1e-30) : A.m, qb = f ? fmax(B.m, 1e-30) : B.m;
        double qn = f ? fmax(r.m, 1e-30) : r.m;
        r.acc = (float)(A.acc * factor_d(sk, qa, qn, p) + B.acc * factor_d(sk, qb, qn, p));
    }
    return r;
}

/* Finaliser: state_finalize_source (emitters.py:522-532) and the skeletons' readouts. */
static float finalize(int sk, ostate s, const oparams* p) {
    if (is_log(sk)) {
        if (s.status & 1) return NAN;
        if (s.status & 2) return INFINITY;
        if (!s.seen) return -INFINITY;
        return (float)((double)s.m + log((double)s.acc + p->tiny));
    }
    if (sk == SK_STABLE_L2) return (float)(fmax(s.m, 1e-30) * sqrt((double)s.acc));
    return s.acc;
}

/* ------------------------------------------------------------------ a1 serial fold */
void oracle_two_pass(int sk, const float* x, int64_t rows, int64_t ncols, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* v = x + r * ncols;
        double m = 0.0, acc = 0.0;
        for (int64_t i = 0; i < ncols; ++i) m += v[i];
        m /= (double)ncols;
        for (int64_t i = 0; i < ncols; ++i) { double d = v[i] - m; acc += d * d; }
        acc /= (double)ncols;
        out[r] = (float)(sk == SK_STD ? sqrt(acc) : acc);
    }
}

/* x is a contiguous fp32 copy of the rows (the reference loads `.to(tl.float32)`); out[r] is the
 * fp32 result before the caller's narrowing to the input dtype. */
void oracle_fold(int sk, const oparams* p, const float* x, int64_t rows, int64_t ncols, int64_t block,
                 float* out) {
    if (sk == SK_VARIANCE || sk == SK_STD) { oracle_two_pass(sk, x, rows, ncols, out); return; }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* v = x + r * ncols;
        ostate s = {0.0f, 0.0f, 0, 0};
        for (int64_t off = 0; off < ncols; off += block) {
            int64_t n = ncols - off < block ? ncols - off : block;
            s = merge_state(sk, s, chunk_state(sk, v + off, n, ncols, p), p);
        }
        out[r] = finalize(sk, s, p);
    }
}

/* ------------------------------------------------------------------ a2 split plan */
/* Chunk states of columns [col_begin, col_begin + shard) in `block` chunks -> states[r*nparts+j]. */
void oracle_partial(int sk, const oparams* p, const float* x, int64_t rows, int64_t ncols,
                    int64_t col_begin, int64_t shard, int64_t block, ostate* states) {
    int64_t nparts = (shard + block - 1) / block;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < nparts; ++j) {
            int64_t lo = col_begin + j * block, hi = lo + block;
            if (hi > col_begin + shard) hi = col_begin + shard;
            states[r * nparts + j] = chunk_state(sk, x + r * ncols + lo, hi - lo, ncols, p);
        }
}

/* Left fold of each row's states in ascending part order, then the finaliser. */
void oracle_merge(int sk, const oparams* p, const ostate* states, int64_t rows, int64_t nparts, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        ostate s = {0.0f, 0.0f, 0, 0};
        for (int64_t j = 0; j < nparts; ++j) s = merge_state(sk, s, states[r * nparts + j], p);
        out[r] = finalize(sk, s, p);
    }
}

/* ------------------------------------------------------------------ readouts */
/* mode 0 softmax exp(x - m) / s, mode 1 log_softmax (x - m) - log(s); NaN rows for NaN, +inf or
 * no finite element. lse[r] receives the logsumexp (fp32). */
void oracle_softmax(int mode, const float* x, int64_t rows, int64_t ncols, float* y, float* lse) {
    oparams p = {0, 0, 1, 1, 1, 1};
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* v = x + r * ncols;
        ostate s = chunk_state(SK_LOGSUMEXP, v, ncols, ncols, &p);
        int bad = s.status != 0 || !s.seen;
        double acc = 0.0;  /* the row's sum again in binary64, unrounded */
        if (!bad)
            for (int64_t i = 0; i < ncols; ++i) acc += exp((double)v[i] - s.m);
        double lg = log(acc);
        for (int64_t i = 0; i < ncols; ++i)
            y[r * ncols + i] = bad ? NAN : (float)(mode == 0 ? exp((double)v[i] - s.m) / acc : ((double)v[i] - s.m) - lg);
        if (lse) lse[r] = finalize(SK_LOGSUMEXP, s, &p);
    }
}

void oracle_l2_normalize(const float* x, int64_t rows, int64_t ncols, int dtype, float* y, float* norm) {
    oparams p = {0, 0, 1, 1, 1, 1};
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* v = x + r * ncols;
        float n = finalize(SK_STABLE_L2, chunk_state(SK_STABLE_L2, v, ncols, ncols, &p), &p);
        for (int64_t i = 0; i < ncols; ++i) y[r * ncols + i] = round_dtype((float)((double)v[i] / n), dtype);
        if (norm) norm[r] = round_dtype(n, dtype);
    }
}

/* ------------------------------------------------------------------ a3 RMSNorm */
static float rsqrt_rn(float v) {
    /* 1/sqrt in 64-bit-significand extended precision, rounded once to binary32. */
    long double r = 1.0L / sqrtl((long double)v);
    return (float)r;
}

/* Per-row fp32 scale rsqrt_rn(div_rn(total, count) + eps) of the RMSNorm stages (emitters.py:576-586),
 * with the binary64-summed total rounded once to binary32. */
void oracle_rms_scale(const float* x, int64_t rows, int64_t ncols, double eps, float* scale) {
    const float count = (float)ncols, e = (float)eps;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* v = x + r * ncols;
        double total_d = 0.0;
        for (int64_t i = 0; i < ncols; ++i) total_d += (double)v[i] * v[i];
        float total = (float)total_d;
        scale[r] = rsqrt_rn(total / count + e);
    }
}

void oracle_rms_norm(const float* x, const float* gamma, int64_t rows, int64_t ncols, double eps,
                     int dtype, float* out) {
    const float count = (float)ncols, e = (float)eps;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        const float* v = x + r * ncols;
        double total_d = 0.0;
        for (int64_t i = 0; i < ncols; ++i) total_d += (double)v[i] * v[i];
        float total = (float)total_d;  /* the fp32 total (order-free: binary64 sum, rounded once) */
        float mean = total / count;
        float scale = rsqrt_rn(mean + e);
        for (int64_t i = 0; i < ncols; ++i) {
            float normalized = round_dtype(v[i] * scale, dtype);
            out[r * ncols + i] = round_dtype(normalized * gamma[i], dtype);
        }
    }
}

/* ------------------------------------------------------------------ a4/a5 segments */
/* Status bits: 1 length negative or > nrows, 2 lengths do not cover nrows (unless unsafe),
 * 4 boundary outside [0, nrows], 8 boundaries not monotonic. */
uint32_t oracle_segment_spans(const int64_t* seg, int64_t nseg, int is_offsets, int unsafe, int64_t nrows,
                              int64_t* spans) {
    uint32_t st = 0;
    if (is_offsets) {
        for (int64_t i = 0; i <= nseg; ++i) spans[i] = seg[i];
    } else {
        int64_t run = 0;
        spans[0] = 0;
        for (int64_t i = 0; i < nseg; ++i) {
            if (seg[i] < 0 || seg[i] > nrows) st |= 1;
            run += seg[i];
            spans[i + 1] = run;
        }
        if (!unsafe && run != nrows) st |= 2;
    }
    for (int64_t i = 0; i <= nseg; ++i) {
        if (spans[i] < 0 || spans[i] > nrows) st |= 4;
        if (i > 0 && spans[i] < spans[i - 1]) st |= 8;
    }
    return st;
}

/* data: fp32 values of the storage-dtype elements, contiguous [nrows, channels]. out: fp32
 * values exactly representable in the storage dtype. */
void oracle_segment_pool(const float* data, int64_t nrows, int64_t channels, const int64_t* spans,
                         int64_t nseg, int reduce, int has_initial, float initial, int dtype, float* out) {
    const float init = has_initial ? round_dtype(initial, dtype) : 0.0f;
#pragma omp parallel for schedule(static)
    for (int64_t s = 0; s < nseg; ++s) {
        int64_t start = spans[s], end = spans[s + 1];
        int valid = start >= 0 && end >= start && end <= nrows;
        for (int64_t c = 0; c < channels; ++c) {
            float acc = init;
            if (valid)
                for (int64_t t = start; t < end; ++t) acc = round_dtype(acc + data[t * channels + c], dtype);
            float res = acc;
            if (reduce == 1) {
                float den = round_dtype((float)(end - start), dtype);
                res = acc / den;
                if (end == start) res = has_initial ? acc : NAN;
            }
            if (!valid) res = NAN;
            out[s * channels + c] = round_dtype(res, dtype);
        }
    }
}

/* In-place storage rounding of an fp32 array (helper for the Python wrapper). */
void oracle_round_array(float* x, int64_t n, int dtype) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) x[i] = round_dtype(x[i], dtype);
}

/* Threads the oracle's parallel loops use (1 when built without OpenMP). */
#ifdef _OPENMP
#include <omp.h>
int oracle_num_threads(void) { return omp_get_max_threads(); }
#else
int oracle_num_threads(void) { return 1; }
#endif
