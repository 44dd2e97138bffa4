/*
 * k1_oracle.c -- TEST INFRASTRUCTURE ONLY.  CPU restatement, in fp64, of the
 * reference's K1 primitive (per-row log-prob / entropy / log-sum-exp, forward and
 * backward).  It is the checker the GPU kernels are compared against; nothing in the
 * product path links or calls it.
 *
 * Parity pins: the fp64 definitions follow the reference tests' ground truth
 * (tests/test_logprob.py:17-25 forward, :160-167 and :184-189 backward) and the
 * reference kernels' edge rules, cited per function.  The restatement is checked in
 * the CPU tests against golden vectors produced by the reference's own test oracle
 * restated in torch fp64 (tests/golden/make_golden.py) and, on the GPU box, against
 * the reference CUDA kernels rebuilt for sm_100a (oracle/build_ref.py).
 *
 * Two-pass exact evaluation per row (max, then sums in fp64) -- deliberately not the
 * streaming formulation, so the checker does not share the kernels' algorithm.
 *
 * Layout: element (r, v) at (r / inner_rows) * outer_stride + (r % inner_rows) *
 * inner_stride + v, the same two-level row layout as include/k1_logprob.h.
 * dtype: 0 = fp32, 1 = fp16, 2 = bf16 (raw bit patterns).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static double f16_to_double(uint16_t h) {
    int sign = (h >> 15) & 1;
    int exp = (h >> 10) & 0x1f;
    int man = h & 0x3ff;
    double v;
    if (exp == 0) {
        v = ldexp((double)man, -24); /* subnormal: man * 2^-14 * 2^-10 */
    } else if (exp == 31) {
        v = man ? NAN : INFINITY;
    } else {
        v = ldexp((double)(man | 0x400), exp - 25);
    }
    return sign ? -v : v;
}

static double bf16_to_double(uint16_t b) {
    uint32_t u = ((uint32_t)b) << 16;
    float f;
    memcpy(&f, &u, sizeof f);
    return (double)f;
}

static inline double load_elem(const void* base, int dtype, int64_t idx) {
    if (dtype == 0) return (double)((const float*)base)[idx];
    if (dtype == 1) return f16_to_double(((const uint16_t*)base)[idx]);
    return bf16_to_double(((const uint16_t*)base)[idx]);
}

static inline int64_t row_offset(int64_t r, int64_t inner_rows, int64_t inner_stride,
                                 int64_t outer_stride) {
    return (r / inner_rows) * outer_stride + (r % inner_rows) * inner_stride;
}

/*
 * Row statistics relative to the row maximum m:
 *   z = sum exp(x - m), t = sum exp(x - m) (x - m), -inf entries skipped
 * (the reference v1 kernel skips them through its -inf sentinel,
 * csrc/fused_logprob.cu:141-143).  Any NaN makes the row NaN (fmaxf + __expf in the
 * reference propagate it into Z).  A +inf entry makes x - m = inf - inf = NaN, as in
 * the reference.  Returns 1 when every entry is -inf.
 */
static int row_stats(const void* logits, int dtype, int64_t off, int64_t vocab, double* m_out,
                     double* z_out, double* t_out, double* logz_out) {
    double m = -INFINITY;
    int has_nan = 0;
    for (int64_t v = 0; v < vocab; ++v) {
        double x = load_elem(logits, dtype, off + v);
        if (isnan(x)) has_nan = 1;
        else if (x > m) m = x;
    }
    if (has_nan || m == INFINITY) {
        *m_out = NAN; *z_out = NAN; *t_out = NAN; *logz_out = NAN;
        return 0;
    }
    if (m == -INFINITY) {
        *m_out = -INFINITY; *z_out = 0.0; *t_out = 0.0; *logz_out = -INFINITY;
        return 1;
    }
    /* z = cnt + zrest: the entries equal to the maximum contribute exactly 1 each and are
     * counted apart from the tail, so log z = log cnt + log1p(zrest / cnt) keeps the
     * tail's relative precision even when one logit dominates the row. */
    double zrest = 0.0, t = 0.0, cnt = 0.0;
    for (int64_t v = 0; v < vocab; ++v) {
        double x = load_elem(logits, dtype, off + v);
        if (x == -INFINITY) continue;
        if (x == m) { cnt += 1.0; continue; }
        double d = x - m;
        double e = exp(d);
        zrest += e;
        t += e * d;
    }
    *m_out = m; *z_out = cnt + zrest; *t_out = t;
    *logz_out = log(cnt) + log1p(zrest / cnt);
    return 0;
}

/*
 * Forward.  lse = m + log z, H = log z - t / z, logprob = x_t - lse with x_t = 0 for
 * a target outside [0, vocab) (reference v1 initialises its shared target logit to
 * 0.0f and only a matching column overwrites it, csrc/fused_logprob.cu:179-185,
 * 220-225).  All -inf row: lse = -inf, H = NaN, logprob = x_t - lse (NaN for an
 * in-range target, +inf otherwise), the values the reference's sentinel state
 * (m = -inf, Z = 0, T = 0) produces at csrc/fused_logprob.cu:221-224.
 */
int k1o_forward(const void* logits, int dtype, int64_t n_rows, int64_t vocab,
                int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                const int64_t* targets, double* logp, double* ent, double* lse,
                int n_threads) {
    if (vocab < 1 || inner_rows < 1 || (n_rows % inner_rows) != 0) return 1;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
    for (int64_t r = 0; r < n_rows; ++r) {
        int64_t off = row_offset(r, inner_rows, inner_stride, outer_stride);
        double m, z, t, logz;
        int all_neg_inf = row_stats(logits, dtype, off, vocab, &m, &z, &t, &logz);
        int64_t tg = targets[r];
        double xt = (tg >= 0 && tg < vocab) ? load_elem(logits, dtype, off + tg) : 0.0;
        if (all_neg_inf) {
            lse[r] = -INFINITY;
            ent[r] = NAN;
            logp[r] = xt - lse[r];
            continue;
        }
        lse[r] = m + logz;
        ent[r] = logz - t / z;
        logp[r] = xt - lse[r];
    }
    return 0;
}

/*
 * Backward (reference csrc/fused_logprob.cu:233-241, 271-281):
 *   d[v] = p_v (g_lse - g_logp - g_ent (log p_v + H)) + [v == t] g_logp,
 *   p_v = exp(x_v - lse), log p_v = x_v - lse.
 * lse / ent are the forward values to use (the exact fp64 ones for ground truth).
 * g_* may be NULL (zero).  For an x_v = -inf entry p_v = 0 and p_v log p_v -> 0, so
 * the entry's gradient is its one-hot term only (the limit; the reference kernel
 * evaluates 0 * inf there and returns NaN).
 * d_logits: n_rows x vocab, contiguous.
 */
int k1o_backward(const void* logits, int dtype, int64_t n_rows, int64_t vocab,
                 int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                 const int64_t* targets, const double* lse, const double* ent,
                 const double* g_logp, const double* g_ent, const double* g_lse,
                 double* d_logits, int n_threads) {
    if (vocab < 1 || inner_rows < 1 || (n_rows % inner_rows) != 0) return 1;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
    for (int64_t r = 0; r < n_rows; ++r) {
        int64_t off = row_offset(r, inner_rows, inner_stride, outer_stride);
        double gl = g_logp ? g_logp[r] : 0.0;
        double ge = g_ent ? g_ent[r] : 0.0;
        double gs = g_lse ? g_lse[r] : 0.0;
        double c0 = gs - gl - ge * ent[r];
        int64_t tg = targets[r];
        double* out = d_logits + r * vocab;
        for (int64_t v = 0; v < vocab; ++v) {
            double x = load_elem(logits, dtype, off + v);
            double dv;
            int finite_row = !isnan(lse[r]) && lse[r] != -INFINITY;
            if (x == -INFINITY && finite_row) {
                dv = (v == tg) ? gl : 0.0;
            } else if (v == tg && finite_row) {
                /* same value, without the cancellation of g_logp - p g_logp for p -> 1:
                 * g_logp (1 - p) + p (g_lse - g_ent (log p + H)), 1 - p = -expm1(log p) */
                double lp = x - lse[r];
                double p = exp(lp);
                dv = gl * (-expm1(lp)) + p * (gs - ge * (lp + ent[r]));
            } else {
                double lp = x - lse[r];
                double p = exp(lp);
                dv = p * (c0 - ge * lp);
                if (v == tg) dv += gl;
            }
            out[v] = dv;
        }
    }
    return 0;
}

/*
 * Vocab-parallel restatement: per-row partial (m, z, t, x_t, has_target) of the shard
 * holding global columns [vocab_offset, vocab_offset + shard_vocab).  The logits
 * pointer addresses the shard's first column.
 */
int k1o_shard_partials(const void* logits, int dtype, int64_t n_rows, int64_t shard_vocab,
                       int64_t inner_rows, int64_t inner_stride, int64_t outer_stride,
                       int64_t vocab_offset, const int64_t* targets, double* m_out,
                       double* z_out, double* t_out, double* xt_out, int32_t* has_out,
                       int n_threads) {
    if (shard_vocab < 1 || inner_rows < 1 || (n_rows % inner_rows) != 0) return 1;
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 4)
#endif
    for (int64_t r = 0; r < n_rows; ++r) {
        int64_t off = row_offset(r, inner_rows, inner_stride, outer_stride);
        double logz;
        row_stats(logits, dtype, off, shard_vocab, &m_out[r], &z_out[r], &t_out[r], &logz);
        int64_t tl = targets[r] - vocab_offset;
        int has = (targets[r] >= 0 && tl >= 0 && tl < shard_vocab);
        has_out[r] = has;
        xt_out[r] = has ? load_elem(logits, dtype, off + tl) : 0.0;
    }
    return 0;
}

/*
 * Merge of shard partials (the reference's (m, Z, T) combine, csrc/fused_logprob.cu:
 * 119-154, evaluated in fp64 after all shards are known):
 *   M = max m_k,  Z = sum z_k e^{m_k - M},  T = sum e^{m_k - M} (t_k + (m_k - M) z_k).
 * Inputs are shard-major arrays of n_shards * n_rows.
 */
int k1o_combine(const double* m, const double* z, const double* t, const double* xt,
                const int32_t* has, int n_shards, int64_t n_rows, double* logp, double* ent,
                double* lse) {
    for (int64_t r = 0; r < n_rows; ++r) {
        double M = -INFINITY;
        int nan = 0;
        for (int k = 0; k < n_shards; ++k) {
            double mk = m[(int64_t)k * n_rows + r];
            if (isnan(mk)) nan = 1;
            else if (mk > M) M = mk;
        }
        double x_t = 0.0;
        for (int k = 0; k < n_shards; ++k)
            if (has[(int64_t)k * n_rows + r]) x_t = xt[(int64_t)k * n_rows + r];
        if (nan) {
            lse[r] = NAN; ent[r] = NAN; logp[r] = NAN;
            continue;
        }
        if (M == -INFINITY) {
            lse[r] = -INFINITY; ent[r] = NAN; logp[r] = x_t - lse[r];
            continue;
        }
        double Z = 0.0, T = 0.0;
        for (int k = 0; k < n_shards; ++k) {
            int64_t i = (int64_t)k * n_rows + r;
            if (m[i] == -INFINITY) continue;
            double dm = m[i] - M;
            double s = exp(dm);
            Z += s * z[i];
            T += s * (t[i] + dm * z[i]);
        }
        double logz = log(Z);
        lse[r] = M + logz;
        ent[r] = logz - T / Z;
        logp[r] = x_t - lse[r];
    }
    return 0;
}
