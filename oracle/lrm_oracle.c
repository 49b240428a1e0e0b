/*
 * lrm_oracle.c -- CPU restatement of the reference's CPU reference (Lrm.Tensor.CpuReference), the parity oracle.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker that the CUDA path is compared against. Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg (and its `--impl reference` arm) load it. The product
 * library (rosylnalive_b200/csrc) never links, includes or calls anything here.
 *
 * Parity is pinned: tests/test_oracle_golden.py checks this file against the reference's committed tiny-model goldens
 * (goldens/tiny/g1: torch32/torch64p taps, 64-step greedy ids, T_spec), the RoPE table digests and the known-answer
 * vectors of the reference's CpuReferenceSemantics contract.
 *
 * Every op exists twice from one macro body, in float (CpuRef F32) and double (CpuRef F64) -- the reference's
 * generic 'T over float32/float. The arithmetic rules it follows (src/Lrm.Tensor.CpuReference/Rows.fs:8-12):
 *   - reductions are sequential in increasing index order from +0;
 *   - products inside a reduction are fused: acc = fma(x, y, acc), one rounding per step;
 *   - element-wise formulas round after every operation in the order written (compiled with -ffp-contract=off);
 *   - exp/log/sqrt come from libm (the reference uses the .NET runtime; bit equality with it is not claimed);
 *   - threads split only independent outputs (rows, (row, head) pairs, 64-column blocks), so the bits do not
 *     depend on the thread count (src/Lrm.Tensor.CpuReference/CpuExec.fs:6-12).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <quadmath.h>

/* ------------------------------------------------------------------------------------------------------------ */
/* Parallel-for over independent outputs (CpuExec.fs:35-49, Par.forEach).                                        */

typedef void (*body_fn)(void *ctx, long lo, long hi);

typedef struct {
    body_fn fn;
    void *ctx;
    long lo, hi;
} par_slice;

static void *par_thread(void *p) {
    par_slice *s = (par_slice *)p;
    s->fn(s->ctx, s->lo, s->hi);
    return NULL;
}

/* Runs fn over [0, count) split into `threads` contiguous slices. Every output index is computed exactly once, by
 * one thread, in the fixed per-element order, so results are the same for every thread count. */
static void par_for(int threads, long count, body_fn fn, void *ctx) {
    if (threads <= 1 || count <= 1) {
        fn(ctx, 0, count);
        return;
    }
    if (threads > 256) threads = 256;
    if (threads > count) threads = (int)count;
    pthread_t tid[256];
    par_slice sl[256];
    long per = (count + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        long lo = t * per, hi = lo + per;
        if (lo >= count) break;
        if (hi > count) hi = count;
        sl[t].fn = fn;
        sl[t].ctx = ctx;
        sl[t].lo = lo;
        sl[t].hi = hi;
        if (pthread_create(&tid[t], NULL, par_thread, &sl[t]) != 0) {
            fn(ctx, lo, hi); /* fall back to the calling thread for this slice */
            sl[t].fn = NULL;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (sl[t].fn) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------------------------------------------------ */
/* bf16 (Lrm.Core Numerics.fs:24-45).                                                                            */

static inline float bf16_widen(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t oracle_bf16_narrow_rne(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (u & 0x80000000u) ? 0xFFC0u : 0x7FC0u;
    return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

void oracle_bf16_narrow_array(const float *x, uint16_t *y, long n) {
    for (long i = 0; i < n; ++i) y[i] = oracle_bf16_narrow_rne(x[i]);
}

/* ------------------------------------------------------------------------------------------------------------ */
/* T_spec, the RoPE table (Rope.fs:17-251). freq = f32(f32(pos) * inv_freq[j]); cos/sin = f32(RN64(cos/sin freq)).
 * The reference computes the correctly rounded float64 in exact integer arithmetic. Here the value is computed in
 * binary128 (libquadmath, 113-bit significand) and the float64 rounding is accepted only when the binary128 result
 * lies more than 2^-100 (relative) away from a float64 rounding boundary; otherwise the function reports failure
 * (the caller raises) rather than guess. Pinned by the table digests in the tests. */

/* RN64 of q with a certainty check; returns 0 on an uncertain rounding. */
static int certain_rn64(__float128 q, double *out) {
    double d = (double)q; /* round to nearest even */
    if (q == 0) {
        *out = d;
        return 1;
    }
    /* distance to the nearest rounding boundary: boundaries are midpoints between d and its neighbours */
    double up = nextafter(d, INFINITY), dn = nextafter(d, -INFINITY);
    __float128 mid_up = ((__float128)d + (__float128)up) / 2;
    __float128 mid_dn = ((__float128)d + (__float128)dn) / 2;
    __float128 aq = q < 0 ? -q : q;
    __float128 tol = aq * 0x1p-100Q;
    __float128 e1 = mid_up - q, e2 = q - mid_dn;
    if (e1 < 0) e1 = -e1;
    if (e2 < 0) e2 = -e2;
    if (e1 <= tol || e2 <= tol) return 0;
    *out = d;
    return 1;
}

/* Returns 0 on success, -1 when an entry's rounding could not be certified. */
int oracle_rope_table(const uint32_t *inv_freq_bits, int half, int max_pos, float *cos_out, float *sin_out) {
    for (int pos = 0; pos < max_pos; ++pos) {
        for (int j = 0; j < half; ++j) {
            float inv;
            memcpy(&inv, &inv_freq_bits[j], 4);
            float freq = (float)pos * inv; /* one float32 multiply of the exact position */
            double c, s;
            if (fabsf(freq) < 0x1p-27f) {
                c = 1.0;
                s = (double)freq;
            } else {
                __float128 fq = (__float128)freq;
                if (!certain_rn64(cosq(fq), &c) || !certain_rn64(sinq(fq), &s)) return -1;
            }
            cos_out[(long)pos * half + j] = (float)c;
            sin_out[(long)pos * half + j] = (float)s;
        }
    }
    return 0;
}

/* Correctly rounded float64 cos/sin of a float32 (ExactTrig.cosSin, Rope.fs:144-161); 0 ok, -1 uncertain. */
int oracle_cos_sin(float x, double *c, double *s) {
    if (!isfinite(x)) {
        *c = NAN;
        *s = NAN;
        return 0;
    }
    if (fabsf(x) < 0x1p-27f) {
        *c = 1.0;
        *s = (double)x;
        return 0;
    }
    __float128 fq = (__float128)x;
    if (!certain_rn64(cosq(fq), c) || !certain_rn64(sinq(fq), s)) return -1;
    return 0;
}

/* ------------------------------------------------------------------------------------------------------------ */
/* The ops, one body per precision. T is float or double; FMA is fmaf or fma; EXP is expf or exp.               */

#define DEFINE_OPS(SUF, T, FMA, EXP, SQRT)                                                                           \
                                                                                                                     \
    /* Rows.dot (Rows.fs:28-35): acc = fma(x[i], y[i], acc) from +0. */                                              \
    T oracle_dot_##SUF(const T *x, const T *y, long n) {                                                             \
        T acc = 0;                                                                                                   \
        for (long i = 0; i < n; ++i) acc = FMA(x[i], y[i], acc);                                                     \
        return acc;                                                                                                  \
    }                                                                                                                \
                                                                                                                     \
    /* CpuRef.embedGather (CpuRef.fs:74-147): widen(table[id]); id >= vocab gives the quiet-NaN row 0x7FC00000. */   \
    void oracle_embed_gather_##SUF(const uint16_t *table, long vocab, long cols, const uint32_t *ids, long rows,     \
                                   T *y) {                                                                           \
        float qnan;                                                                                                  \
        uint32_t qb = 0x7FC00000u;                                                                                   \
        memcpy(&qnan, &qb, 4);                                                                                       \
        for (long r = 0; r < rows; ++r) {                                                                            \
            T *dst = y + r * cols;                                                                                   \
            if ((long)ids[r] < vocab) {                                                                              \
                const uint16_t *src = table + (long)ids[r] * cols;                                                   \
                for (long c = 0; c < cols; ++c) dst[c] = (T)bf16_widen(src[c]);                                      \
            } else {                                                                                                 \
                for (long c = 0; c < cols; ++c) dst[c] = (T)qnan;                                                    \
            }                                                                                                        \
        }                                                                                                            \
    }                                                                                                                \
                                                                                                                     \
    /* Rows.rmsNorm (Rows.fs:50-71): ss = sum fma(x,x); mean = ss/n; r = 1/sqrt(mean+eps); y = widen(w)*(x*r). */    \
    static void rms_row_##SUF(const T *x, const uint16_t *w, long n, T eps, T *y) {                                  \
        T ss = 0;                                                                                                    \
        for (long i = 0; i < n; ++i) ss = FMA(x[i], x[i], ss);                                                       \
        T mean = ss / (T)n;                                                                                          \
        T r = (T)1 / SQRT(mean + eps);                                                                               \
        for (long i = 0; i < n; ++i) {                                                                               \
            T xr = x[i] * r;                                                                                         \
            y[i] = (T)bf16_widen(w[i]) * xr;                                                                         \
        }                                                                                                            \
    }                                                                                                                \
    typedef struct {                                                                                                 \
        const T *x;                                                                                                  \
        const uint16_t *w;                                                                                           \
        long n;                                                                                                      \
        T eps;                                                                                                       \
        T *y;                                                                                                        \
    } rms_ctx_##SUF;                                                                                                 \
    static void rms_body_##SUF(void *p, long lo, long hi) {                                                          \
        rms_ctx_##SUF *c = (rms_ctx_##SUF *)p;                                                                       \
        for (long r = lo; r < hi; ++r) rms_row_##SUF(c->x + r * c->n, c->w, c->n, c->eps, c->y + r * c->n);         \
    }                                                                                                                \
    /* CpuRef.rmsNorm (CpuRef.fs:150-180): rows of w.Length elements. */                                             \
    void oracle_rmsnorm_##SUF(const T *x, long rows, long cols, const uint16_t *w, T eps, T *y, int threads) {       \
        rms_ctx_##SUF c = {x, w, cols, eps, y};                                                                      \
        par_for(threads, rows, rms_body_##SUF, &c);                                                                  \
    }                                                                                                                \
                                                                                                                     \
    /* CpuRef.matmulBf16W (CpuRef.fs:186-221) via Rows.dotBf16 (Rows.fs:38-46): y[i,j] = sum_p fma(x[i,p],          \
     * widen(w[j,p]), .) sequential in p; tasks are (row, 64-column block) as in the reference. */                   \
    typedef struct {                                                                                                 \
        const T *x;                                                                                                  \
        const uint16_t *w;                                                                                           \
        long m, n, k, blocks;                                                                                        \
        T *y;                                                                                                        \
    } mm_ctx_##SUF;                                                                                                  \
    static void mm_body_##SUF(void *p, long lo, long hi) {                                                           \
        mm_ctx_##SUF *c = (mm_ctx_##SUF *)p;                                                                         \
        for (long t = lo; t < hi; ++t) {                                                                             \
            long i = t / c->blocks, j0 = (t % c->blocks) * 64, j1 = j0 + 64;                                         \
            if (j1 > c->n) j1 = c->n;                                                                                \
            const T *xi = c->x + i * c->k;                                                                           \
            for (long j = j0; j < j1; ++j) {                                                                         \
                const uint16_t *wj = c->w + j * c->k;                                                                \
                T acc = 0;                                                                                           \
                for (long q = 0; q < c->k; ++q) acc = FMA(xi[q], (T)bf16_widen(wj[q]), acc);                         \
                c->y[i * c->n + j] = acc;                                                                            \
            }                                                                                                        \
        }                                                                                                            \
    }                                                                                                                \
    void oracle_matmul_bf16w_##SUF(const T *x, long m, long k, const uint16_t *w, long n, T *y, int threads) {       \
        long blocks = (n + 63) / 64;                                                                                 \
        mm_ctx_##SUF c = {x, w, m, n, k, blocks, y};                                                                 \
        par_for(threads, m * blocks, mm_body_##SUF, &c);                                                             \
    }                                                                                                                \
                                                                                                                     \
    /* CpuRef.ropeApply (CpuRef.fs:225-271) via Rows.ropeHead (Rows.fs:205-227): row t has position pos0 + t;        \
     * y[i] = x[i]*c - x[i+h]*s; y[i+h] = x[i+h]*c + x[i]*s, every product rounded. cos/sin are T_spec rows. */      \
    void oracle_rope_apply_##SUF(const T *x, long rows, long heads, long hd, const float *cos_t, const float *sin_t,  \
                                 long pos0, T *y) {                                                                  \
        long half = hd / 2, cols = heads * hd;                                                                       \
        for (long t = 0; t < rows; ++t) {                                                                            \
            const float *cr = cos_t + (pos0 + t) * half, *sr = sin_t + (pos0 + t) * half;                           \
            for (long h = 0; h < heads; ++h) {                                                                       \
                const T *xh = x + t * cols + h * hd;                                                                 \
                T *yh = y + t * cols + h * hd;                                                                       \
                for (long i = 0; i < half; ++i) {                                                                    \
                    T c = (T)cr[i], s = (T)sr[i];                                                                    \
                    T a = xh[i], b = xh[i + half];                                                                   \
                    T ac = a * c, bs = b * s, bc = b * c, as = a * s;                                                \
                    yh[i] = ac - bs;                                                                                 \
                    yh[i + half] = bc + as;                                                                          \
                }                                                                                                    \
            }                                                                                                        \
        }                                                                                                            \
    }                                                                                                                \
                                                                                                                     \
    /* Rows.attention (Rows.fs:232-270) per (query row, head), CpuRef.attention (CpuRef.fs:274-332): s_j =           \
     * dot(q, k_j) * scale; softmax (max by '>', sequential plain-add sum, divide); y[d] = sum_j fma(p_j, v_j[d]).   \
     * Caches are [Tk, kv_heads*hd] (contiguous, row p = position p). */                                             \
    typedef struct {                                                                                                 \
        const T *q, *k, *v;                                                                                          \
        long rows, qh, kvh, hd, past;                                                                                \
        T scale;                                                                                                     \
        T *y;                                                                                                        \
    } att_ctx_##SUF;                                                                                                 \
    static void att_body_##SUF(void *p, long lo, long hi) {                                                          \
        att_ctx_##SUF *c = (att_ctx_##SUF *)p;                                                                       \
        long hd = c->hd, qcols = c->qh * hd, kvcols = c->kvh * hd, group = c->qh / c->kvh;                           \
        long maxkeys = c->past + c->rows;                                                                            \
        T *sc = (T *)malloc(sizeof(T) * (size_t)(maxkeys > 0 ? maxkeys : 1));                                        \
        for (long t = lo; t < hi; ++t) {                                                                             \
            long i = t / c->qh, h = t % c->qh, keys = c->past + i + 1, off = (h / group) * hd;                       \
            const T *qv = c->q + i * qcols + h * hd;                                                                 \
            for (long j = 0; j < keys; ++j) {                                                                        \
                const T *kj = c->k + j * kvcols + off;                                                               \
                T acc = 0;                                                                                           \
                for (long d = 0; d < hd; ++d) acc = FMA(qv[d], kj[d], acc);                                          \
                sc[j] = acc * c->scale;                                                                              \
            }                                                                                                        \
            T m = sc[0];                                                                                             \
            for (long j = 1; j < keys; ++j)                                                                          \
                if (sc[j] > m) m = sc[j];                                                                            \
            T l = 0;                                                                                                 \
            for (long j = 0; j < keys; ++j) {                                                                        \
                T e = EXP(sc[j] - m);                                                                                \
                sc[j] = e;                                                                                           \
                l = l + e;                                                                                           \
            }                                                                                                        \
            for (long j = 0; j < keys; ++j) sc[j] = sc[j] / l;                                                       \
            T *yv = c->y + i * qcols + h * hd;                                                                       \
            for (long d = 0; d < hd; ++d) yv[d] = 0;                                                                 \
            for (long j = 0; j < keys; ++j) {                                                                        \
                const T *vj = c->v + j * kvcols + off;                                                               \
                T pj = sc[j];                                                                                        \
                for (long d = 0; d < hd; ++d) yv[d] = FMA(pj, vj[d], yv[d]);                                         \
            }                                                                                                        \
        }                                                                                                            \
        free(sc);                                                                                                    \
    }                                                                                                                \
    void oracle_attention_##SUF(const T *q, long rows, const T *kcache, const T *vcache, long qh, long kvh, long hd,  \
                                long past, T scale, T *y, int threads) {                                             \
        att_ctx_##SUF c = {q, kcache, vcache, rows, qh, kvh, hd, past, scale, y};                                    \
        par_for(threads, rows * qh, att_body_##SUF, &c);                                                             \
    }                                                                                                                \
                                                                                                                     \
    /* Rows.siluMul (Rows.fs:185-192): s = g / (1 + exp(-g)); y = s * u. */                                          \
    void oracle_silu_mul_##SUF(const T *g, const T *u, long n, T *y) {                                               \
        for (long i = 0; i < n; ++i) {                                                                               \
            T gi = g[i];                                                                                             \
            T den = (T)1 + EXP(-gi);                                                                                 \
            T s = gi / den;                                                                                          \
            y[i] = s * u[i];                                                                                         \
        }                                                                                                            \
    }                                                                                                                \
                                                                                                                     \
    /* Rows.add (Rows.fs:195-201). */                                                                                \
    void oracle_add_##SUF(const T *a, const T *b, long n, T *y) {                                                    \
        for (long i = 0; i < n; ++i) y[i] = a[i] + b[i];                                                             \
    }                                                                                                                \
                                                                                                                     \
    /* CpuRef.argmaxRows (CpuRef.fs:453-467) via Rows.tryArgmax (Rows.fs:138-154): lowest index of the maximum by    \
     * strict '>', 0xFFFFFFFF for a row that holds a NaN. */                                                         \
    void oracle_argmax_rows_##SUF(const T *x, long rows, long cols, uint32_t *y) {                                   \
        for (long r = 0; r < rows; ++r) {                                                                            \
            const T *row = x + r * cols;                                                                             \
            long best = 0;                                                                                           \
            int nan = isnan(row[0]);                                                                                 \
            for (long i = 1; !nan && i < cols; ++i) {                                                                \
                if (isnan(row[i]))                                                                                   \
                    nan = 1;                                                                                         \
                else if (row[i] > row[best])                                                                         \
                    best = i;                                                                                        \
            }                                                                                                        \
            y[r] = nan ? 0xFFFFFFFFu : (uint32_t)best;                                                               \
        }                                                                                                            \
    }                                                                                                                \
                                                                                                                     \
    /* Rows.logSumExp (Rows.fs:115-135) and Rows.softmax (Rows.fs:84-111), used by the comparators. */               \
    T oracle_logsumexp_##SUF(const T *x, long n) {                                                                   \
        T m = x[0];                                                                                                  \
        for (long i = 1; i < n; ++i)                                                                                 \
            if (x[i] > m) m = x[i];                                                                                  \
        if (isinf(m)) {                                                                                              \
            T r = m;                                                                                                 \
            for (long i = 0; i < n; ++i)                                                                             \
                if (isnan(x[i])) r = (T)NAN;                                                                         \
            return r;                                                                                                \
        }                                                                                                            \
        T l = 0;                                                                                                     \
        for (long i = 0; i < n; ++i) l = l + EXP(x[i] - m);                                                          \
        return m + (T)log((double)l);                                                                                \
    }

DEFINE_OPS(f32, float, fmaf, expf, sqrtf)
DEFINE_OPS(f64, double, fma, exp, sqrt)

/* Widening helpers for the F64 mode: float32 values widen exactly. */
void oracle_f32_to_f64(const float *x, double *y, long n) {
    for (long i = 0; i < n; ++i) y[i] = (double)x[i];
}

/* CpuRef.attentionScale (CpuRef.fs:56-60): head_dim ** -0.5 in float64, rounded once. */
double oracle_attention_scale_f64(long hd) { return pow((double)hd, -0.5); }
float oracle_attention_scale_f32(long hd) { return (float)pow((double)hd, -0.5); }
