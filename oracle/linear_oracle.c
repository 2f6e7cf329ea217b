/* linear_oracle.c -- CPU restatement of the reference's FP16 Linear / HardSigmoid arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker: only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference arm load it. The product library never links it
 * and never falls back to it.
 *
 * What it restates (paths relative to the reference project root, CO = research/custom-ops):
 *   CO/tools/python/cli_gate.py:38-49   oracle(): per-256-K-tile math.fsum partial, running sum
 *                                        dot = f16(dot + partial), affine = f16(f16(dot) + b),
 *                                        y = f16(min(1, max(0, affine/6 + 0.5))).
 *   CO/tools/python/ktiling_gate.py:83-118  reference(): the same fold with a sequential double
 *                                        tile sum, plus the FP64 reference (raw64/act64) and the
 *                                        "perf-unfused" variant that narrows each tile sum first.
 *   CO/tools/c/ktiling_probe.c:108-128  reference_variant(): the C form of the above.
 *   CO/src/linear_hardsigmoid.c:51-82   emit_tiled(): bias only when present, HardSigmoid only for
 *                                        CO_LINEAR_HSIG, last K tile writes y directly otherwise.
 *
 * Modes (ORACLE_*):
 *   TILE16_EXACT  tile sums exactly rounded once to double (what math.fsum returns), computed
 *                 with a 128-bit fixed-point accumulator: every FP16 value is an integer multiple
 *                 of 2^-24, so a product is an integer multiple of 2^-48 below 2^80 and a sum of
 *                 up to 2^20 products fits in 101 bits.  Bit-identical to cli_gate.oracle.
 *   TILE16_SEQ    tile sums accumulated left to right in double (ktiling_gate.reference).
 *   TILE16_FAST   tile sums in double with a reordered (vectorisable) reduction; used only as the
 *                 timed CPU baseline of the reference arithmetic.
 *   UNFUSED_SEQ   TILE16_SEQ with each tile sum narrowed to FP16 before the fold
 *                 (ktiling_gate.reference(unfused=True)).
 *   FP64          full-K double sum (sum of sequential tile sums, ktiling_gate raw64/act64);
 *                 bias and HardSigmoid in double, no FP16 narrowing anywhere.
 *   FP32ACC       full-K float sum, float epilogue, one FP16 rounding at the end: a model of an
 *                 FP32-accumulating GPU kernel (not bitwise the same summation order).
 *
 * Outputs (any pointer may be NULL):
 *   y16   final FP16 output bits, [m,n] row-major
 *   act   final value before the last FP16 rounding, as double
 *   raw   pre-bias accumulator (FP16-valued for TILE16 modes), as double
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum {
    ORACLE_TILE16_EXACT = 0,
    ORACLE_TILE16_SEQ = 1,
    ORACLE_TILE16_FAST = 2,
    ORACLE_UNFUSED_SEQ = 3,
    ORACLE_FP64 = 4,
    ORACLE_FP32ACC = 5,
};

#define ORACLE_K_TILE 256u

/* ------------------------------------------------------------------ FP16 conversions */

double oracle_f16_to_double(uint16_t h) {
    unsigned sign = h >> 15, e = (h >> 10) & 31u, f = h & 1023u;
    double v;
    if (e == 0) v = ldexp((double)f, -24);
    else if (e == 31) v = f ? NAN : INFINITY;
    else v = ldexp((double)(f | 1024u), (int)e - 25);
    return sign ? -v : v;
}

/* Round-to-nearest-even double -> binary16, overflow to infinity (IEEE 754). */
uint16_t oracle_f16_from_double(double d) {
    uint16_t sign = signbit(d) ? 0x8000u : 0u;
    if (isnan(d)) return (uint16_t)(sign | 0x7e00u);
    double a = fabs(d);
    if (a >= 65520.0) return (uint16_t)(sign | 0x7c00u);  /* 65520 = 65504 + half ulp: ties to inf */
    int e2;
    frexp(a, &e2);                          /* a = f * 2^e2, f in [0.5,1) */
    int q = e2 - 11;                        /* quantum exponent for an 11-bit significand */
    if (q < -24) q = -24;                   /* subnormal quantum 2^-24 */
    double n = nearbyint(ldexp(a, -q));     /* exact scaling; default rounding mode is RNE */
    if (n == 0.0) return sign;
    /* n may have carried to 2048: the encoding below handles it */
    long iv = (long)n;
    int exp_q = q;
    while (iv >= 2048) { iv >>= 1; exp_q++; }   /* only an exact carry (iv == 2048) gets here */
    if (iv < 1024) return (uint16_t)(sign | (uint16_t)iv);   /* subnormal (exp_q == -24) */
    int biased = exp_q + 25;                /* value = iv * 2^exp_q, iv in [1024,2048) */
    if (biased >= 31) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | (uint16_t)(biased << 10) | (uint16_t)(iv - 1024));
}

static inline double f16r(double v) { return oracle_f16_to_double(oracle_f16_from_double(v)); }

/* ------------------------------------------------------------------ exact tile sums */

typedef __int128 i128;

/* FP16 value times 2^24 as an exact integer (|v| <= 65504 * 2^24 < 2^40). */
static inline int64_t f16_fixed(uint16_t h) {
    unsigned e = (h >> 10) & 31u, f = h & 1023u;
    int64_t mag = e ? ((int64_t)(f | 1024u) << (e - 1)) : (int64_t)f;
    return (h & 0x8000u) ? -mag : mag;
}

/* Correctly rounded (RNE) conversion of an exact 128-bit integer to double. */
static double i128_to_double(i128 v) {
    if (v == 0) return 0.0;
    int neg = v < 0;
    unsigned __int128 u = neg ? (unsigned __int128)(-v) : (unsigned __int128)v;
    int top = 127;
    while (!((u >> top) & 1)) top--;
    double r;
    if (top < 53) {
        r = (double)(uint64_t)u;
    } else {
        int shift = top - 52;                                     /* keep 53 bits */
        unsigned __int128 keep = u >> shift;
        unsigned __int128 rem = u - (keep << shift);
        unsigned __int128 half = (unsigned __int128)1 << (shift - 1);
        if (rem > half || (rem == half && (keep & 1))) keep++;
        r = ldexp((double)(uint64_t)keep, shift);
    }
    return neg ? -r : r;
}

static double tile_sum_exact(const uint16_t *x, const uint16_t *w, unsigned len) {
    i128 s = 0;
    for (unsigned c = 0; c < len; c++) s += (i128)f16_fixed(x[c]) * (i128)f16_fixed(w[c]);
    return ldexp(i128_to_double(s), -48);
}

/* ------------------------------------------------------------------ one output element */

typedef struct {
    int mode, post;
    unsigned m, k, n;
    const uint16_t *x, *w, *bias;
    const double *xd, *wd;       /* FP16 operands widened once (FAST / SEQ / FP64 modes) */
    uint16_t *y16;
    double *act, *raw;
    unsigned row_begin, row_end;
} oracle_job;

static double hsig(double v) {
    double r = v / 6.0 + 0.5;
    return r < 0.0 ? 0.0 : (r > 1.0 ? 1.0 : r);
}

static void element(const oracle_job *j, unsigned r, unsigned col) {
    const unsigned k = j->k;
    const size_t out = (size_t)r * j->n + col;
    double rawv, actv;
    if (j->mode == ORACLE_FP32ACC) {
        float s = 0.0f;
        const double *xr = j->xd + (size_t)r * k, *wr = j->wd + (size_t)col * k;
        for (unsigned c = 0; c < k; c++) s += (float)xr[c] * (float)wr[c];
        rawv = s;
        float a = s;
        if (j->bias) a += (float)oracle_f16_to_double(j->bias[col]);
        if (j->post) {
            float t = a / 6.0f + 0.5f;
            a = t < 0.0f ? 0.0f : (t > 1.0f ? 1.0f : t);
        }
        actv = a;
    } else if (j->mode == ORACLE_FP64) {
        const double *xr = j->xd + (size_t)r * k, *wr = j->wd + (size_t)col * k;
        double s64 = 0.0;
        for (unsigned k0 = 0; k0 < k; k0 += ORACLE_K_TILE) {
            unsigned end = k - k0 > ORACLE_K_TILE ? k0 + ORACLE_K_TILE : k;
            double ts = 0.0;
            for (unsigned c = k0; c < end; c++) ts += xr[c] * wr[c];
            s64 += ts;
        }
        rawv = s64;
        actv = s64;
        if (j->bias) actv += oracle_f16_to_double(j->bias[col]);
        if (j->post) actv = hsig(actv);
    } else {
        double dot = 0.0;
        for (unsigned k0 = 0, t = 0; k0 < k; k0 += ORACLE_K_TILE, t++) {
            unsigned len = k - k0 > ORACLE_K_TILE ? ORACLE_K_TILE : k - k0;
            double ts;
            if (j->mode == ORACLE_TILE16_EXACT) {
                ts = tile_sum_exact(j->x + (size_t)r * k + k0, j->w + (size_t)col * k + k0, len);
            } else if (j->mode == ORACLE_TILE16_FAST) {
                const double *xr = j->xd + (size_t)r * k + k0, *wr = j->wd + (size_t)col * k + k0;
                double s = 0.0;
#pragma omp simd reduction(+ : s)
                for (unsigned c = 0; c < len; c++) s += xr[c] * wr[c];
                ts = s;
            } else {
                const double *xr = j->xd + (size_t)r * k + k0, *wr = j->wd + (size_t)col * k + k0;
                ts = 0.0;
                for (unsigned c = 0; c < len; c++) ts += xr[c] * wr[c];
            }
            if (j->mode == ORACLE_UNFUSED_SEQ) ts = f16r(ts);
            dot = t == 0 ? f16r(ts) : f16r(dot + ts);
        }
        rawv = dot;
        double affine = j->bias ? f16r(dot + oracle_f16_to_double(j->bias[col])) : dot;
        actv = j->post ? hsig(affine) : affine;
    }
    if (j->raw) j->raw[out] = rawv;
    if (j->act) j->act[out] = actv;
    if (j->y16) j->y16[out] = oracle_f16_from_double(actv);
}

static void *worker(void *arg) {
    const oracle_job *j = arg;
    for (unsigned r = j->row_begin; r < j->row_end; r++)
        for (unsigned c = 0; c < j->n; c++) element(j, r, c);
    return NULL;
}

static double f16_table[65536];
static pthread_once_t f16_table_once = PTHREAD_ONCE_INIT;
static void f16_table_init(void) {
    for (unsigned i = 0; i < 65536; i++) f16_table[i] = oracle_f16_to_double((uint16_t)i);
}

static double *widen(const uint16_t *v, size_t n) {
    pthread_once(&f16_table_once, f16_table_init);
    double *d = malloc(n * sizeof(*d));
    if (!d) return NULL;
    for (size_t i = 0; i < n; i++) d[i] = f16_table[v[i]];
    return d;
}

/* Returns 0 on success, -1 on bad arguments, -3 on allocation failure. */
/* `w_wide`, when not NULL, is W already widened to double ([n,k]); it is used as is (and not
 * freed) by the modes that work on widened operands, so repeated calls skip the conversion. */
int oracle_linear_pre(int mode, unsigned m, unsigned k, unsigned n,
                      const uint16_t *x, const uint16_t *w, const double *w_wide,
                      const uint16_t *bias, int post,
                      uint16_t *y16, double *act, double *raw, int threads) {
    if (!m || !k || !n || !x || !w || mode < 0 || mode > ORACLE_FP32ACC || (post != 0 && post != 1))
        return -1;
    double *xd = NULL, *wd = NULL;
    const double *wuse = NULL;
    if (mode != ORACLE_TILE16_EXACT) {
        xd = widen(x, (size_t)m * k);
        if (!w_wide) wd = widen(w, (size_t)n * k);
        wuse = w_wide ? w_wide : wd;
        if (!xd || !wuse) { free(xd); free(wd); return -3; }
    }
    if (threads < 1) threads = 1;
    if ((unsigned)threads > m) threads = (int)m;
    oracle_job *jobs = calloc((size_t)threads, sizeof(*jobs));
    pthread_t *tid = calloc((size_t)threads, sizeof(*tid));
    if (!jobs || !tid) { free(jobs); free(tid); free(xd); free(wd); return -3; }
    for (int t = 0; t < threads; t++) {
        jobs[t] = (oracle_job){mode, post, m, k, n, x, w, bias, xd, wuse, y16, act, raw,
                               (unsigned)((size_t)m * t / threads),
                               (unsigned)((size_t)m * (t + 1) / threads)};
    }
    char *created = calloc((size_t)threads, 1);
    if (!created) { free(jobs); free(tid); free(xd); free(wd); return -3; }
    for (int t = 1; t < threads; t++)
        created[t] = pthread_create(&tid[t], NULL, worker, &jobs[t]) == 0;
    worker(&jobs[0]);
    for (int t = 1; t < threads; t++) {
        if (created[t]) pthread_join(tid[t], NULL);
        else worker(&jobs[t]);          /* a thread that could not start runs inline */
    }
    free(created); free(jobs); free(tid); free(xd); free(wd);
    return 0;
}

int oracle_linear(int mode, unsigned m, unsigned k, unsigned n,
                  const uint16_t *x, const uint16_t *w, const uint16_t *bias, int post,
                  uint16_t *y16, double *act, double *raw, int threads) {
    return oracle_linear_pre(mode, m, k, n, x, w, NULL, bias, post, y16, act, raw, threads);
}

/* Batch FP16 conversion helpers for the Python side. */
void oracle_f16_encode(const double *in, uint16_t *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = oracle_f16_from_double(in[i]);
}
void oracle_f16_decode(const uint16_t *in, double *out, size_t n) {
    for (size_t i = 0; i < n; i++) out[i] = oracle_f16_to_double(in[i]);
}
