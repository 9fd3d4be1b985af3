/*
 * Double-double oracle of the CPU checker -- TEST INFRASTRUCTURE ONLY.
 *
 * The DoubleDouble precisions of vkfft-rs (src/double_double.rs: a value is hi + lo of
 * two binary64 words, complex values are (re.hi, re.lo, im.hi, im.lo)) are checked
 * against the method the crate's own double-double golden vectors were made with
 * (tests/fixtures/quad_precision_medium_double_double_v1.txt header: "source
 * libquadmath-direct-113bit-kahan-v1", "rounding double-double-hi-lo-rne-from-f128-v1"):
 * a direct O(n^2) DFT evaluated in binary128 with Kahan-compensated sums, each result
 * rounded to the nearest double (hi) plus the nearest double of the remainder (lo).
 * The roots are exp(sign 2 pi i m / n) with m = j k mod n reduced exactly.  The same
 * evaluation gives the eight DCT/DST kinds from their FFTW definitions (the direct sums
 * of r2r_ir.rs:2351-2433).  tests/test_oracle.py pins these functions against the
 * crate's committed double-double fixtures.  Only the tests load this library.
 */
#include <pthread.h>
#include <quadmath.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef __float128 q128;

static q128 qpi(void) { return 4 * atanq((q128)1); }

static q128 dd_read(const double *w) { return (q128)w[0] + (q128)w[1]; }

static void dd_write(q128 v, double *w) {
    const double hi = (double)v;
    w[0] = hi;
    w[1] = (double)(v - (q128)hi);
}

/* Kahan-compensated accumulator */
typedef struct {
    q128 sum, comp;
} kahan;

static void kahan_add(kahan *k, q128 v) {
    const q128 y = v - k->comp;
    const q128 t = k->sum + y;
    k->comp = (t - k->sum) - y;
    k->sum = t;
}

/* ---- complex DFT ------------------------------------------------------------------ */

typedef struct {
    const double *in;
    double *out;
    size_t n, line0, line1;
    int inverse, normalize;
    const q128 *wr, *wi; /* roots exp(sign 2 pi i m / n) */
} dft_job;

static void *dft_lines(void *arg) {
    dft_job *j = (dft_job *)arg;
    const size_t n = j->n;
    q128 *xr = (q128 *)malloc(n * sizeof(q128)), *xi = (q128 *)malloc(n * sizeof(q128));
    for (size_t line = j->line0; line < j->line1; line++) {
        const double *src = j->in + line * n * 4;
        for (size_t m = 0; m < n; m++) {
            xr[m] = dd_read(src + 4 * m);
            xi[m] = dd_read(src + 4 * m + 2);
        }
        double *dst = j->out + line * n * 4;
        for (size_t k = 0; k < n; k++) {
            kahan re = {0, 0}, im = {0, 0};
            for (size_t m = 0; m < n; m++) {
                const size_t r = (size_t)(((unsigned __int128)m * k) % n);
                kahan_add(&re, xr[m] * j->wr[r] - xi[m] * j->wi[r]);
                kahan_add(&im, xr[m] * j->wi[r] + xi[m] * j->wr[r]);
            }
            q128 vr = re.sum, vi = im.sum;
            if (j->inverse && j->normalize) {
                vr /= (q128)n;
                vi /= (q128)n;
            }
            dd_write(vr, dst + 4 * k);
            dd_write(vi, dst + 4 * k + 2);
        }
    }
    free(xr);
    free(xi);
    return NULL;
}

static int run_jobs(void *(*fn)(void *), void *jobs, size_t job_size, size_t lines, int threads) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > lines) threads = lines ? (int)lines : 1;
    pthread_t tid[256];
    if (threads > 256) threads = 256;
    for (int t = 0; t < threads; t++) {
        char *job = (char *)jobs + (size_t)t * job_size;
        if (pthread_create(&tid[t], NULL, fn, job) != 0) return -1;
    }
    for (int t = 0; t < threads; t++) pthread_join(tid[t], NULL);
    return 0;
}

/* lines x n complex double-double values (4 words each), transformed along n. */
int oracle_dd_dft_lines(const double *in, double *out, size_t n, size_t lines, int inverse, int normalize,
                        int threads) {
    if (n == 0) return -1;
    q128 *wr = (q128 *)malloc(n * sizeof(q128)), *wi = (q128 *)malloc(n * sizeof(q128));
    const q128 sign = inverse ? 1 : -1;
    for (size_t m = 0; m < n; m++) {
        const q128 a = sign * 2 * qpi() * (q128)m / (q128)n;
        wr[m] = cosq(a);
        wi[m] = sinq(a);
    }
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    dft_job jobs[256];
    const size_t per = (lines + threads - 1) / threads;
    int used = 0;
    for (int t = 0; t < threads; t++) {
        const size_t a = (size_t)t * per, b = a + per < lines ? a + per : lines;
        if (a >= b) break;
        jobs[t] = (dft_job){in, out, n, a, b, inverse, normalize, wr, wi};
        used++;
    }
    const int rc = run_jobs(dft_lines, jobs, sizeof(dft_job), (size_t)used, used);
    free(wr);
    free(wi);
    return rc;
}

/* ---- DCT / DST ---------------------------------------------------------------------- */

/* 2 * cos or 2 * sin of pi * num / den, num reduced modulo 2 den first */
static q128 trig(int use_sin, uint64_t num, uint64_t den) {
    num %= 2 * den;
    const q128 a = qpi() * (q128)num / (q128)den;
    return use_sin ? sinq(a) : cosq(a);
}

/* matrix entry M[k][j] of the unnormalised kind (0..3 DCT-I..IV, 4..7 DST-I..IV) */
static q128 r2r_entry(int kind, size_t n, size_t k, size_t j) {
    switch (kind) {
        case 0:
            if (j == 0) return 1;
            if (j == n - 1) return (k % 2) ? -1 : 1;
            return 2 * trig(0, (uint64_t)j * k, n - 1);
        case 1: return 2 * trig(0, (uint64_t)(2 * j + 1) * k, 2 * n);
        case 2: return j == 0 ? (q128)1 : 2 * trig(0, (uint64_t)j * (2 * k + 1), 2 * n);
        case 3: return 2 * trig(0, (uint64_t)(2 * j + 1) * (2 * k + 1), 4 * n);
        case 4: return 2 * trig(1, (uint64_t)(j + 1) * (k + 1), n + 1);
        case 5: return 2 * trig(1, (uint64_t)(2 * j + 1) * (k + 1), 2 * n);
        case 6:
            if (j == n - 1) return (k % 2) ? -1 : 1;
            return 2 * trig(1, (uint64_t)(j + 1) * (2 * k + 1), 2 * n);
        default: return 2 * trig(1, (uint64_t)(2 * j + 1) * (2 * k + 1), 4 * n);
    }
}

typedef struct {
    const double *in;
    double *out;
    size_t n, line0, line1;
    const q128 *m; /* n x n matrix, row k */
} r2r_job;

static void *r2r_lines(void *arg) {
    r2r_job *j = (r2r_job *)arg;
    const size_t n = j->n;
    q128 *x = (q128 *)malloc(n * sizeof(q128));
    for (size_t line = j->line0; line < j->line1; line++) {
        for (size_t m = 0; m < n; m++) x[m] = dd_read(j->in + (line * n + m) * 2);
        for (size_t k = 0; k < n; k++) {
            kahan acc = {0, 0};
            for (size_t m = 0; m < n; m++) kahan_add(&acc, j->m[k * n + m] * x[m]);
            dd_write(acc.sum, j->out + (line * n + k) * 2);
        }
    }
    free(x);
    return NULL;
}

/* lines x n real double-double values (2 words each): the R2R kind along n.  inverse:
 * the partner kind (II <-> III), normalised by inverse_pair_scale of `kind`. */
int oracle_dd_r2r_lines(const double *in, double *out, size_t n, size_t lines, int kind, int inverse,
                        int normalize, int threads) {
    if (n == 0 || (kind == 0 && n < 2)) return -1;
    int eff = kind;
    if (inverse && ((kind & 3) == 1 || (kind & 3) == 2)) eff = kind ^ 3;
    q128 scale = 1;
    if (inverse && normalize) {
        const size_t den = kind == 0 ? 2 * (n - 1) : (kind == 4 ? 2 * (n + 1) : 2 * n);
        scale = (q128)1 / (q128)den;
    }
    q128 *mat = (q128 *)malloc(n * n * sizeof(q128));
    for (size_t k = 0; k < n; k++)
        for (size_t j = 0; j < n; j++) mat[k * n + j] = r2r_entry(eff, n, k, j) * scale;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    r2r_job jobs[256];
    const size_t per = (lines + threads - 1) / threads;
    int used = 0;
    for (int t = 0; t < threads; t++) {
        const size_t a = (size_t)t * per, b = a + per < lines ? a + per : lines;
        if (a >= b) break;
        jobs[t] = (r2r_job){in, out, n, a, b, mat};
        used++;
    }
    const int rc = run_jobs(r2r_lines, jobs, sizeof(r2r_job), (size_t)used, used);
    free(mat);
    return rc;
}
