/*
 * CPU oracle for the vkfft-rs FFT hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the crate's independent CPU reference
 * transform (vkfft-rs src/reference.rs) so that parity tests and the CPU
 * baseline leg of bench.py can check the B200 kernels against it.  Only the
 * test suite, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm load this library; the product path (libb200fft.so) never links it.
 *
 * Parity is pinned: tests/test_oracle.py checks this oracle against every
 * C2C/R2C FFTW 3.3.9 golden vector the reference commits under
 * tests/fixtures/ (extracted into tests/golden/fftw_golden.npz) at the
 * reference's own CPU tolerance 2e-10*n (tests/fftw_medium_golden.rs:161-171).
 *
 * Arithmetic follows reference.rs term by term so that rounding matches:
 *   - radix choice: first of {2,3,5,7,11,13} dividing n  (reference.rs:66-73,
 *     STOCKHAM_PRIMES planner.rs:10), else Bluestein    (reference.rs:74)
 *   - mixed radix: one exp_i per (k, lane) with angle
 *     sign*2*PI*lane*k/n evaluated left to right       (reference.rs:76-105)
 *   - Bluestein: M = next_smooth_at_least(2n-1,{2,3,5,7}) (reference.rs:114-115,
 *     planner.rs:684-733); chirp angle sign*PI*i*i/n NOT reduced mod 2n
 *     (reference.rs:121-125); kernel b[i] = b[M-i] = exp_i(-angle)
 *     (:125-130); FFT a, FFT b, product, inverse FFT, scale 1/M, post-chirp
 *     recomputed from the same angle expression         (reference.rs:132-151)
 *   - inverse normalisation multiplies by 1/n only when requested
 *     (reference.rs:35-41); Direction sign -1 forward / +1 inverse
 *     (config.rs:9-16); exp_i = (cos, sin) via libm   (complex.rs:97-99)
 * Build with -ffp-contract=off so no FMA changes the rounding.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    double re, im;
} cplx;

static const double PI = 3.14159265358979323846264338327950288;
static const size_t STOCKHAM_PRIMES[6] = {2, 3, 5, 7, 11, 13};
static const size_t BLUESTEIN_SMOOTH_PRIMES[4] = {2, 3, 5, 7};

static inline cplx c_mul(cplx a, cplx b) {
    cplx r;
    r.re = a.re * b.re - a.im * b.im;
    r.im = a.re * b.im + a.im * b.re;
    return r;
}

static inline cplx exp_i(double angle) {
    cplx r;
    r.re = cos(angle);
    r.im = sin(angle);
    return r;
}

/* planner.rs:684-733 next_smooth_at_least: depth-first search over exponents */
static void smooth_visit(const size_t *primes, size_t count, size_t index, size_t current,
                         size_t target, size_t *best) {
    if (current >= *best) return;
    if (index == count) {
        if (current >= target) *best = current;
        return;
    }
    size_t prime = primes[index];
    size_t value = current;
    for (;;) {
        smooth_visit(primes, count, index + 1, value, target, best);
        if (value > SIZE_MAX / prime) break;
        size_t next = value * prime;
        if (next < *best)
            value = next;
        else
            break;
    }
}

size_t oracle_next_smooth_at_least(size_t target) {
    if (target <= 1) return 1;
    size_t best = SIZE_MAX;
    /* 2 is in the set: start from the next power of two */
    size_t p = 1;
    while (p < target && p <= SIZE_MAX / 2) p <<= 1;
    if (p >= target) best = p;
    smooth_visit(BLUESTEIN_SMOOTH_PRIMES, 4, 0, 1, target, &best);
    return best;
}

static int fft_unscaled(const cplx *input, cplx *output, size_t n, double sign);

/* reference.rs:76-105 */
static int mixed_radix_unscaled(const cplx *input, cplx *output, size_t n, double sign,
                                size_t radix) {
    size_t inner_len = n / radix;
    cplx *seq = (cplx *)malloc(sizeof(cplx) * inner_len);
    cplx *inner = (cplx *)malloc(sizeof(cplx) * n); /* radix blocks of inner_len */
    if (!seq || !inner) {
        free(seq);
        free(inner);
        return -1;
    }
    for (size_t lane = 0; lane < radix; lane++) {
        for (size_t index = 0; index < inner_len; index++) seq[index] = input[lane + radix * index];
        if (fft_unscaled(seq, inner + lane * inner_len, inner_len, sign) != 0) {
            free(seq);
            free(inner);
            return -1;
        }
    }
    for (size_t k = 0; k < n; k++) {
        size_t inner_index = k % inner_len;
        cplx sum = {0.0, 0.0};
        for (size_t lane = 0; lane < radix; lane++) {
            double angle = sign * 2.0 * PI * (double)lane * (double)k / (double)n;
            cplx t = c_mul(inner[lane * inner_len + inner_index], exp_i(angle));
            sum.re += t.re;
            sum.im += t.im;
        }
        output[k] = sum;
    }
    free(seq);
    free(inner);
    return 0;
}

/* reference.rs:107-153 */
static int bluestein_unscaled(const cplx *input, cplx *output, size_t n, double sign) {
    size_t minimum = n * 2 - 1;
    size_t m = oracle_next_smooth_at_least(minimum);
    cplx *a = (cplx *)calloc(m, sizeof(cplx));
    cplx *b = (cplx *)calloc(m, sizeof(cplx));
    cplx *af = (cplx *)malloc(sizeof(cplx) * m);
    cplx *bf = (cplx *)malloc(sizeof(cplx) * m);
    cplx *conv = (cplx *)malloc(sizeof(cplx) * m);
    int status = -1;
    if (!a || !b || !af || !bf || !conv) goto done;
    for (size_t index = 0; index < n; index++) {
        double x = (double)index;
        double angle = sign * PI * x * x / (double)n;
        cplx chirp = exp_i(angle);
        cplx inverse_chirp = exp_i(-angle);
        a[index] = c_mul(input[index], chirp);
        b[index] = inverse_chirp;
        if (index != 0) b[m - index] = inverse_chirp;
    }
    if (fft_unscaled(a, af, m, -1.0) != 0) goto done;
    if (fft_unscaled(b, bf, m, -1.0) != 0) goto done;
    for (size_t index = 0; index < m; index++) a[index] = c_mul(af[index], bf[index]);
    if (fft_unscaled(a, conv, m, 1.0) != 0) goto done;
    {
        double scale = 1.0 / (double)m;
        for (size_t index = 0; index < n; index++) {
            cplx v = conv[index];
            v.re *= scale;
            v.im *= scale;
            double x = (double)index;
            double angle = sign * PI * x * x / (double)n;
            output[index] = c_mul(v, exp_i(angle));
        }
    }
    status = 0;
done:
    free(a);
    free(b);
    free(af);
    free(bf);
    free(conv);
    return status;
}

/* reference.rs:60-75 */
static int fft_unscaled(const cplx *input, cplx *output, size_t n, double sign) {
    if (n <= 1) {
        if (n == 1) output[0] = input[0];
        return 0;
    }
    for (int i = 0; i < 6; i++) {
        if (n % STOCKHAM_PRIMES[i] == 0) return mixed_radix_unscaled(input, output, n, sign, STOCKHAM_PRIMES[i]);
    }
    return bluestein_unscaled(input, output, n, sign);
}

/* reference.rs:25-42; direction: 0 forward, 1 inverse.  in/out interleaved re,im. */
int oracle_fft(const double *in, double *out, size_t n, int inverse, int normalize) {
    if (n == 0) return 0;
    double sign = inverse ? 1.0 : -1.0;
    int status = fft_unscaled((const cplx *)in, (cplx *)out, n, sign);
    if (status != 0) return status;
    if (inverse && normalize) {
        double scale = 1.0 / (double)n;
        for (size_t i = 0; i < 2 * n; i++) out[i] *= scale;
    }
    return 0;
}

/* reference.rs:14-23 and :44-58: the O(n^2) direct DFT */
int oracle_dft(const double *in, double *out, size_t n, int inverse, int normalize) {
    const cplx *input = (const cplx *)in;
    cplx *output = (cplx *)out;
    double sign = inverse ? 1.0 : -1.0;
    for (size_t k = 0; k < n; k++) {
        cplx sum = {0.0, 0.0};
        for (size_t index = 0; index < n; index++) {
            double angle = sign * 2.0 * PI * (double)index * (double)k / (double)n;
            cplx t = c_mul(input[index], exp_i(angle));
            sum.re += t.re;
            sum.im += t.im;
        }
        output[k] = sum;
    }
    if (inverse && normalize && n > 0) {
        double scale = 1.0 / (double)n;
        for (size_t i = 0; i < 2 * n; i++) out[i] *= scale;
    }
    return 0;
}

/* ---- batched / multi-axis drivers (thread-parallel over independent lines) ---- */

typedef struct {
    /* one job = a set of lines along one axis of a dense [outer][len][inner] tensor */
    const double *in;
    double *out;
    size_t len, inner, lines;
    size_t first, last; /* line range [first, last) */
    int inverse, normalize;
    int kind; /* 0 c2c, 1 r2c (in real, out half complex), 2 c2r (in half, out real) */
    int status;
} line_job;

static void *run_lines(void *arg) {
    line_job *job = (line_job *)arg;
    size_t len = job->len;
    size_t half = len / 2 + 1;
    cplx *buf = (cplx *)malloc(sizeof(cplx) * len);
    cplx *res = (cplx *)malloc(sizeof(cplx) * len);
    if (!buf || !res) {
        job->status = -1;
        free(buf);
        free(res);
        return NULL;
    }
    for (size_t line = job->first; line < job->last && job->status == 0; line++) {
        size_t o = line / job->inner, i = line % job->inner;
        if (job->kind == 0) {
            const cplx *src = (const cplx *)job->in;
            cplx *dst = (cplx *)job->out;
            for (size_t e = 0; e < len; e++) buf[e] = src[(o * len + e) * job->inner + i];
            if (oracle_fft((const double *)buf, (double *)res, len, job->inverse, job->normalize)) job->status = -1;
            for (size_t e = 0; e < len; e++) dst[(o * len + e) * job->inner + i] = res[e];
        } else if (job->kind == 1) {
            /* R2C over the contiguous axis (inner == 1): first len/2+1 bins of the
             * complex FFT of (x, 0) */
            const double *src = job->in + line * len;
            cplx *dst = (cplx *)job->out + line * half;
            for (size_t e = 0; e < len; e++) {
                buf[e].re = src[e];
                buf[e].im = 0.0;
            }
            if (oracle_fft((const double *)buf, (double *)res, len, 0, 0)) job->status = -1;
            for (size_t e = 0; e < half; e++) dst[e] = res[e];
        } else {
            /* C2R: Hermitian expansion then inverse complex FFT, keep .re
             * (real_ir.rs:1037-1053 FullComplex branch) */
            const cplx *src = (const cplx *)job->in + line * half;
            double *dst = job->out + line * len;
            for (size_t k = 0; k < len; k++) {
                if (k < half) {
                    buf[k] = src[k];
                } else {
                    buf[k].re = src[len - k].re;
                    buf[k].im = -src[len - k].im;
                }
            }
            if (oracle_fft((const double *)buf, (double *)res, len, 1, job->normalize)) job->status = -1;
            for (size_t e = 0; e < len; e++) dst[e] = res[e].re;
        }
    }
    free(buf);
    free(res);
    return NULL;
}

static int run_parallel(line_job proto, size_t lines, int threads) {
    if (threads < 1) threads = 1;
    if ((size_t)threads > lines) threads = (int)(lines ? lines : 1);
    pthread_t *tid = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)threads);
    line_job *jobs = (line_job *)malloc(sizeof(line_job) * (size_t)threads);
    if (!tid || !jobs) {
        free(tid);
        free(jobs);
        return -1;
    }
    size_t per = (lines + (size_t)threads - 1) / (size_t)threads;
    int started = 0;
    for (int t = 0; t < threads; t++) {
        jobs[t] = proto;
        jobs[t].first = (size_t)t * per;
        jobs[t].last = jobs[t].first + per > lines ? lines : jobs[t].first + per;
        jobs[t].status = 0;
        if (jobs[t].first >= jobs[t].last) continue;
        if (threads == 1) {
            run_lines(&jobs[t]);
        } else if (pthread_create(&tid[t], NULL, run_lines, &jobs[t]) == 0) {
            started |= 0;
        } else {
            run_lines(&jobs[t]);
            jobs[t].first = jobs[t].last; /* mark as not joinable */
        }
    }
    int status = 0;
    for (int t = 0; t < threads; t++) {
        if (threads > 1 && jobs[t].first < jobs[t].last) pthread_join(tid[t], NULL);
        if (jobs[t].status) status = -1;
    }
    free(tid);
    free(jobs);
    (void)started;
    return status;
}

/* Complex FFT along one axis of a dense tensor viewed as [outer][len][inner];
 * in and out may alias. */
int oracle_fft_axis(const double *in, double *out, size_t outer, size_t len, size_t inner,
                    int inverse, int normalize, int threads) {
    line_job job;
    memset(&job, 0, sizeof(job));
    job.in = in;
    job.out = out;
    job.len = len;
    job.inner = inner;
    job.inverse = inverse;
    job.normalize = normalize;
    job.kind = 0;
    return run_parallel(job, outer * inner, threads);
}

/* Batched contiguous C2C: batch lines of length n. */
int oracle_fft_batch(const double *in, double *out, size_t n, size_t batch, int inverse,
                     int normalize, int threads) {
    return oracle_fft_axis(in, out, batch, n, 1, inverse, normalize, threads);
}

/* Batched R2C over contiguous real lines of length n -> n/2+1 complex bins. */
int oracle_r2c_batch(const double *in, double *out, size_t n, size_t batch, int threads) {
    line_job job;
    memset(&job, 0, sizeof(job));
    job.in = in;
    job.out = out;
    job.len = n;
    job.inner = 1;
    job.kind = 1;
    return run_parallel(job, batch, threads);
}

/* Batched C2R: n/2+1 complex bins -> n real values, optional 1/n. */
int oracle_c2r_batch(const double *in, double *out, size_t n, size_t batch, int normalize,
                     int threads) {
    line_job job;
    memset(&job, 0, sizeof(job));
    job.in = in;
    job.out = out;
    job.len = n;
    job.inner = 1;
    job.kind = 2;
    job.normalize = normalize;
    return run_parallel(job, batch, threads);
}
