// Lowering: per-axis plans -> B200 launch programs.
//
// Every axis transform becomes one pass when its working set fits in one CTA's
// shared memory (Stockham / Rader / Bluestein all fused into a single
// load -> on-chip program -> store), otherwise a four-step split (Stockham) or a
// three-pass convolution (Bluestein) through device scratch.  Tables are built
// on the host in f64 (roots from long double, the Bluestein chirp with the
// reference's own f64 expression) and rounded to f32 for f32 passes.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include <quadmath.h>

#include "lower.hpp"

namespace b200fft {

FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{};
    f.d = d;
    uint32_t s = 0;
    while (s < 31 && (1u << s) < d) s++;
    f.s = s;
    f.m = (uint32_t)((((uint64_t)1 << 32) * (((uint64_t)1 << s) - d)) / d + 1);
    return f;
}

// ---- host tables ------------------------------------------------------------

static std::complex<double> root(size_t m, size_t n) {
    // exp(-2 pi i m / n) rounded from long double
    const long double PIL = 3.141592653589793238462643383279502884L;
    long double a = -2.0L * PIL * (long double)(m % n) / (long double)n;
    return {(double)cosl(a), (double)sinl(a)};
}

// ---- double-double tables: computed in binary128 (libquadmath), each value split into
// the nearest double (hi) and the nearest double of the remainder (lo) ---------------
using q128 = __float128;
struct QC {
    q128 re, im;
};

static QC qmul(QC a, QC b) { return {a.re * b.re - a.im * b.im, a.re * b.im + a.im * b.re}; }

static QC root_q(size_t m, size_t n) {
    // exp(-2 pi i m / n), the ratio reduced exactly before the angle is formed
    static const q128 pi = 4 * atanq((q128)1);
    const q128 a = -2 * pi * (q128)(m % n) / (q128)n;
    return {cosq(a), sinq(a)};
}

static void put_q(HostTable &t, size_t idx, QC v) {
    if (t.c.size() <= idx) t.c.resize(idx + 1);
    if (t.lo.size() <= idx) t.lo.resize(idx + 1);
    const double hr = (double)v.re, hi_ = (double)v.im;
    t.c[idx] = {hr, hi_};
    t.lo[idx] = {(double)(v.re - (q128)hr), (double)(v.im - (q128)hi_)};
}

// Table entry idx = W_n^m (conjugated when `conj`), in the program's table precision.
static void put_root(HostTable &t, const Program &prog, size_t idx, size_t m, size_t n, bool conj = false);

// The host Stockham FFT of host_fft_inplace in binary128 (double-double spectra).
static void host_fft_q(std::vector<QC> &x) {
    const size_t n = x.size();
    if (n <= 1) return;
    auto f = prime_factorization(n);
    std::vector<QC> w(n), y(n);
    for (size_t m = 0; m < n; m++) w[m] = root_q(m, n);
    size_t P = 1;
    for (size_t r : f) {
        const size_t nbl = n / r;
        const size_t tstep = n / (P * r);
        std::vector<QC> v(r), o(r);
        for (size_t bb = 0; bb < nbl; bb++) {
            const size_t j = bb % P;
            for (size_t q = 0; q < r; q++) v[q] = qmul(x[bb + q * nbl], w[(j * q * tstep) % n]);
            for (size_t k = 0; k < r; k++) {
                QC acc{0, 0};
                for (size_t q = 0; q < r; q++) {
                    const QC u = qmul(v[q], w[((q * k) % r) * (n / r)]);
                    acc.re += u.re;
                    acc.im += u.im;
                }
                o[k] = acc;
            }
            const size_t e0 = (bb - j) * r + j;
            for (size_t q = 0; q < r; q++) y[e0 + q * P] = o[q];
        }
        std::swap(x, y);
        P *= r;
    }
}

static int add_table(Program &prog, const std::string &key, HostTable t) {
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    t.key = key;
    prog.tables.push_back(std::move(t));
    int id = (int)prog.tables.size() - 1;
    prog.table_cache[key] = id;
    return id;
}

int table_twiddle(Program &prog, size_t n) {
    std::string key = "W" + std::to_string(n);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    HostTable t;
    t.c.resize(n);
    for (size_t m = 0; m < n; m++) put_root(t, prog, m, m, n);
    return add_table(prog, key, std::move(t));
}

static void put_root(HostTable &t, const Program &prog, size_t idx, size_t m, size_t n, bool conj) {
    if (prog.is_dd) {
        QC v = root_q(m, n);
        if (conj) v.im = -v.im;
        put_q(t, idx, v);
        return;
    }
    if (t.c.size() <= idx) t.c.resize(idx + 1);
    const std::complex<double> v = root(m, n);
    t.c[idx] = conj ? std::conj(v) : v;
}

static std::string reg_twiddle_key(size_t n, int variant) {
    int rad[8];
    const int ns = reg_variant_radices(variant, rad);
    // keyed by the radix sequence too: two variants of one length may order their stages
    // differently (and so need different tables)
    std::string key = "regtw" + std::to_string(n);
    for (int s = 0; s < ns; s++) key += "_" + std::to_string(rad[s]);
    return key;
}

// Stage twiddles of a register-kernel variant: for every stage s > 0 (span P, radix R)
// a transposed block tw[(q-1)*P + j] = W_{P R}^{j q}, q = 1..R-1, j = 0..P-1, blocks in
// stage order (reg_kernels.cu reads them at compile-time offsets).
int table_reg_twiddles(Program &prog, size_t n, int variant) {
    int rad[8];
    const int ns = reg_variant_radices(variant, rad);
    const std::string key = reg_twiddle_key(n, variant);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    HostTable t;
    size_t P = 1;
    for (int s = 0; s < ns; s++) {
        const size_t R = (size_t)rad[s];
        if (P > 1)
            for (size_t q = 1; q < R; q++)
                for (size_t j = 0; j < P; j++) t.c.push_back(root(j * q, P * R));
        P *= R;
    }
    if (t.c.empty()) t.c.push_back({1.0, 0.0});
    return add_table(prog, key, std::move(t));
}

void check_reg_twiddle_tables(const Program &prog) {
    for (const PassPlan &pp : prog.passes) {
        if (pp.kernel != KERNEL_REG || pp.reg_table < 0 || pp.reg_variant < 0) continue;
        if ((size_t)pp.reg_table >= prog.tables.size()) fail_runtime("register pass names a missing table");
        const std::string &key = prog.tables[(size_t)pp.reg_table].key;
        if (key.compare(0, 5, "regtw") != 0) continue;  // not a stage-twiddle table
        for (int v : {pp.reg_variant, pp.reg_variant_plain})
            if (v >= 0 && key != reg_twiddle_key((size_t)reg_variant_length(v), v))
                fail_runtime("register pass reads the stage twiddles of another length or radix split");
    }
}

// Twiddles of one radix-R Stockham stage of span P, transposed: entry (q-1)*P + j holds
// W_{P R}^{j q} (q = 1..R-1), so the butterflies of a warp (consecutive j) read
// consecutive entries.
int table_stage_twiddles(Program &prog, size_t R, size_t P) {
    std::string key = "stw" + std::to_string(R) + "_" + std::to_string(P);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    HostTable t;
    t.c.reserve((R - 1) * P);
    for (size_t q = 1; q < R; q++)
        for (size_t j = 0; j < P; j++) put_root(t, prog, (q - 1) * P + j, j * q, P * R);
    return add_table(prog, key, std::move(t));
}

// Rader line kernel table (reg_kernels.cu reg_rader_kernel): FFT_{P-1} of the Rader
// kernel b[q] = W_P^(g^-q mod P), divided by P - 1, with g the smallest primitive root of
// P; evaluated in binary128 from exactly reduced ratios.
int table_rader_line(Program &prog, size_t P) {
    std::string key = "rline" + std::to_string(P);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    const size_t L = P - 1;
    size_t g = 2;
    for (;; g++) {
        size_t v = 1, order = 0;
        do {
            v = v * g % P;
            order++;
        } while (v != 1);
        if (order == L) break;
    }
    size_t ginv = 1;
    for (size_t k = 0; k < P - 2; k++) ginv = ginv * g % P;
    std::vector<size_t> r(L);  // g^-q mod P
    size_t v = 1;
    for (size_t q = 0; q < L; q++, v = v * ginv % P) r[q] = v;
    HostTable t;
    for (size_t k = 0; k < L; k++) {
        QC acc{0, 0};
        for (size_t q = 0; q < L; q++) {
            const QC b = root_q(r[q], P), w = root_q((q * k) % L, L);
            acc.re += b.re * w.re - b.im * w.im;
            acc.im += b.re * w.im + b.im * w.re;
        }
        acc.re /= (q128)L;
        acc.im /= (q128)L;
        put_q(t, k, acc);
    }
    return add_table(prog, key, std::move(t));
}

// Four-step twiddles W_N^{c e} for line (column) c < ncols and element e < nrows, stored
// element-major (entry e*ncols + c): lines-fastest passes read consecutive entries.
int table_twiddle_transposed(Program &prog, size_t ncols, size_t nrows, size_t N) {
    std::string key = "ttw" + std::to_string(ncols) + "_" + std::to_string(nrows) + "_" + std::to_string(N);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    HostTable t;
    t.c.reserve(ncols * nrows);
    for (size_t e = 0; e < nrows; e++)
        for (size_t c = 0; c < ncols; c++) put_root(t, prog, e * ncols + c, (c * e) % N, N);
    return add_table(prog, key, std::move(t));
}

// Bluestein chirp exactly as the reference evaluates it (reference.rs:121-125,
// lut.rs:295-299): angle = sign * PI * (i as f64) * (i as f64) / (n as f64), not
// reduced modulo 2n, then libm cos / sin.  Forward sign (-1); inverse transforms
// use the conjugate, which is bit-identical to the +1 evaluation.
static std::vector<std::complex<double>> reference_chirp(size_t n) {
    const double PI = 3.14159265358979323846264338327950288;
    std::vector<std::complex<double>> c(n);
    for (size_t i = 0; i < n; i++) {
        double x = (double)i;
        double angle = -1.0 * PI * x * x / (double)n;
        c[i] = {std::cos(angle), std::sin(angle)};
    }
    return c;
}

int table_bluestein_chirp(Program &prog, size_t n) {
    std::string key = "chirp" + std::to_string(n);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    HostTable t;
    if (prog.is_dd) {
        // double-double: the chirp reduced exactly, W_2n^(i^2 mod 2n) (lut.rs:325-371)
        for (size_t i = 0; i < n; i++) put_q(t, i, root_q((size_t)(((unsigned __int128)i * i) % (2 * n)), 2 * n));
    } else {
        t.c = reference_chirp(n);
    }
    return add_table(prog, key, std::move(t));
}

// FFT_M(b) / M with b[i] = b[M-i] = conj(chirp[i]) (bluestein_ir.rs:629, reference.rs:125-130).
int table_bluestein_spectrum(Program &prog, size_t n, size_t m) {
    std::string key = "bspec" + std::to_string(n) + "_" + std::to_string(m);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    if (prog.is_dd) {
        std::vector<QC> b(m, QC{0, 0});
        for (size_t i = 0; i < n; i++) {
            QC ic = root_q((size_t)(((unsigned __int128)i * i) % (2 * n)), 2 * n);
            ic.im = -ic.im;
            b[i] = ic;
            if (i != 0) b[m - i] = ic;
        }
        host_fft_q(b);
        HostTable t;
        for (size_t k = 0; k < m; k++) put_q(t, k, QC{b[k].re / (q128)m, b[k].im / (q128)m});
        return add_table(prog, key, std::move(t));
    }
    auto chirp = reference_chirp(n);
    std::vector<std::complex<double>> b(m, {0.0, 0.0});
    for (size_t i = 0; i < n; i++) {
        std::complex<double> ic = std::conj(chirp[i]);
        b[i] = ic;
        if (i != 0) b[m - i] = ic;
    }
    host_fft_inplace(b, false);
    double s = 1.0 / (double)m;
    for (auto &v : b) v *= s;
    HostTable t;
    t.c = std::move(b);
    return add_table(prog, key, std::move(t));
}

// The Bluestein spectrum in the row order of a three-pass convolution: entry k1 M2 + k2
// holds spectrum[k1 + M1 k2] (the rows of the middle pass are then read contiguously).
int table_bluestein_spectrum_rows(Program &prog, size_t n, size_t m, size_t m1, size_t m2) {
    std::string key = "bspecrows" + std::to_string(n) + "_" + std::to_string(m) + "_" + std::to_string(m1);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    const HostTable &src = prog.tables[table_bluestein_spectrum(prog, n, m)];
    HostTable t;
    t.c.resize(m);
    if (!src.lo.empty()) t.lo.resize(m);
    for (size_t k1 = 0; k1 < m1; k1++)
        for (size_t k2 = 0; k2 < m2; k2++) {
            t.c[k1 * m2 + k2] = src.c[k1 + m1 * k2];
            if (!src.lo.empty()) t.lo[k1 * m2 + k2] = src.lo[k1 + m1 * k2];
        }
    return add_table(prog, key, std::move(t));
}

// Accurate host mixed-radix FFT (Stockham, twiddles from long double), used only to
// build kernel spectra.  O(n * sum of prime factors).
void host_fft_inplace(std::vector<std::complex<double>> &x, bool inverse) {
    const size_t n = x.size();
    if (n <= 1) return;
    auto f = prime_factorization(n);
    std::vector<std::complex<double>> w(n);
    for (size_t m = 0; m < n; m++) {
        auto r = root(m, n);
        w[m] = inverse ? std::conj(r) : r;
    }
    std::vector<std::complex<double>> y(n);
    size_t P = 1;
    for (size_t r : f) {
        const size_t nbl = n / r;
        const size_t tstep = n / (P * r);
        std::vector<std::complex<double>> v(r), o(r);
        for (size_t bb = 0; bb < nbl; bb++) {
            const size_t j = bb % P;
            for (size_t q = 0; q < r; q++) v[q] = x[bb + q * nbl] * w[(j * q * tstep) % n];
            for (size_t k = 0; k < r; k++) {
                std::complex<double> s = 0;
                for (size_t q = 0; q < r; q++) s += v[q] * w[((q * k) % r) * (n / r)];
                o[k] = s;
            }
            const size_t e0 = (bb - j) * r + j;
            for (size_t q = 0; q < r; q++) y[e0 + q * P] = o[q];
        }
        std::swap(x, y);
        P *= r;
    }
}

// Rader tables for prime p with generator g (rader_ir.rs:35-380, lut.rs:375-435):
// perm[m] = g^m mod p, ginv[m] = g^-m mod p, b[m] = W_p^{ginv[m]};
// FFT mode uses FFT_{p-1}(b) / (p-1).
struct RaderTables {
    int perm, ginv, kernel;
};

static RaderTables table_rader(Program &prog, size_t p, size_t g, bool fft_mode) {
    std::string kp = "rperm" + std::to_string(p), ki = "rginv" + std::to_string(p);
    std::string kk = (fft_mode ? "rspec" : "rker") + std::to_string(p);
    RaderTables rt{};
    std::vector<int32_t> perm(p - 1), ginv(p - 1);
    size_t v = 1;
    for (size_t m = 0; m < p - 1; m++) {
        perm[m] = (int32_t)v;
        v = (v * g) % p;
    }
    // g^-1 = g^(p-2)
    size_t gi = 1;
    for (size_t m = 0; m < p - 2; m++) gi = (gi * g) % p;
    v = 1;
    for (size_t m = 0; m < p - 1; m++) {
        ginv[m] = (int32_t)v;
        v = (v * gi) % p;
    }
    HostTable tp;
    tp.is_int = true;
    tp.i = perm;
    rt.perm = add_table(prog, kp, std::move(tp));
    HostTable ti;
    ti.is_int = true;
    ti.i = ginv;
    rt.ginv = add_table(prog, ki, std::move(ti));
    if (prog.is_dd) {
        std::vector<QC> b(p - 1);
        for (size_t m = 0; m < p - 1; m++) b[m] = root_q((size_t)ginv[m], p);
        if (fft_mode) host_fft_q(b);
        const q128 s = fft_mode ? (q128)1 / (q128)(p - 1) : (q128)1;
        HostTable tk;
        for (size_t m = 0; m < p - 1; m++) put_q(tk, m, QC{b[m].re * s, b[m].im * s});
        rt.kernel = add_table(prog, kk, std::move(tk));
        return rt;
    }
    std::vector<std::complex<double>> b(p - 1);
    for (size_t m = 0; m < p - 1; m++) b[m] = root((size_t)ginv[m], p);
    if (fft_mode) {
        host_fft_inplace(b, false);
        double s = 1.0 / (double)(p - 1);
        for (auto &x : b) x *= s;
    }
    HostTable tk;
    tk.c = std::move(b);
    rt.kernel = add_table(prog, kk, std::move(tk));
    return rt;
}

// ---- radix schedules ----------------------------------------------------------

// Radix stages for a {2,3,5,7,11,13}-smooth length (the B200 kernel's own choice;
// only the algorithm family is contractual).
std::vector<int> radix_schedule(size_t L) {
    std::vector<int> st;
    if (L <= 1) return st;
    size_t e2 = 0, e3 = 0, rem = L;
    while (rem % 2 == 0) rem /= 2, e2++;
    while (rem % 3 == 0) rem /= 3, e3++;
    while (e2 >= 4) st.push_back(16), e2 -= 4;
    while (e3 >= 2) st.push_back(9), e3 -= 2;
    if (e2 == 3) {
        st.push_back(8);
    } else if (e2 == 2) {
        if (e3) {
            st.push_back(12);
            e3--;
        } else {
            st.push_back(4);
        }
    } else if (e2 == 1) {
        if (e3) {
            st.push_back(6);
            e3--;
        } else if (rem % 5 == 0) {
            st.push_back(10);
            rem /= 5;
        } else {
            st.push_back(2);
        }
    }
    if (e3) st.push_back(3);
    for (int p : {5, 7, 11, 13})
        while (rem % p == 0) st.push_back(p), rem /= p;
    if (rem != 1) fail_invalid_ir("radix schedule requested for a non-smooth length");
    return st;
}

static bool is_kernel_smooth(size_t L) {
    for (size_t p : {2, 3, 5, 7, 11, 13})
        while (L % p == 0) L /= p;
    return L == 1;
}

// ---- one pass --------------------------------------------------------------------

static int odd_stride(int len_with_pad) { return len_with_pad | 1; }
static int spad_h(int e) { return e + (e >> 4); }
static int line_stride_for(int L) { return odd_stride(spad_h(L) + 1); }

struct StageSpec {
    int radix;
    bool rader = false;
    bool direct = false;
    size_t generator = 0;
    std::vector<StageSpec> sub;  // FFT-convolution Rader: stages of the (p-1)-point sub-transform
    bool ok = true;              // false when some factor has no kernel (nested Bluestein)
};

static const PlannerTuning *g_tuning = nullptr;  // tuning of the axis being lowered

// Stages of a line of length L for an axis algorithm: Stockham radices first, then one
// Rader stage per Rader prime occurrence.  An FFT-convolution Rader prime p carries the
// stages of its (p-1)-point convolution, planned with the axis tuning (the recursive
// tuning can make that convolution Rader again, planner.rs:512-529).
std::vector<StageSpec> line_stages(size_t L, const AxisAlgorithm *alg) {
    std::vector<StageSpec> out;
    size_t smooth = L;
    std::vector<StageSpec> rader;
    if (alg && alg->kind == AlgorithmKind::Rader) {
        for (auto &rp : alg->primes) {
            for (size_t k = 0; k < rp.multiplicity; k++) {
                StageSpec s;
                s.radix = (int)rp.prime;
                s.rader = true;
                s.direct = !rp.fft_convolution;
                s.generator = rp.generator;
                if (!s.direct) {
                    const PlannerTuning t = g_tuning ? *g_tuning : PlannerTuning::portable();
                    AxisAlgorithm nested = plan_axis_algorithm(rp.prime - 1, t);
                    if (nested.kind == AlgorithmKind::Bluestein) {
                        s.ok = false;
                    } else {
                        s.sub = line_stages(rp.prime - 1, &nested);
                        for (auto &x : s.sub) s.ok = s.ok && x.ok;
                    }
                }
                rader.push_back(s);
                smooth /= rp.prime;
            }
        }
    }
    if (!is_kernel_smooth(smooth)) {
        StageSpec bad;
        bad.radix = 0;
        bad.ok = false;
        out.push_back(bad);
        return out;
    }
    for (int r : radix_schedule(smooth)) out.push_back(StageSpec{r});
    for (auto &s : rader) out.push_back(s);
    return out;
}

static bool stages_ok(const std::vector<StageSpec> &st) {
    for (auto &s : st)
        if (!s.ok) return false;
    return true;
}

// Extra shared memory (complex elements) of the Rader stages of a stage list applied to
// nsub sub-lines of length L whose line regions have stride ls.  A Rader stage gathers
// from the current buffer into W, which reuses the free ping-pong partner when it fits,
// runs its sub-transform between W and W2, and scatters back into the current buffer.
// Stages at one level run one after another, so they share the same region.
static size_t rader_extra(size_t L, const std::vector<StageSpec> &stages, size_t nsub, size_t ls) {
    size_t best = 0;
    for (auto &st : stages) {
        if (!st.rader) continue;
        const size_t p = (size_t)st.radix;
        const size_t nb = nsub * (L / p);
        const size_t ws = (size_t)line_stride_for((int)(p - 1));
        const bool w_in_partner = nb * ws <= nsub * ls;
        size_t need = 2 * nb;  // X0 pairs
        if (!st.direct) {
            need += nb * ws;  // W2
            need += rader_extra(p - 1, st.sub, nb, ws);
        }
        if (!w_in_partner) need += nb * ws;
        best = std::max(best, need);
    }
    return best;
}

struct CtaShape {
    int G = 1, threads = 64, ls = 1;
    size_t extra = 0;  // Rader region elements
    size_t smem = 0, meta_off = 0;
};

static size_t budget_bytes() { return 200 * 1024; }

// Choose lines per CTA, threads and shared-memory layout.  Returns false when one
// line does not fit on chip.
static bool shape_pass(int ce, int L, const std::vector<StageSpec> &stages, bool strided, int64_t nlines,
                       int nops, CtaShape &sh) {
    if (!stages_ok(stages)) return false;
    const size_t esz = (size_t)ce;  // bytes of one complex element (8 f32, 16 f64, 32 dd)
    sh.ls = line_stride_for(L);
    auto data_for = [&](int G) {
        size_t data = (2 * (size_t)G * sh.ls + rader_extra((size_t)L, stages, (size_t)G, (size_t)sh.ls)) * esz;
        return (data + 15) & ~size_t(15);
    };
    auto bytes_for = [&](int G) {
        size_t meta = (size_t)G * 16 + (size_t)((G + 3) & ~3) * 8;
        meta = (meta + 15) & ~size_t(15);
        return data_for(G) + meta + (size_t)nops * sizeof(Op);
    };
    const int gmin = strided ? (ce >= 16 ? 4 : 8) : 1;
    int G = std::max(gmin, (int)((2048 + L - 1) / L));
    if (!strided) G = std::min<int64_t>(G, std::max<int64_t>(nlines, 1));
    const size_t soft = 96 * 1024;
    while (G > gmin && bytes_for(G) > soft) G--;
    while (G > 1 && bytes_for(G) > budget_bytes()) G--;
    if (bytes_for(G) > budget_bytes()) return false;
    sh.G = G;
    sh.extra = rader_extra((size_t)L, stages, (size_t)G, (size_t)sh.ls);
    sh.meta_off = data_for(G);
    sh.smem = bytes_for(G);
    const int maxt = ce == 8 ? 1024 : (ce == 16 ? 512 : 256);  // the pass kernel variants
    int64_t work = (int64_t)G * L / 8;
    int t = (int)std::min<int64_t>(std::max<int64_t>(work, 64), maxt);
    sh.threads = (t + 31) / 32 * 32;
    return true;
}

// Shared-memory capacity only (for passes without an FFT network, e.g. real pre/post).
static bool line_capacity_ok(int ce, size_t L) {
    if (L > (1u << 20)) return false;
    CtaShape sh;
    return shape_pass(ce, (int)L, {}, false, 1 << 20, 8, sh);
}

bool line_fits_on_chip(int ce, size_t L, const AxisAlgorithm *alg, bool strided) {
    if (L > (1u << 20)) return false;
    CtaShape sh;
    return shape_pass(ce, (int)L, line_stages(L, alg), strided, 1 << 20, kMaxOps, sh);
}

// ---- shared-memory layout choice ------------------------------------------------------
// Wavefronts of one warp access to 8-byte (complex f32) or 16-byte slots: the largest
// number of distinct 4-byte rows any bank is asked for.
static int bank_wavefronts(const int *slot, int n, int words) {
    int rows[32][16];
    int cnt[32] = {};
    int worst = 0;
    for (int i = 0; i < n; i++)
        for (int w = 0; w < words; w++) {
            const int word = slot[i] * words + w, bank = word & 31, row = word >> 5;
            bool seen = false;
            for (int k = 0; k < cnt[bank]; k++) seen |= rows[bank][k] == row;
            if (!seen && cnt[bank] < 16) rows[bank][cnt[bank]++] = row;
            worst = std::max(worst, cnt[bank]);
        }
    return worst;
}

// Modelled shared-memory wavefronts of a Stockham-only pass (radix stages between the
// two line buffers, an element-fast and a line-fast load/store) for a padding shift and
// line stride: the same index arithmetic as op_stage / op_load / op_store, over the first
// warps of every access pattern.
static long smem_cost(const std::vector<StageSpec> &stages, int L, int G, int threads, int shift, int ls, int words) {
    auto spad = [&](int e) { return e + (e >> shift); };
    long cost = 0;
    int slot[32];
    int P = 1;
    const int kWarps = 24;
    for (const StageSpec &st : stages) {
        const int R = st.radix, NBL = L / R, NB = G * NBL;
        for (int w = 0; w < kWarps && w * 32 < NB; w++)
            for (int q = 0; q < R; q++) {
                int n = 0, m = 0, wslot[32];
                for (int l = 0; l < 32 && w * 32 + l < NB; l++, n++) {
                    const int b = w * 32 + l, s = b / NBL, bb = b - s * NBL, j = bb % P;
                    slot[n] = s * ls + spad(bb + q * NBL);
                    wslot[m++] = G * ls + s * ls + spad((bb - j) * R + j + q * P);
                }
                cost += bank_wavefronts(slot, n, words) + bank_wavefronts(wslot, m, words);
            }
        P *= R;
    }
    for (int pattern = 0; pattern < 2; pattern++)
        for (int w = 0; w < kWarps && w * 32 < G * L; w++) {
            int n = 0;
            for (int l = 0; l < 32 && w * 32 + l < G * L; l++, n++) {
                const int f = w * 32 + l;
                const int g = pattern ? f % G : f / L, e = pattern ? f / G : f % L;
                slot[n] = g * ls + spad(e);
            }
            cost += 2 * bank_wavefronts(slot, n, words);
        }
    (void)threads;
    return cost;
}

// Padding shift (4 or unpadded) and line stride of a pass: the current layout unless the
// model finds an unpadded one with fewer wavefronts that fits in the same stride budget.
// Passes with Rader stages keep the padded layout their region sizes assume.
static void choose_smem_layout(const std::vector<StageSpec> &stages, int L, int G, int threads, int words,
                               int &shift, int &ls) {
    shift = 4;
    for (const StageSpec &st : stages)
        if (st.rader || st.radix < 2 || L % st.radix) return;
    if (stages.empty()) return;
    const int ls0 = ls;
    long best = smem_cost(stages, L, G, threads, 4, ls0, words);
    // unpadded strides from L + 2 (ops address elements L and L + 1: the even-half post /
    // pre-processing and the saved DC slot) within the padded stride, 65 candidates at most
    for (int cand = L + 2; cand <= std::min(ls0, L + 66); cand++) {
        const long c = smem_cost(stages, L, G, threads, 31, cand, words);
        if (c < best) {
            best = c;
            shift = 31;
            ls = cand;
        }
    }
}

// Builds the op program of one pass.
class PassBuilder {
   public:
    PassBuilder(Program &prog, int L, std::vector<StageSpec> stages, bool strided, int64_t nlines, int nops_hint)
        : prog_(prog), L_(L), stages_(std::move(stages)) {
        if (!shape_pass(prog.cbytes(), L, stages_, strided, nlines, std::max(nops_hint, (int)kMaxOps), sh_))
            fail_resource("B200 FFT pass shared memory", (size_t)L * 2 * prog.cbytes(), budget_bytes());
        choose_smem_layout(stages_, L, sh_.G, sh_.threads, prog.cbytes() / 4, pad_shift_, sh_.ls);
        A_ = 0;
        B_ = sh_.G * sh_.ls;
        extra_base_ = 2 * sh_.G * sh_.ls;
        cur_ = A_;
        other_ = B_;
        for (auto &row : plan_.op_tables) row[0] = row[1] = row[2] = -1;
    }
    int G() const { return sh_.G; }

    Op &push(int type) {
        if (nops_ >= kMaxOps) fail_invalid_ir("pass op program exceeds the kernel's op capacity");
        Op &o = plan_.p.ops[nops_++];
        std::memset(&o, 0, sizeof(Op));
        o.type = type;
        o.pad_shift = pad_shift_;
        return o;
    }
    void set_tables(int a, int b = -1, int c = -1) {
        plan_.op_tables[nops_ - 1][0] = a;
        plan_.op_tables[nops_ - 1][1] = b;
        plan_.op_tables[nops_ - 1][2] = c;
    }

    // global -> line region A.  own_em > 0: the table index of the multiply is e*own_em
    // (instead of the side's logical index).
    void load(int len, int flags, int mul = MUL_NONE, int table = -1, double scale = 1.0, int own_em = 0,
              int own_cm = 0) {
        Op &o = push(OP_LOAD);
        o.len = len;
        o.flags = flags | (own_em ? F_OWN_INDEX : 0);
        o.em = own_em;
        o.cm = own_cm;
        o.mul = mul;
        o.dst_base = A_;
        o.sub_stride = sh_.ls;
        o.scale = scale;
        o.div_a = make_fastdiv((uint32_t)len);
        set_tables(table);
        cur_ = A_;
        other_ = B_;
    }

    // the full FFT network of the line (length L_) on the current region
    void fft() { emit_stages((size_t)L_, stages_, (size_t)sh_.G, sh_.ls, cur_, other_, extra_base_); }

    void mul_region(int table, int flags, int cm, int em, int count = 0, int64_t om = 0, int64_t lut_off = 0) {
        Op &o = push(OP_MUL);
        o.om = om;
        o.lut_off = lut_off;
        o.nfull = count;
        o.len = L_;
        o.nsub = sh_.G;
        o.src_base = cur_;
        o.sub_stride = sh_.ls;
        o.mul = MUL_LUT_N;
        o.cm = cm;
        o.em = em;
        // a table indexed line-fastest (cm = 1) is read coalesced when threads walk lines
        o.flags = flags | (cm == 1 && em > 1 ? F_LINE_FAST : 0);
        o.div_a = make_fastdiv((uint32_t)L_);
        o.div_b = make_fastdiv((uint32_t)sh_.G);
        set_tables(table);
    }

    void herm_expand(int n) {
        Op &o = push(OP_HERM_EXPAND);
        o.src_base = cur_;
        o.sub_stride = sh_.ls;
        o.nfull = n;
    }

    void r2c_post(int h, int wn_table) {
        Op &o = push(OP_R2C_POST);
        o.len = h;
        o.src_base = cur_;
        o.sub_stride = sh_.ls;
        o.nfull = 2 * h;
        set_tables(-1, wn_table);
    }

    void c2r_pre(int h, int wn_table, int flags, double scale) {
        Op &o = push(OP_C2R_PRE);
        o.len = h;
        o.src_base = cur_;
        o.sub_stride = sh_.ls;
        o.nfull = 2 * h;
        o.flags = flags;
        o.scale = scale;
        set_tables(-1, wn_table);
    }

    // Rader pass-level permutations (rader_ir.rs gather / scatter dispatches): see
    // OP_PERMUTE_GATHER / OP_PERMUTE_SCATTER in pass_desc.hpp.
    void permute_gather(int p, int perm_table) {
        Op &o = push(OP_PERMUTE_GATHER);
        o.radix = p;
        o.nsub = sh_.G;
        o.src_base = cur_;
        o.dst_base = other_;
        o.sub_stride = sh_.ls;
        o.div_c = make_fastdiv((uint32_t)(p + 1));
        set_tables(-1, perm_table);
        std::swap(cur_, other_);
    }
    void permute_scatter(int p, int ginv_table, int flags, double scale) {
        Op &o = push(OP_PERMUTE_SCATTER);
        o.radix = p;
        o.nsub = sh_.G;
        o.src_base = cur_;
        o.dst_base = other_;
        o.sub_stride = sh_.ls;
        o.flags = flags;
        o.scale = scale;
        o.div_c = make_fastdiv((uint32_t)p);
        set_tables(-1, -1, ginv_table);
        std::swap(cur_, other_);
    }
    void save_dc(int slot) {
        Op &o = push(OP_SAVE_DC);
        o.nsub = sh_.G;
        o.src_base = cur_;
        o.sub_stride = sh_.ls;
        o.nfull = slot;
    }

    void store(int len, int flags, int mul = MUL_NONE, int table = -1, double scale = 1.0, int own_em = 0,
               int own_cm = 0) {
        Op &o = push(OP_STORE);
        o.len = len;
        o.flags = flags | (own_em ? F_OWN_INDEX : 0);
        o.em = own_em;
        o.cm = own_cm;
        o.mul = mul;
        o.src_base = cur_;
        o.sub_stride = sh_.ls;
        o.scale = scale;
        o.div_a = make_fastdiv((uint32_t)len);
        set_tables(table);
    }

    PassPlan finish(int64_t no, int64_t ni, int64_t nc, const Side &in, const Side &out, int src_buf, int64_t src_off,
                    int dst_buf, int64_t dst_off, const std::string &label) {
        PassParams &p = plan_.p;
        p.nlines = no * ni * nc;
        p.ni = ni;
        p.nc = nc;
        p.G = sh_.G;
        p.div_g = make_fastdiv((uint32_t)sh_.G);
        p.nops = nops_;
        p.line_len = L_;
        p.line_stride = sh_.ls;
        p.meta_off = (int32_t)sh_.meta_off;
        p.in = in;
        p.out = out;
        plan_.src_buf = src_buf;
        plan_.src_off = src_off;
        plan_.dst_buf = dst_buf;
        plan_.dst_off = dst_off;
        plan_.grid = (p.nlines + sh_.G - 1) / sh_.G;
        plan_.threads = sh_.threads;
        // shared memory = data regions + per-line metadata + the op program actually emitted
        size_t meta = (size_t)sh_.G * 16 + (size_t)((sh_.G + 3) & ~3) * 8;
        meta = (meta + 15) & ~size_t(15);
        plan_.smem = sh_.meta_off + meta + (size_t)nops_ * sizeof(Op);
        if (plan_.smem > 232448) fail_resource("B200 FFT pass shared memory", plan_.smem, 232448);
        plan_.label = label;
        return plan_;
    }

   private:
    // Stages of a transform of length L on nsub sub-lines (stride ls) held in region cur;
    // other is its free partner, extra the first free element for Rader work regions.
    // On return cur holds the result.
    void emit_stages(size_t L, const std::vector<StageSpec> &stages, size_t nsub, int ls, int &cur, int &other,
                     size_t extra) {
        const int tw = table_twiddle(prog_, L);
        int P = 1;
        for (auto &st : stages) {
            if (!st.rader) {
                Op &o = push(OP_STAGE);
                o.radix = st.radix;
                o.P = P;
                o.len = (int)L;
                o.nsub = (int)nsub;
                o.src_base = cur;
                o.dst_base = other;
                o.sub_stride = ls;
                o.div_a = make_fastdiv((uint32_t)(L / st.radix));
                o.div_b = make_fastdiv((uint32_t)P);
                set_tables(P > 1 ? table_stage_twiddles(prog_, (size_t)st.radix, (size_t)P) : -1);
                std::swap(cur, other);
            } else {
                emit_rader(st, L, nsub, ls, P, tw, cur, other, extra);
            }
            P *= st.radix;
        }
    }

    void emit_rader(const StageSpec &st, size_t L, size_t nsub, int ls, int P, int tw, int cur, int other,
                    size_t extra) {
        const int p = st.radix;
        const size_t nb = nsub * (L / p);
        const int ws = line_stride_for(p - 1);
        const bool w_in_partner = nb * (size_t)ws <= nsub * (size_t)ls;
        size_t at = extra;
        const int W = w_in_partner ? other : (int)at;
        if (!w_in_partner) at += nb * ws;
        int W2 = 0;
        if (!st.direct) {
            W2 = (int)at;
            at += nb * ws;
        }
        const int X0 = (int)at;
        at += 2 * nb;
        RaderTables rt = table_rader(prog_, (size_t)p, st.generator, !st.direct);
        {
            Op &o = push(OP_RADER_GATHER);
            o.radix = p;
            o.P = P;
            o.len = (int)L;
            o.nsub = (int)nsub;
            o.src_base = cur;
            o.sub_stride = ls;
            o.w_base = W;
            o.w_stride = ws;
            o.x0_base = X0;
            o.div_a = make_fastdiv((uint32_t)(L / p));
            o.div_b = make_fastdiv((uint32_t)P);
            o.div_c = make_fastdiv((uint32_t)p);
            set_tables(tw, rt.perm);
        }
        int wcur = W;
        if (!st.direct) {
            int wother = W2;
            emit_stages((size_t)(p - 1), st.sub, nb, ws, wcur, wother, at);
            {
                Op &o = push(OP_MUL);
                o.len = p - 1;
                o.nsub = (int)nb;
                o.src_base = wcur;
                o.sub_stride = ws;
                o.mul = MUL_LUT_N;
                o.cm = 0;
                o.em = 1;
                o.x0_base = X0;
                o.flags = F_SAVE_DC | F_CONJ_OUT;
                o.div_a = make_fastdiv((uint32_t)(p - 1));
                set_tables(rt.kernel);
            }
            emit_stages((size_t)(p - 1), st.sub, nb, ws, wcur, wother, at);
        }
        {
            Op &o = push(OP_RADER_SCATTER);
            o.radix = p;
            o.P = P;
            o.len = (int)L;
            o.nsub = (int)nsub;
            o.dst_base = cur;  // the gathered line buffer is free again
            o.sub_stride = ls;
            o.w_base = wcur;
            o.w_stride = ws;
            o.x0_base = X0;
            o.flags = st.direct ? F_DIRECT : F_CONJ_IN;
            o.div_a = make_fastdiv((uint32_t)(L / p));
            o.div_b = make_fastdiv((uint32_t)P);
            o.div_c = make_fastdiv((uint32_t)p);
            set_tables(rt.kernel, -1, rt.ginv);
        }
    }

    Program &prog_;
    int L_;
    std::vector<StageSpec> stages_;
    CtaShape sh_;
    int pad_shift_ = 4;  // shared-memory padding of the pass (choose_smem_layout)
    PassPlan plan_{};
    int nops_ = 0;
    int A_, B_, cur_, other_;
    size_t extra_base_;
};

static Side make_side(int64_t os, int64_t is, int64_t cs, int64_t es, bool real, int64_t count, int cm, int em,
                      int herm = 0) {
    Side s{};
    s.os = os;
    s.is = is;
    s.cs = cs;
    s.es = es;
    s.real = real ? 1 : 0;
    s.count = (int32_t)std::min<int64_t>(count, INT32_MAX);
    s.cm = cm;
    s.em = em;
    s.herm = herm;
    return s;
}

// ---- axis lowering ----------------------------------------------------------------

// The part of an axis algorithm that applies to a factor n of the axis: the Rader
// primes dividing n (with the multiplicity they have in n), Stockham otherwise.
static AxisAlgorithm restrict_algorithm(const AxisAlgorithm &alg, size_t n) {
    AxisAlgorithm r;
    r.kind = AlgorithmKind::Stockham;
    if (alg.kind != AlgorithmKind::Rader) return r;
    for (const RaderPrimePlan &rp : alg.primes) {
        size_t m = 0, v = n;
        while (v % rp.prime == 0) v /= rp.prime, m++;
        if (!m) continue;
        RaderPrimePlan c = rp;
        c.multiplicity = std::min(m, rp.multiplicity);
        r.primes.push_back(c);
        r.kind = AlgorithmKind::Rader;
    }
    return r;
}

// Four-step split N = N1 (columns, strided) x N2 (rows) with both factors executable in
// one CTA; the most balanced such split.
static bool four_step_split(int ce, size_t N, const AxisAlgorithm &alg, size_t &N1, size_t &N2) {
    size_t best = 0;
    double best_score = 1e300;
    for (size_t d = 2; d * d <= N; d++) {
        if (N % d) continue;
        for (int flip = 0; flip < 2; flip++) {
            const size_t a = flip ? N / d : d, b = N / a;
            AxisAlgorithm ra = restrict_algorithm(alg, a), rb = restrict_algorithm(alg, b);
            if (!line_fits_on_chip(ce, a, &ra, true) || !line_fits_on_chip(ce, b, &rb, true)) continue;
            const double score = std::fabs(std::log((double)a) - std::log((double)b)) + (flip ? 1e-9 : 0);
            if (score < best_score) {
                best_score = score;
                best = a;
            }
        }
    }
    if (!best) return false;
    N1 = best;
    N2 = N / best;
    return true;
}

static size_t small_prime_part(size_t n) {
    size_t a = 1;
    for (size_t p : {2, 3, 5, 7, 11, 13})
        while (n % p == 0) n /= p, a *= p;
    return a;
}

// The register kernels are not part of the CPU emulation build (their threads
// exchange data inside one op); B200FFT_DISABLE_REG=1 forces the generic pass kernel.
static bool reg_kernels_enabled() {
#ifdef B200FFT_EMULATE
    return false;
#else
    const char *e = std::getenv("B200FFT_DISABLE_REG");
    return !(e && e[0] == '1');
#endif
}

// Register-kernel variant for the program's precision (none for double-double: its
// 32-byte points do not fit the register budget of the register-resident kernels).
static int reg_variant(const Program &prog, size_t n, int mode, bool strided) {
    if (prog.is_dd) return -1;
    return reg_variant_for(prog.is_double, n, mode, strided);
}

void lower_c2c_axis(Program &prog, const AxisJob &job) {
    const PlannerTuning *saved_tuning = g_tuning;
    g_tuning = &job.tuning;
    struct Restore {
        const PlannerTuning *t;
        ~Restore() { g_tuning = t; }
    } restore{saved_tuning};
    const bool dbl = prog.is_double;
    const int ce = prog.cbytes();
    const bool inv = job.inverse;
    const size_t N = job.N;
    const AxisAlgorithm *alg = job.alg;
    const int64_t no = job.no, S = job.S;
    const int64_t So = job.out_S ? job.out_S : S;  // output element stride
    const bool strided = S > 1;
    // inverse = conj(forward(conj(x))): conjugate the raw input before any multiply of
    // the first load and the final value after every multiply of the last store
    const int cin = inv ? F_CONJ_IN : 0;
    const int cout = inv ? F_CONJ_OUT : 0;
    const double scale = job.scale;
    const int fscale = scale != 1.0 ? F_SCALE : 0;
    const size_t out_count = job.out_count ? job.out_count : N;
    const int herm = job.in_herm ? (int)N : 0;

    if (N == 1) {
        PassBuilder b(prog, 1, {}, strided, no * S, 4);
        b.load(1, cin);
        b.store(1, cout | fscale, MUL_NONE, -1, scale);
        prog.passes.push_back(b.finish(no, S, 1, make_side(job.in_os, 1, 0, S, job.in_real, 1, 0, 1),
                                       make_side(job.out_os, 1, 0, So, job.out_real, 1, 0, 1), job.in_buf, job.in_off,
                                       job.out_buf, job.out_off, "copy"));
        return;
    }

    // Fast path: power-of-two Stockham lines run in the register-resident kernels
    // (one global read and write, shared memory only between the middle stages).
    if (alg->kind == AlgorithmKind::Stockham && is_pow2(N) && reg_kernels_enabled()) {
        int mode = -1;
        if (!job.in_real && !job.in_herm && !job.out_real && out_count == N)
            mode = REG_C2C;
        else if (job.in_real && !job.out_real && out_count == N / 2 + 1 && !strided)
            mode = REG_R2C_FULL;
        else if (job.in_herm && job.out_real && out_count == N && !strided)
            mode = REG_C2R_FULL;
        const int rv = mode >= 0 ? reg_variant(prog, N, mode, strided) : -1;
        if (rv >= 0) {
            PassPlan pp{};
            pp.kernel = KERNEL_REG;
            pp.reg_variant = rv;
            pp.reg_table = table_reg_twiddles(prog, N, rv);
            pp.rp.nlines = no * S;
            pp.rp.ni = S;
            pp.rp.src = RegSide{job.in_os, strided ? 1 : 0, S};
            pp.rp.dst = RegSide{job.out_os, strided ? 1 : 0, So};
            pp.rp.scale = scale;
            pp.rp.conj = (mode == REG_C2C && inv) ? 1 : 0;
            pp.rp.n = (int32_t)N;
            pp.reg_in_real = mode == REG_R2C_FULL;
            pp.reg_out_real = mode == REG_C2R_FULL;
            pp.src_buf = job.in_buf;
            pp.src_off = job.in_off;
            pp.dst_buf = job.out_buf;
            pp.dst_off = job.out_off;
            pp.label = "register stockham";
            // dense contiguous lines: the persistent variant prefetches each CTA's next
            // line group with a bulk copy while the current one is transformed
            if (mode == REG_C2C && !strided && job.in_os == (int64_t)N && job.in_off == 0) {
                const int pv = reg_variant_persistent_twin(rv);
                if (pv >= 0) {
                    pp.reg_variant_plain = rv;
                    pp.reg_variant = pv;
                    pp.label = "register stockham (bulk prefetch)";
                }
            }
            for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
            prog.passes.push_back(pp);
            return;
        }
    }

    // Strided prime lines whose Rader convolution is one codelet FFT: one thread per
    // line, Rader's algorithm in registers (reg_rader_kernel)
    if (alg->kind == AlgorithmKind::Rader && strided && reg_kernels_enabled() && !job.in_real && !job.in_herm &&
        !job.out_real && out_count == N && alg->primes.size() == 1 && alg->primes[0].prime == N) {
        const int rv = reg_variant(prog, N, REG_RADER_LINE, true);
        if (rv >= 0) {
            PassPlan pp{};
            pp.kernel = KERNEL_REG;
            pp.reg_variant = rv;
            pp.reg_table = table_rader_line(prog, N);
            pp.rp.nlines = no * S;
            pp.rp.ni = S;
            pp.rp.src = RegSide{job.in_os, 1, S};
            pp.rp.dst = RegSide{job.out_os, 1, So};
            pp.rp.scale = scale;
            pp.rp.conj = inv ? 1 : 0;
            pp.rp.n = (int32_t)N;
            pp.src_buf = job.in_buf;
            pp.src_off = job.in_off;
            pp.dst_buf = job.out_buf;
            pp.dst_off = job.out_off;
            pp.label = "register rader line";
            for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
            prog.passes.push_back(pp);
            return;
        }
    }

    const Side in_line = make_side(job.in_os, 1, 0, S, job.in_real, N, 0, 1, herm);
    const Side out_line = make_side(job.out_os, 1, 0, So, job.out_real, out_count, 0, 1);

    if (alg->kind != AlgorithmKind::Bluestein) {
        // one pass: Stockham radices and Rader stages (nested when the convolution is
        // itself Rader) on chip
        if (line_fits_on_chip(ce, N, alg, strided)) {
            PassBuilder b(prog, (int)N, line_stages(N, alg), strided, no * S, kMaxOps);
            b.load((int)N, cin);
            b.fft();
            b.store((int)out_count, cout | fscale, MUL_NONE, -1, scale);
            prog.passes.push_back(b.finish(no, S, 1, in_line, out_line, job.in_buf, job.in_off, job.out_buf,
                                           job.out_off, alg->kind == AlgorithmKind::Rader ? "rader" : "stockham"));
            return;
        }
        // four-step through scratch 0: columns (N1, stride N2) with the twiddle W_N^{n2 k1}
        // fused into their store, then rows (N2) with the transposed store
        size_t N1, N2;
        if (four_step_split(ce, N, *alg, N1, N2)) {
            const AxisAlgorithm a1 = restrict_algorithm(*alg, N1), a2 = restrict_algorithm(*alg, N2);
            const int64_t scr_os = (int64_t)N * S;
            prog.scratch_elems[0] = std::max(prog.scratch_elems[0], (size_t)(no * N * S));
            {
                PassBuilder b(prog, (int)N1, line_stages(N1, &a1), true, no * S * N2, kMaxOps);
                b.load((int)N1, cin);
                b.fft();
                b.store((int)N1, 0, MUL_TWIDDLE_CE, table_twiddle_transposed(prog, N2, N1, N), 1.0, (int)N2, 1);
                prog.passes.push_back(b.finish(
                    no, S, (int64_t)N2, make_side(job.in_os, 1, S, (int64_t)N2 * S, job.in_real, N, 1, (int)N2, herm),
                    make_side(scr_os, 1, S, (int64_t)N2 * S, false, N, 1, (int)N2), job.in_buf, job.in_off,
                    BUF_SCRATCH0, 0, "four-step columns"));
            }
            {
                PassBuilder b(prog, (int)N2, line_stages(N2, &a2), true, no * S * N1, kMaxOps);
                b.load((int)N2, 0);
                b.fft();
                b.store((int)N2, cout | fscale, MUL_NONE, -1, scale);
                prog.passes.push_back(
                    b.finish(no, S, (int64_t)N1, make_side(scr_os, 1, (int64_t)N2 * S, S, false, N, (int)N2, 1),
                             make_side(job.out_os, 1, So, (int64_t)N1 * So, job.out_real, out_count, 1, (int)N1),
                             BUF_SCRATCH0, 0, job.out_buf, job.out_off, "four-step rows"));
            }
            return;
        }
        // pass-level Rader for a prime axis whose convolution does not fit one CTA
        // (rader_ir.rs:706-1957: gather -> FFT(p-1) -> multiply -> FFT(p-1) -> scatter)
        if (alg->kind == AlgorithmKind::Rader && alg->primes.size() == 1 && alg->primes[0].prime == N &&
            alg->primes[0].fft_convolution && !job.in_nested_rader) {
            const size_t p = N;
            const RaderPrimePlan &rp = alg->primes[0];
            RaderTables rt = table_rader(prog, p, rp.generator, true);
            const AxisAlgorithm nested = plan_axis_algorithm(p - 1, job.tuning);
            const int64_t Ls = (int64_t)(p + 1);  // [a_0 .. a_{p-2}, x0, A0]
            const int64_t scr_os = Ls * S;
            prog.scratch_elems[3] = std::max(prog.scratch_elems[3], (size_t)(no * Ls * S));
            const Side scr_line = make_side(scr_os, 1, 0, S, false, Ls, 0, 1);
            {
                PassBuilder b(prog, (int)Ls, {}, strided, no * S, 4);
                b.load((int)p, cin);
                b.permute_gather((int)p, rt.perm);
                b.store((int)p, 0);
                prog.passes.push_back(b.finish(no, S, 1, in_line, scr_line, job.in_buf, job.in_off, BUF_SCRATCH3, 0,
                                               "rader gather"));
            }
            AxisJob sub;
            sub.N = p - 1;
            sub.alg = &nested;
            sub.tuning = job.tuning;
            sub.no = no;
            sub.S = S;
            sub.in_buf = sub.out_buf = BUF_SCRATCH3;
            sub.in_os = sub.out_os = scr_os;
            sub.in_nested_rader = true;
            lower_c2c_axis(prog, sub);
            {
                PassBuilder b(prog, (int)Ls, {}, strided, no * S, 4);
                b.load((int)Ls, 0);
                b.save_dc((int)p);
                b.mul_region(rt.kernel, F_CONJ_OUT, 0, 1, (int)(p - 1));
                b.store((int)Ls, 0);
                prog.passes.push_back(
                    b.finish(no, S, 1, scr_line, scr_line, BUF_SCRATCH3, 0, BUF_SCRATCH3, 0, "rader multiply"));
            }
            lower_c2c_axis(prog, sub);
            {
                PassBuilder b(prog, (int)Ls, {}, strided, no * S, 4);
                b.load((int)Ls, 0);
                b.permute_scatter((int)p, rt.ginv, F_CONJ_IN | cout | fscale, scale);
                b.store((int)out_count, 0);
                prog.passes.push_back(b.finish(no, S, 1, scr_line, out_line, BUF_SCRATCH3, 0, job.out_buf,
                                               job.out_off, "rader scatter"));
            }
            return;
        }
        fail_unsupported("B200 engine: axis too large for one CTA and not four-step decomposable");
    }

    // Bluestein (bluestein_ir.rs:436-933): chirp, zero-pad to M, FFT_M, x spectrum, IFFT_M,
    // chirp and take N.  With the conjugation trick the inverse uses the forward chirp.
    const size_t M = alg->convolution_len;
    const int chirp = table_bluestein_chirp(prog, N);
    if (line_fits_on_chip(ce, M, nullptr, strided)) {
        const int spec = table_bluestein_spectrum(prog, N, M);
        PassBuilder b(prog, (int)M, line_stages(M, nullptr), strided, no * S, kMaxOps);
        b.load((int)M, cin, MUL_LUT_N, chirp);
        b.fft();
        b.mul_region(spec, F_CONJ_OUT, 0, 1);
        b.fft();
        // store: conj (undo the inner inverse trick), multiply chirp, conj again if inverse
        b.store((int)out_count, F_CONJ_IN | cout | fscale, MUL_LUT_N, chirp, scale);
        prog.passes.push_back(b.finish(no, S, 1, in_line, out_line, job.in_buf, job.in_off, job.out_buf, job.out_off,
                                       "bluestein fused"));
        return;
    }
    // f64: when N has small prime factors A (B = N / A), the reference's CPU path splits
    // them off first and runs Bluestein on B only (reference.rs:60-75); its unreduced-chirp
    // error is then that of B.  Mirror that structure so the f64 result stays within 1e-13
    // of it: columns = Bluestein(B) with chirp(B) and the four-step twiddle, rows = FFT(A).
    const size_t A = small_prime_part(N), B = N / A;
    if (dbl && A > 1 && B > 1) {
        const size_t MB = next_smooth_at_least(2 * B - 1, {2, 3, 5, 7});
        if (line_fits_on_chip(ce, MB, nullptr, true) && line_fits_on_chip(ce, A, nullptr, true)) {
            const int chirpB = table_bluestein_chirp(prog, B);
            const int specB = table_bluestein_spectrum(prog, B, MB);
            const int64_t scr_os = (int64_t)N * S;
            prog.scratch_elems[0] = std::max(prog.scratch_elems[0], (size_t)(no * N * S));
            {
                PassBuilder b(prog, (int)MB, line_stages(MB, nullptr), true, no * S * A, kMaxOps);
                b.load((int)MB, cin, MUL_LUT_N, chirpB, 1.0, 1);
                b.fft();
                b.mul_region(specB, F_CONJ_OUT, 0, 1);
                b.fft();
                b.mul_region(chirpB, F_CONJ_IN, 0, 1, (int)B);
                b.store((int)B, 0, MUL_TWIDDLE_CE, table_twiddle_transposed(prog, A, B, N), 1.0, (int)A, 1);
                prog.passes.push_back(b.finish(
                    no, S, (int64_t)A, make_side(job.in_os, 1, S, (int64_t)A * S, job.in_real, N, 1, (int)A, herm),
                    make_side(scr_os, 1, S, (int64_t)A * S, false, N, 1, (int)A), job.in_buf, job.in_off,
                    BUF_SCRATCH0, 0, "bluestein(B) columns"));
            }
            {
                PassBuilder b(prog, (int)A, line_stages(A, nullptr), true, no * S * B, kMaxOps);
                b.load((int)A, 0);
                b.fft();
                b.store((int)A, cout | fscale, MUL_NONE, -1, scale);
                prog.passes.push_back(
                    b.finish(no, S, (int64_t)B, make_side(scr_os, 1, (int64_t)A * S, S, false, N, (int)A, 1),
                             make_side(job.out_os, 1, So, (int64_t)B * So, job.out_real, out_count, 1, (int)B),
                             BUF_SCRATCH0, 0, job.out_buf, job.out_off, "small-prime rows"));
            }
            return;
        }
    }
    size_t M1, M2;
    AxisAlgorithm smooth;
    if (!four_step_split(ce, M, smooth, M1, M2)) fail_unsupported("B200 engine: Bluestein length not decomposable");
    const int64_t scr_os = (int64_t)M * S;
    prog.scratch_elems[0] = std::max(prog.scratch_elems[0], (size_t)(no * M * S));
    // contiguous complex axis: the three passes in the register kernels (REG_BLU_A/B/C)
    {
        const int va = reg_variant(prog, M1, REG_BLU_A, true), vc = reg_variant(prog, M1, REG_BLU_C, true);
        if (S == 1 && So == 1 && va >= 0 && vc >= 0 && reg_kernels_enabled() && !job.in_real && !herm &&
            !job.out_real) {
            const int ttw = table_twiddle_transposed(prog, M2, M1, M);  // W_M^(n2 k1) at k1 M2 + n2
            auto reg_pass = [&](int rv, size_t len, int64_t nlines, int64_t ni, RegSide src, RegSide dst, int t2, int t3,
                                int64_t n, int in_buf, int64_t in_off, int out_buf, int64_t out_off, double sc,
                                const char *label) {
                PassPlan pp{};
                pp.kernel = KERNEL_REG;
                pp.reg_variant = rv;
                pp.reg_table = table_reg_twiddles(prog, len, rv);
                pp.reg_table2 = t2;
                pp.reg_table3 = t3;
                pp.rp.nlines = nlines;
                pp.rp.ni = ni;
                pp.rp.src = src;
                pp.rp.dst = dst;
                pp.rp.scale = sc;
                pp.rp.conj = inv ? 1 : 0;
                pp.rp.n = (int32_t)n;
                pp.src_buf = in_buf;
                pp.src_off = in_off;
                pp.dst_buf = out_buf;
                pp.dst_off = out_off;
                pp.label = label;
                for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
                prog.passes.push_back(pp);
            };
            const int64_t m2 = (int64_t)M2;
            reg_pass(va, M1, no * m2, m2, RegSide{job.in_os, 1, m2}, RegSide{scr_os, 1, m2}, chirp, ttw, (int64_t)N,
                     job.in_buf, job.in_off, BUF_SCRATCH0, 0, 1.0, "bluestein columns (register)");
            {
                // the rows (FFT * spectrum * inverse FFT of length M2) stay on the generic
                // pass: the register version (radices 5 3 3 3 3, 15 points per thread)
                // needs 174 registers, one 216-thread CTA per SM, and measured 4.3 ms per
                // direction for 65537 x 2048 against the generic pass's 2.6 ms
                PassBuilder b(prog, (int)M2, line_stages(M2, nullptr), true, no * (int64_t)M1, kMaxOps);
                b.load((int)M2, 0);
                b.fft();
                b.mul_region(table_bluestein_spectrum_rows(prog, N, M, M1, M2), F_CONJ_OUT, (int)M2, 1);
                b.fft();
                b.store((int)M2, F_CONJ_IN | F_CONJ_LUT, MUL_TWIDDLE_CE, ttw, 1.0, 1, (int)M2);
                prog.passes.push_back(b.finish(no, 1, (int64_t)M1, make_side(scr_os, 1, m2, 1, false, M, (int)M2, 1),
                                               make_side(scr_os, 1, m2, 1, false, M, (int)M2, 1), BUF_SCRATCH0, 0,
                                               BUF_SCRATCH0, 0, "bluestein rows"));
            }
            reg_pass(vc, M1, no * m2, m2, RegSide{scr_os, 1, m2}, RegSide{job.out_os, 1, m2}, chirp, -1,
                     (int64_t)out_count, BUF_SCRATCH0, 0, job.out_buf, job.out_off, scale,
                     "bluestein columns inverse (register)");
            return;
        }
    }
    const int spec = table_bluestein_spectrum(prog, N, M);
    // contiguous axis (S = 1): the rows of pass B are contiguous in scratch and its threads
    // walk elements, so its spectrum and twiddle tables are laid out row by row
    const bool rows_contig = S == 1;
    // pass A: columns n2: x[n2 + M2 n1] * chirp (n < N, else 0), FFT over n1, * W_M^{n2 k1}
    {
        PassBuilder b(prog, (int)M1, line_stages(M1, nullptr), true, no * S * M2, kMaxOps);
        b.load((int)M1, cin, MUL_LUT_N, chirp);
        b.fft();
        b.store((int)M1, 0, MUL_TWIDDLE_CE, table_twiddle_transposed(prog, M2, M1, M), 1.0, (int)M2, 1);
        prog.passes.push_back(b.finish(no, S, (int64_t)M2,
                                       make_side(job.in_os, 1, S, (int64_t)M2 * S, job.in_real, N, 1, (int)M2, herm),
                                       make_side(scr_os, 1, S, (int64_t)M2 * S, false, M, 1, (int)M2), job.in_buf,
                                       job.in_off, BUF_SCRATCH0, 0, "bluestein columns"));
    }
    // pass B: rows k1: FFT over n2 -> k2, * spectrum[k1 + M1 k2], inverse FFT over k2 -> n2,
    // * conj(W_M^{n2 k1}), in place in scratch
    {
        PassBuilder b(prog, (int)M2, line_stages(M2, nullptr), true, no * S * M1, kMaxOps);
        b.load((int)M2, 0);
        b.fft();
        if (rows_contig)
            b.mul_region(table_bluestein_spectrum_rows(prog, N, M, M1, M2), F_CONJ_OUT, (int)M2, 1);
        else
            b.mul_region(spec, F_CONJ_OUT, 1, (int)M1);
        b.fft();
        if (rows_contig)  // W_M^{k1 n2} at k1 M2 + n2
            b.store((int)M2, F_CONJ_IN | F_CONJ_LUT, MUL_TWIDDLE_CE, table_twiddle_transposed(prog, M2, M1, M), 1.0,
                    1, (int)M2);
        else
            b.store((int)M2, F_CONJ_IN | F_CONJ_LUT, MUL_TWIDDLE_CE, table_twiddle_transposed(prog, M1, M2, M), 1.0,
                    (int)M1, 1);
        prog.passes.push_back(b.finish(no, S, (int64_t)M1,
                                       make_side(scr_os, 1, (int64_t)M2 * S, S, false, M, (int)M2, 1),
                                       make_side(scr_os, 1, (int64_t)M2 * S, S, false, M, (int)M2, 1), BUF_SCRATCH0,
                                       0, BUF_SCRATCH0, 0, "bluestein rows"));
    }
    // pass C: columns n2: inverse FFT over k1 -> n1, * chirp[n2 + M2 n1], keep n < out_count
    {
        PassBuilder b(prog, (int)M1, line_stages(M1, nullptr), true, no * S * M2, kMaxOps);
        b.load((int)M1, F_CONJ_OUT);
        b.fft();
        b.store((int)M1, F_CONJ_IN | cout | fscale, MUL_LUT_N, chirp, scale);
        prog.passes.push_back(
            b.finish(no, S, (int64_t)M2, make_side(scr_os, 1, S, (int64_t)M2 * S, false, M, 1, (int)M2),
                     make_side(job.out_os, 1, So, (int64_t)M2 * So, job.out_real, out_count, 1, (int)M2), BUF_SCRATCH0,
                     0, job.out_buf, job.out_off, "bluestein columns inverse"));
    }
}

// R2C of the contiguous axis.  EvenHalfSize (real_ir.rs:1002-1013): the real line is
// read as N/2 complex pairs, transformed and post-processed into N/2+1 bins; fused into
// one pass when the half-length child runs on chip, otherwise the child transform writes
// scratch 2 and a post-processing pass produces the bins.  FullComplex: the real line is
// promoted on load and the complex child keeps the first N/2+1 bins.
// f64 even-half with a Bluestein child cannot stay within 1e-13 of the reference's CPU
// path: that path transforms the even and odd samples separately, and Bluestein with the
// reference's unreduced chirp is not exactly Hermitian-symmetric, so the even-half
// extraction differs from it at ~1e-12.  Those f64 lines use the full complex transform.
static bool even_half_usable(const Program &prog, const RealAxisJob &job) {
    return !(prog.is_double && job.alg->kind == AlgorithmKind::Bluestein);
}

// Power-of-two rows run the even-half algebra in the register kernel whatever the
// plan's real algorithm (the planner's FullComplex / EvenHalfSize choice is kept and
// reported): one read and one write of the tensor and half the butterflies of the
// FullComplex transform.  R2C: both algorithms are the DFT of the real input.  C2R: the
// FullComplex result is the real part of the Hermitian expansion, which ignores the
// imaginary parts of X[0] and X[h]; for a FullComplex plan the kernel drops them, and the
// even-half algebra then computes the same real inverse DFT.
// DCT/DST reduction twiddles of a register pass, indexed by FFT position p < L:
// [A | B] with A the pre-processing and B the post-processing factor of the type
// (reg_kernels.cu r2r_load_all / r2r_store_all):
//   II:  A[p] = W_4n^p                        (post)
//   III: A[p] = conj W_4n^p                   (pre)
//   IV, n even (L = n/2): A[p] = conj W_4n^2p (pre), B[p] = W_8n^(4p+1) (post)
//   IV, n odd (L = 2n):   A[p] = W_4n^p (pre), B[p] = W_8n^(2p+1) (post), p < n
int table_r2r(Program &prog, int type, size_t n, size_t L) {
    std::string key = "r2r" + std::to_string(type) + "_" + std::to_string(n) + "_" + std::to_string(L);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    HostTable t;
    t.c.assign(2 * L, std::complex<double>(0.0, 0.0));
    if (prog.is_dd) t.lo.assign(2 * L, std::complex<double>(0.0, 0.0));
    for (size_t p = 0; p < L; p++) {
        if (type == 1) {
            put_root(t, prog, p, p, 4 * n);
        } else if (type == 2) {
            put_root(t, prog, p, p, 4 * n, true);
        } else if (n % 2 == 0) {
            put_root(t, prog, p, 2 * p, 4 * n, true);
            put_root(t, prog, L + p, 4 * p + 1, 8 * n);
        } else if (p < n) {
            put_root(t, prog, p, p, 4 * n);
            put_root(t, prog, L + p, 2 * p + 1, 8 * n);
        }
    }
    return add_table(prog, key, std::move(t));
}

// [W_n^k | W_4n^k], k = 0..n/2: the even-half and rotation twiddles of REG_R2R_HALF.
static int table_r2r_half(Program &prog, size_t n) {
    std::string key = "r2rh" + std::to_string(n);
    auto it = prog.table_cache.find(key);
    if (it != prog.table_cache.end()) return it->second;
    const size_t h = n / 2;
    HostTable t;
    t.c.resize(2 * (h + 1));
    for (size_t k = 0; k <= h; k++) {
        put_root(t, prog, k, k, n);
        put_root(t, prog, h + 1 + k, k, 4 * n);
    }
    return add_table(prog, key, std::move(t));
}

// DCT/DST-II/III of contiguous even-length lines: the reduction's real length-n sequence
// through the even-half algebra, one register pass with an FFT of length n/2.
static bool lower_r2r_half_register(Program &prog, const R2rAxisJob &job) {
    const int type = job.kind & 3;
    const size_t n = job.n, h = n / 2;
    // f32 only: the f64 even-half variants need ~145 registers and measured slower than the
    // full-length REG_R2R pass
    if ((type != 1 && type != 2) || job.inner != 1 || n % 2 || !is_pow2(h) || !reg_kernels_enabled() || !job.alg ||
        job.alg->kind != AlgorithmKind::Stockham || prog.is_double)
        return false;
    const int rv = reg_variant(prog, h, REG_R2R_HALF, false);
    if (rv < 0) return false;
    PassPlan pp{};
    pp.kernel = KERNEL_REG;
    pp.reg_variant = rv;
    pp.reg_table = table_reg_twiddles(prog, h, rv);
    pp.reg_table2 = table_r2r_half(prog, n);
    pp.rp.nlines = job.outer;
    pp.rp.ni = 1;
    pp.rp.src = pp.rp.dst = RegSide{(int64_t)n, 0, 1};
    pp.rp.scale = job.scale;
    pp.rp.conj = type == 2 ? 1 : 0;
    pp.rp.n = (int32_t)h;
    pp.rp.r2r_kind = job.kind;
    pp.rp.r2r_n = (int32_t)n;
    pp.reg_in_real = pp.reg_out_real = true;
    pp.src_buf = job.in_buf;
    pp.dst_buf = job.out_buf;
    pp.label = "register dct/dst even-half";
    // type III (four reals per point) runs faster from the bulk-copied line; type II
    // measured faster on the plain kernel
    if (type == 2 && (n * (size_t)prog.rbytes()) % 16 == 0) {
        const int pv = reg_variant_persistent_twin(rv);
        if (pv >= 0) {
            pp.reg_variant_plain = rv;
            pp.reg_variant = pv;
            pp.label = "register dct/dst even-half (bulk prefetch)";
        }
    }
    for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
    prog.passes.push_back(pp);
    return true;
}

bool lower_r2r_axis_register(Program &prog, const R2rAxisJob &job) {
    if (lower_r2r_half_register(prog, job)) return true;
    const size_t L = job.L;
    if (!is_pow2(L) || !reg_kernels_enabled() || !job.alg || job.alg->kind != AlgorithmKind::Stockham) return false;
    if (job.n > (size_t)INT32_MAX / 4) return false;
    const bool strided = job.inner > 1;
    const int rv = reg_variant(prog, L, REG_R2R, strided);
    if (rv < 0) return false;
    PassPlan pp{};
    pp.kernel = KERNEL_REG;
    pp.reg_variant = rv;
    pp.reg_table = table_reg_twiddles(prog, L, rv);
    pp.reg_table2 = (job.kind & 3) == 0 ? -1 : table_r2r(prog, job.kind & 3, job.n, L);
    pp.rp.nlines = job.outer * job.inner;
    pp.rp.ni = job.inner;
    pp.rp.src = pp.rp.dst = RegSide{(int64_t)job.n * job.inner, strided ? 1 : 0, job.inner};
    pp.rp.scale = job.scale;
    pp.rp.conj = job.fft_inverse ? 1 : 0;
    pp.rp.n = (int32_t)L;
    pp.rp.r2r_kind = job.kind;
    pp.rp.r2r_n = (int32_t)job.n;
    pp.reg_in_real = pp.reg_out_real = true;
    pp.src_buf = job.in_buf;
    pp.dst_buf = job.out_buf;
    pp.label = "register dct/dst";
    // dense contiguous lines whose byte length is a multiple of 16: the persistent
    // variant fetches each CTA's next line group with one bulk copy
    const size_t line_bytes = job.n * (size_t)prog.rbytes();
    if (!strided && line_bytes % 16 == 0 && job.n <= 2 * L) {
        const int pv = reg_variant_persistent_twin(rv);
        if (pv >= 0) {
            pp.reg_variant_plain = rv;
            pp.reg_variant = pv;
            pp.label = "register dct/dst (bulk prefetch)";
        }
    }
    for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
    prog.passes.push_back(pp);
    return true;
}

static bool lower_real_axis_register(Program &prog, const RealAxisJob &job, bool r2c) {
    const size_t N = job.N, h = N / 2;
    if (N % 2 || !is_pow2(h) || !reg_kernels_enabled() || job.in_off || job.out_off) return false;
    const int rv = reg_variant(prog, h, r2c ? REG_R2C_HALF : REG_C2R_HALF, false);
    if (rv < 0) return false;
    PassPlan pp{};
    pp.kernel = KERNEL_REG;
    pp.reg_variant = rv;
    pp.reg_table = table_reg_twiddles(prog, h, rv);
    pp.reg_table2 = table_twiddle(prog, N);
    pp.rp.nlines = job.lines;
    pp.rp.ni = 1;
    pp.rp.src = RegSide{(int64_t)(r2c ? h : h + 1), 0, 1};
    pp.rp.dst = RegSide{(int64_t)(r2c ? h + 1 : h), 0, 1};
    pp.rp.scale = (!r2c && job.normalize) ? 1.0 / (double)h : 1.0;
    pp.rp.scale2 = (!r2c && job.normalize) ? 0.5 : 1.0;
    pp.rp.conj = r2c ? 0 : 1;
    pp.rp.n = (int32_t)h;
    pp.rp.real_ends = (!r2c && job.full_complex) ? 1 : 0;
    pp.src_buf = job.in_buf;
    pp.dst_buf = job.out_buf;
    pp.label = r2c ? "register r2c even-half" : "register c2r even-half";
    // dense C2R lines: the persistent variant fetches each CTA's next group of bins with
    // one bulk copy when every group (the last, partial one included) is a multiple of 16
    // bytes (its loads gather X[p] and X[h-p]; R2C measured faster without it)
    if (!r2c) {
        const int pv = reg_variant_persistent_twin(rv);
        if (pv >= 0) {
            const size_t G = (size_t)reg_variant_lines_per_cta(pv);
            const size_t line_bytes = (r2c ? h : h + 1) * (size_t)prog.cbytes();
            const size_t tail = (size_t)job.lines % G;
            if ((G * line_bytes) % 16 == 0 && (tail * line_bytes) % 16 == 0) {
                pp.reg_variant_plain = rv;
                pp.reg_variant = pv;
                pp.label = "register c2r even-half (bulk prefetch)";
            }
        }
    }
    for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
    prog.passes.push_back(pp);
    return true;
}

void lower_r2c_axis(Program &prog, const RealAxisJob &job) {
    const size_t N = job.N;
    const PlannerTuning *saved = g_tuning;
    g_tuning = &job.tuning;
    struct Restore {
        const PlannerTuning *t;
        ~Restore() { g_tuning = t; }
    } restore{saved};
    if (lower_real_axis_register(prog, job, true)) return;
    if (!job.full_complex && N % 2 == 0 && N >= 2 && even_half_usable(prog, job)) {
        const size_t h = N / 2;
        const int wn = table_twiddle(prog, N);
        const bool fused = job.alg->kind != AlgorithmKind::Bluestein && line_fits_on_chip(prog.cbytes(), h, job.alg, false) &&
                           line_capacity_ok(prog.cbytes(), h + 1);
        if (fused) {
            PassBuilder b(prog, (int)h, line_stages(h, job.alg), false, job.lines, 24);
            b.load((int)h, 0);
            b.fft();
            b.r2c_post((int)h, wn);
            b.store((int)(h + 1), 0);
            prog.passes.push_back(b.finish(job.lines, 1, 1, make_side((int64_t)h, 0, 0, 1, false, h, 0, 1),
                                           make_side((int64_t)(h + 1), 0, 0, 1, false, h + 1, 0, 1), job.in_buf,
                                           job.in_off, job.out_buf, job.out_off, "r2c even-half"));
            return;
        }
        if (!line_capacity_ok(prog.cbytes(), h + 1))
            fail_unsupported("B200 engine: real axis post-processing exceeds on-chip capacity");
        prog.scratch_elems[2] = std::max(prog.scratch_elems[2], (size_t)job.lines * h);
        AxisJob a;
        a.N = h;
        a.alg = job.alg;
        a.tuning = job.tuning;
        a.no = job.lines;
        a.in_buf = job.in_buf;
        a.in_off = job.in_off;
        a.in_os = (int64_t)h;
        a.out_buf = BUF_SCRATCH2;
        a.out_os = (int64_t)h;
        lower_c2c_axis(prog, a);
        PassBuilder b(prog, (int)h, {}, false, job.lines, 4);
        b.load((int)h, 0);
        b.r2c_post((int)h, wn);
        b.store((int)(h + 1), 0);
        prog.passes.push_back(b.finish(job.lines, 1, 1, make_side((int64_t)h, 0, 0, 1, false, h, 0, 1),
                                       make_side((int64_t)(h + 1), 0, 0, 1, false, h + 1, 0, 1), BUF_SCRATCH2, 0,
                                       job.out_buf, job.out_off, "r2c post-process"));
        return;
    }
    AxisJob a;
    a.N = N;
    AxisAlgorithm full_alg;
    if (!job.full_complex) {
        // even-half was planned (child of length N/2) but is not usable: plan the full length
        full_alg = plan_axis_algorithm(N, job.tuning);
        a.alg = &full_alg;
    } else {
        a.alg = job.alg;
    }
    a.tuning = job.tuning;
    a.no = job.lines;
    a.S = 1;
    a.in_buf = job.in_buf;
    a.in_off = job.in_off;
    a.in_os = (int64_t)N;
    a.in_real = true;
    a.out_buf = job.out_buf;
    a.out_off = job.out_off;
    a.out_os = (int64_t)(N / 2 + 1);
    a.out_count = N / 2 + 1;
    lower_c2c_axis(prog, a);
}

// C2R of the contiguous axis.  EvenHalfSize (real_ir.rs:1087-1100): N/2+1 bins ->
// packed half spectrum -> inverse FFT_{N/2} -> N reals stored as N/2 complex pairs
// (fused, or a pre-processing pass into scratch 2 followed by the child transform).
// FullComplex: Hermitian expansion on chip, inverse complex transform, real part.
void lower_c2r_axis(Program &prog, const RealAxisJob &job) {
    const size_t N = job.N;
    const PlannerTuning *saved = g_tuning;
    g_tuning = &job.tuning;
    struct Restore {
        const PlannerTuning *t;
        ~Restore() { g_tuning = t; }
    } restore{saved};
    if (lower_real_axis_register(prog, job, false)) return;
    if (!job.full_complex && N % 2 == 0 && N >= 2 && even_half_usable(prog, job)) {
        const size_t h = N / 2;
        const int wn = table_twiddle(prog, N);
        const bool fused = job.alg->kind != AlgorithmKind::Bluestein && line_fits_on_chip(prog.cbytes(), h, job.alg, false) &&
                           line_capacity_ok(prog.cbytes(), h + 1);
        const int fsc = job.normalize ? F_SCALE : 0;
        if (fused) {
            PassBuilder b(prog, (int)h, line_stages(h, job.alg), false, job.lines, 24);
            b.load((int)(h + 1), 0);
            b.c2r_pre((int)h, wn, F_CONJ_OUT | fsc, job.normalize ? 0.5 : 1.0);
            b.fft();
            b.store((int)h, F_CONJ_OUT | fsc, MUL_NONE, -1, job.normalize ? 1.0 / (double)h : 1.0);
            prog.passes.push_back(b.finish(job.lines, 1, 1, make_side((int64_t)(h + 1), 0, 0, 1, false, h + 1, 0, 1),
                                           make_side((int64_t)h, 0, 0, 1, false, h, 0, 1), job.in_buf, job.in_off,
                                           job.out_buf, job.out_off, "c2r even-half"));
            return;
        }
        if (!line_capacity_ok(prog.cbytes(), h + 1))
            fail_unsupported("B200 engine: real axis pre-processing exceeds on-chip capacity");
        prog.scratch_elems[2] = std::max(prog.scratch_elems[2], (size_t)job.lines * h);
        {
            PassBuilder b(prog, (int)h, {}, false, job.lines, 4);
            b.load((int)(h + 1), 0);
            b.c2r_pre((int)h, wn, fsc, job.normalize ? 0.5 : 1.0);
            b.store((int)h, 0);
            prog.passes.push_back(b.finish(job.lines, 1, 1, make_side((int64_t)(h + 1), 0, 0, 1, false, h + 1, 0, 1),
                                           make_side((int64_t)h, 0, 0, 1, false, h, 0, 1), job.in_buf, job.in_off,
                                           BUF_SCRATCH2, 0, "c2r pre-process"));
        }
        AxisJob a;
        a.N = h;
        a.alg = job.alg;
        a.tuning = job.tuning;
        a.no = job.lines;
        a.inverse = true;
        a.scale = job.normalize ? 1.0 / (double)h : 1.0;
        a.in_buf = BUF_SCRATCH2;
        a.in_os = (int64_t)h;
        a.out_buf = job.out_buf;
        a.out_off = job.out_off;
        a.out_os = (int64_t)h;
        lower_c2c_axis(prog, a);
        return;
    }
    AxisJob a;
    a.N = N;
    AxisAlgorithm full_alg;
    if (!job.full_complex) {
        full_alg = plan_axis_algorithm(N, job.tuning);
        a.alg = &full_alg;
    } else {
        a.alg = job.alg;
    }
    a.tuning = job.tuning;
    a.no = job.lines;
    a.S = 1;
    a.inverse = true;
    a.scale = job.normalize ? 1.0 / (double)N : 1.0;
    a.in_buf = job.in_buf;
    a.in_off = job.in_off;
    a.in_os = (int64_t)(N / 2 + 1);
    a.in_herm = true;
    a.out_buf = job.out_buf;
    a.out_off = job.out_off;
    a.out_os = (int64_t)N;
    a.out_real = true;
    lower_c2c_axis(prog, a);
}

// Convolution multiply pass (convolution_ir.rs:4235-4246) for K kernels: for every kernel k
// and coordinate c, out[(k C + c) L + i] = policy(in[c L + i]) * ker[(k C + c) L + i]
// (ker[i] when one spectrum copy is broadcast).  Lines are chunks of the compact tensor.
void lower_convolution_multiply(Program &prog, int64_t L, int64_t C, int64_t K, int in_buf, int out_buf,
                                int spec_table, int64_t spec_copies, bool conj_sequence, bool cross_power) {
    int64_t chunk = 1;
    for (int64_t d = std::min<int64_t>(L, 4096); d >= 1; d--)
        if (L % d == 0) {
            chunk = d;
            break;
        }
    const int mflags = (conj_sequence ? F_CONJ_IN : 0) | (cross_power ? F_NORMALIZE : 0);
    const Side side = make_side(L, 0, chunk, 1, false, L, (int)chunk, 1);
    for (int64_t k = 0; k < K; k++) {
        PassBuilder b(prog, (int)chunk, {}, false, C * (L / chunk), 4);
        b.load((int)chunk, 0);
        b.mul_region(spec_table, mflags, (int)chunk, 1, 0, spec_copies > 1 ? L : 0, spec_copies > 1 ? k * C * L : 0);
        b.store((int)chunk, 0);
        prog.passes.push_back(b.finish(C, 1, L / chunk, side, side, in_buf, 0, out_buf, k * C * L, "convolution multiply"));
    }
}

// Fused outermost convolution axis (convolution_ir.rs:4185-4250 multiply, here between the
// forward and the inverse transform of the same lines): forward FFT of length H, multiply by
// the kernel spectrum ker[o*om + c + e*inner] (policy: sequence conjugation, cross-power
// normalisation), inverse FFT, scale.  In place on `buf`.
void lower_convolution_axis0(Program &prog, size_t H, const AxisAlgorithm *alg, const PlannerTuning &tuning,
                             int64_t systems, int64_t inner, int buf, int spec_table, int64_t spec_outer_stride,
                             bool conj_sequence, bool cross_power, double scale) {
    const PlannerTuning *saved = g_tuning;
    g_tuning = &tuning;
    struct Restore {
        const PlannerTuning *t;
        ~Restore() { g_tuning = t; }
    } restore{saved};
    const int mflags = (conj_sequence ? F_CONJ_IN : 0) | (cross_power ? F_NORMALIZE : 0) | F_CONJ_OUT;
    // power-of-two axis: forward FFT, multiply and inverse FFT in the register kernel
    if (alg->kind == AlgorithmKind::Stockham && is_pow2(H) && reg_kernels_enabled()) {
        const int rv = reg_variant(prog, H, REG_CONV, true);
        if (rv >= 0) {
            PassPlan pp{};
            pp.kernel = KERNEL_REG;
            pp.reg_variant = rv;
            pp.reg_table = table_reg_twiddles(prog, H, rv);
            pp.reg_table2 = spec_table;
            pp.rp.nlines = systems * inner;
            pp.rp.ni = inner;
            pp.rp.src = pp.rp.dst = RegSide{(int64_t)H * inner, 1, inner};
            pp.rp.scale = scale;
            pp.rp.conj = 1;
            pp.rp.n = (int32_t)H;
            pp.rp.conv_flags = mflags;
            pp.rp.conv_em = inner;
            pp.rp.conv_om = spec_outer_stride;
            pp.src_buf = pp.dst_buf = buf;
            pp.label = "register convolution axis";
            for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
            prog.passes.push_back(pp);
            return;
        }
    }
    const Side side = make_side((int64_t)H * inner, 0, 1, inner, false, (int64_t)H * inner, 1, (int)inner);
    if (alg->kind != AlgorithmKind::Bluestein && line_fits_on_chip(prog.cbytes(), H, alg, true)) {
        PassBuilder b(prog, (int)H, line_stages(H, alg), true, systems * inner, kMaxOps);
        b.load((int)H, 0);
        b.fft();
        b.mul_region(spec_table, mflags, 1, (int)inner, 0, spec_outer_stride);
        b.fft();
        b.store((int)H, F_CONJ_OUT | F_SCALE, MUL_NONE, -1, scale);
        prog.passes.push_back(b.finish(systems, 1, inner, side, side, buf, 0, buf, 0, "convolution axis fused"));
        return;
    }
    // unfused: forward axis, multiply pass, inverse axis
    AxisJob job;
    job.N = H;
    job.alg = alg;
    job.tuning = tuning;
    job.no = systems;
    job.S = inner;
    job.in_buf = job.out_buf = buf;
    job.in_os = job.out_os = (int64_t)H * inner;
    lower_c2c_axis(prog, job);
    const int64_t L = (int64_t)H * inner;
    lower_convolution_multiply(prog, L, systems, 1, buf, buf, spec_table, spec_outer_stride ? systems : 1,
                               conj_sequence, cross_power);
    job.inverse = true;
    job.scale = scale;
    lower_c2c_axis(prog, job);
}

}  // namespace b200fft
