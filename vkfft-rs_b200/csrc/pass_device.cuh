// Device side of the B200 FFT pass kernel: the per-CTA prologue and the op functions
// (load, radix stages, multiplies, Rader, real pre/post processing, store).  Included
// by kernels.cu (the precompiled op-program interpreter, and the CPU emulator) and by
// the ahead-of-time specialised pass kernels the build generates (aot.hpp), which call
// the same functions with the pass's structure as compile-time constants.
#pragma once

#include <cmath>
#include <cstdint>

#include "dft_codelets.cuh"
#include "dd.cuh"
#include "pass_desc.hpp"

// Threads of the CTA: each unit of specialised kernels defines it as their literal
// thread count, so every op loop below has a compile-time stride (the compiler unrolls
// the rounds of a radix stage and overlaps their loads); the interpreter reads blockDim.x.
#ifndef B200FFT_NT
#define B200FFT_NT blockDim.x
#define B200FFT_STAGE_UNROLL
#else
#define B200FFT_STAGE_UNROLL _Pragma("unroll")
#endif

namespace b200fft {

template <typename T> struct vec2;
template <> struct vec2<float> { using type = float2; };
template <> struct vec2<double> { using type = double2; };

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) { return (__umulhi(n, f.m) + n) >> f.s; }
// Shared-memory slot of line element e >= 0 (Op::pad_shift: one spare slot every
// 2^shift elements, or none for shift 31 -- the unpadded layout; pad_shift is a literal
// in the specialised kernels, so the branch folds away there).
__device__ __forceinline__ int spad(int e, int shift) { return shift >= 31 ? e : e + (e >> shift); }

template <typename T> __device__ __forceinline__ cplx<T> cmul(cplx<T> a, cplx<T> b) {
    return {a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x};
}
template <typename T> __device__ __forceinline__ cplx<T> cconj(cplx<T> a) { return {a.x, -a.y}; }
template <typename T> __device__ __forceinline__ cplx<T> ld_ro(const void *base, int64_t idx) {
    auto v = __ldg(reinterpret_cast<const typename vec2<T>::type *>(base) + idx);
    return {v.x, v.y};
}
template <typename T> __device__ __forceinline__ cplx<T> ld_data(const void *base, int64_t idx) {
    auto v = __ldcs(reinterpret_cast<const typename vec2<T>::type *>(base) + idx);
    return {v.x, v.y};
}
template <typename T> __device__ __forceinline__ void st_data(void *base, int64_t idx, cplx<T> v) {
    typename vec2<T>::type w;
    w.x = v.x;
    w.y = v.y;
    __stcs(reinterpret_cast<typename vec2<T>::type *>(base) + idx, w);
}

// Double-double complex elements are 32 bytes (re.hi, re.lo, im.hi, im.lo): two
// 16-byte accesses each.
template <> __device__ __forceinline__ cplx<dd> ld_ro<dd>(const void *base, int64_t idx) {
    const double2 *q = reinterpret_cast<const double2 *>(base) + 2 * idx;
    const double2 a = __ldg(q), b = __ldg(q + 1);
    return {dd(a.x, a.y), dd(b.x, b.y)};
}
template <> __device__ __forceinline__ cplx<dd> ld_data<dd>(const void *base, int64_t idx) {
    const double2 *q = reinterpret_cast<const double2 *>(base) + 2 * idx;
    const double2 a = __ldcs(q), b = __ldcs(q + 1);
    return {dd(a.x, a.y), dd(b.x, b.y)};
}
__device__ __forceinline__ double2 dd_words(dd v) {
    double2 w;
    w.x = v.hi;
    w.y = v.lo;
    return w;
}
template <> __device__ __forceinline__ void st_data<dd>(void *base, int64_t idx, cplx<dd> v) {
    double2 *q = reinterpret_cast<double2 *>(base) + 2 * idx;
    __stcs(q, dd_words(v.x));
    __stcs(q + 1, dd_words(v.y));
}

// One real scalar of a real side.
template <typename T> __device__ __forceinline__ T ld_real(const void *base, int64_t idx) {
    return __ldcs(reinterpret_cast<const T *>(base) + idx);
}
template <> __device__ __forceinline__ dd ld_real<dd>(const void *base, int64_t idx) {
    const double2 a = __ldcs(reinterpret_cast<const double2 *>(base) + idx);
    return dd(a.x, a.y);
}
template <typename T> __device__ __forceinline__ void st_real(void *base, int64_t idx, T v) {
    __stcs(reinterpret_cast<T *>(base) + idx, v);
}
template <> __device__ __forceinline__ void st_real<dd>(void *base, int64_t idx, dd v) {
    __stcs(reinterpret_cast<double2 *>(base) + idx, dd_words(v));
}

__device__ __forceinline__ void raise_error(int *err, int code) {
    if (err && threadIdx.x == 0) atomicOr(err, code);
}

// value *= table (kind/flags of the op), with the optional conjugations and scale.
template <typename T>
__device__ __forceinline__ cplx<T> apply_mul(cplx<T> v, const Op &op, int c, int e, int n) {
    if (op.flags & F_CONJ_IN) v = cconj(v);
    if (op.mul != MUL_NONE) {
        const int idx = (op.flags & F_OWN_INDEX) ? c * op.cm + e * op.em : (op.mul == MUL_LUT_N ? n : c * e);
        cplx<T> w = ld_ro<T>(op.lut, idx);
        if (op.flags & F_CONJ_LUT) w = cconj(w);
        v = cmul(v, w);
    }
    if (op.flags & F_SCALE) {
        v.x *= kc<T>(op.scale, op.scale_lo);
        v.y *= kc<T>(op.scale, op.scale_lo);
    }
    if (op.flags & F_CONJ_OUT) v = cconj(v);
    return v;
}

struct LineMeta {
    const int64_t *ib;
    const int64_t *ob;
    const int *col;
    const int *oidx;  // outer index o of each line
    int nl;           // valid lines in this CTA
};

constexpr int kLoadUnroll = 8;

// global -> region dst_base (line g at dst_base + g*sub_stride)
template <typename T>
__device__ __forceinline__ void op_load(const PassShape &p, const Op &op, cplx<T> *sm, const LineMeta &lm) {
    const int len = op.len;
    const int G = p.G;
    const int total = G * len;
    const Side &s = p.in;
    const bool efast = s.es == 1;
    for (int f0 = 0; f0 < total; f0 += kLoadUnroll * B200FFT_NT) {
        cplx<T> v[kLoadUnroll];
        int dst[kLoadUnroll];
#pragma unroll
        for (int u = 0; u < kLoadUnroll; u++) {
            const int f = f0 + threadIdx.x + u * B200FFT_NT;
            dst[u] = -1;
            v[u] = {T(0), T(0)};
            if (f < total) {
                int g, e;
                if (efast) {
                    g = fdiv(f, op.div_a);
                    e = f - g * len;
                } else {
                    e = fdiv(f, p.div_g);
                    g = f - e * G;
                }
                dst[u] = op.dst_base + g * op.sub_stride + spad(e, op.pad_shift);
                const int c = lm.col[g];
                const int n = c * s.cm + e * s.em;
                if (g < lm.nl && n < s.count) {
                    int64_t a = lm.ib[g] + (int64_t)e * s.es;
                    bool mirrored = false;
                    if (s.herm && n > s.herm / 2) {
                        // Hermitian input: X[n] = conj(X[N - n]), N - n < N/2 is stored
                        const int n2 = s.herm - n;
                        const int e2 = n2 / s.em;
                        const int c2 = s.cm ? n2 - e2 * s.em : c;
                        a = lm.ib[g] + (int64_t)(c2 - c) * s.cs + (int64_t)e2 * s.es;
                        mirrored = true;
                    }
                    if (s.real) {
                        v[u].x = ld_real<T>(p.src, a);
                    } else {
                        v[u] = ld_data<T>(p.src, a);
                        if (mirrored) v[u].y = -v[u].y;
                    }
                    v[u] = apply_mul(v[u], op, c, e, n);
                }
            }
        }
#pragma unroll
        for (int u = 0; u < kLoadUnroll; u++)
            if (dst[u] >= 0) sm[dst[u]] = v[u];
    }
}

// region src_base -> global
template <typename T>
__device__ __forceinline__ void op_store(const PassShape &p, const Op &op, const cplx<T> *sm, const LineMeta &lm) {
    const int len = op.len;
    const int G = p.G;
    const int total = G * len;
    const Side &s = p.out;
    const bool efast = s.es == 1;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        int g, e;
        if (efast) {
            g = fdiv(f, op.div_a);
            e = f - g * len;
        } else {
            e = fdiv(f, p.div_g);
            g = f - e * G;
        }
        const int c = lm.col[g];
        const int n = c * s.cm + e * s.em;
        if (g < lm.nl && n < s.count) {
            cplx<T> v = sm[op.src_base + g * op.sub_stride + spad(e, op.pad_shift)];
            v = apply_mul(v, op, c, e, n);
            int64_t a = lm.ob[g] + (int64_t)e * s.es;
            void *dst = p.dst;
            if (p.peer.n) {
                const int r = (int)fdiv((uint32_t)n, p.peer.div);
                dst = p.peer.ptr[r];
                a += p.peer.off - (int64_t)r * p.peer.sub;
            }
            if (s.real) {
                st_real<T>(dst, a, v.x);
            } else {
                st_data<T>(dst, a, v);
            }
        }
    }
    // peer stores are visible system-wide before the rank's exchange signal
    if (p.peer.n) __threadfence_system();
}

// One radix-R Stockham stage over nsub sub-lines of length len, src -> dst.
// Butterfly b = (sub-line s, index bb); j = bb mod P.  Inputs bb + q*len/R,
// twiddled by W_{P*R}^{j*q}; outputs (bb - j)*R + j + q*P.
template <typename T, int R>
__device__ __forceinline__ void op_stage(const Op &op, cplx<T> *sm) {
    const int NBL = op.len / R;
    const int NB = op.nsub * NBL;
    const int P = op.P;
    B200FFT_STAGE_UNROLL
    for (int b = threadIdx.x; b < NB; b += B200FFT_NT) {
        const int s = op.nsub == 1 ? 0 : (int)fdiv(b, op.div_a);
        const int bb = b - s * NBL;
        const int j = bb - (int)fdiv(bb, op.div_b) * P;
        const cplx<T> *src = sm + op.src_base + s * op.sub_stride;
        cplx<T> *dst = sm + op.dst_base + s * op.sub_stride;
        cplx<T> v[R];
#pragma unroll
        for (int q = 0; q < R; q++) v[q] = src[spad(bb + q * NBL, op.pad_shift)];
        if (P > 1) {
            // Large stage tables (and every f64 table) miss L1 next to the line buffers:
            // only their power-of-two rows are read and w_q = w_{q - lowbit(q)} w_{lowbit(q)}
            // forms the rest (at most three products deep).  Small f32 tables stay L1-resident
            // and are read whole, which costs fewer issue slots than the products.
            // Double-double reads every row (its products cost more than the loads).
            if (sizeof(T) <= 8 && (sizeof(T) == 8 || (R - 1) * P >= 512)) {
                cplx<T> w[R];
#pragma unroll
                for (int q = 1; q < R; q++) {
                    if ((q & (q - 1)) == 0) {
                        w[q] = ld_ro<T>(op.lut, (q - 1) * P + j);
                    } else {
                        const int lb = q & (-q);
                        w[q] = cmul(w[q - lb], w[lb]);
                    }
                }
#pragma unroll
                for (int q = 1; q < R; q++) v[q] = cmul(v[q], w[q]);
            } else {
#pragma unroll
                for (int q = 1; q < R; q++) v[q] = cmul(v[q], ld_ro<T>(op.lut, (q - 1) * P + j));
            }
        }
        dft<R, T>(v);
        const int e0 = (bb - j) * R + j;
#pragma unroll
        for (int q = 0; q < R; q++) dst[spad(e0 + q * P, op.pad_shift)] = v[q];
    }
}

template <typename T>
__device__ __forceinline__ void op_stage_dispatch(const Op &op, cplx<T> *sm, int *err) {
    switch (op.radix) {
        case 2: op_stage<T, 2>(op, sm); break;
        case 3: op_stage<T, 3>(op, sm); break;
        case 4: op_stage<T, 4>(op, sm); break;
        case 5: op_stage<T, 5>(op, sm); break;
        case 6: op_stage<T, 6>(op, sm); break;
        case 7: op_stage<T, 7>(op, sm); break;
        case 8: op_stage<T, 8>(op, sm); break;
        case 9: op_stage<T, 9>(op, sm); break;
        case 10: op_stage<T, 10>(op, sm); break;
        case 11: op_stage<T, 11>(op, sm); break;
        case 12: op_stage<T, 12>(op, sm); break;
        case 13: op_stage<T, 13>(op, sm); break;
        case 16: op_stage<T, 16>(op, sm); break;
        default: raise_error(err, 2); break;
    }
}

// In-place pointwise multiply of the src region (sub-line s, element e) by lut[c*cm + e*em].
template <typename T>
__device__ __forceinline__ void op_mul(const Op &op, cplx<T> *sm, const LineMeta &lm) {
    const int len = op.len;
    const int total = op.nsub * len;
    const bool line_fast = op.flags & F_LINE_FAST;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        int s, e;
        if (line_fast) {
            e = fdiv(f, op.div_b);
            s = f - e * op.nsub;
        } else {
            s = fdiv(f, op.div_a);
            e = f - s * len;
        }
        cplx<T> *ptr = sm + op.src_base + s * op.sub_stride + spad(e, op.pad_shift);
        const cplx<T> v = *ptr;
        if ((op.flags & F_SAVE_DC) && e == 0) sm[op.x0_base + 2 * s + 1] = v;
        const int c = op.cm ? lm.col[s] : 0;
        const int n = c * op.cm + e * op.em;
        if (op.nfull && n >= op.nfull) continue;
        if (op.om || op.lut_off) {
            // table index with the outer term (one table copy per outer index)
            cplx<T> x = v;
            if (op.flags & F_CONJ_IN) x = cconj(x);
            cplx<T> w = ld_ro<T>(op.lut, (int64_t)n + (int64_t)lm.oidx[s] * op.om + op.lut_off);
            if (op.flags & F_CONJ_LUT) w = cconj(w);
            x = cmul(x, w);
            if (op.flags & F_NORMALIZE) {
                const T r = T(1) / sqrt(x.x * x.x + x.y * x.y);
                x.x *= r;
                x.y *= r;
            }
            if (op.flags & F_CONJ_OUT) x = cconj(x);
            *ptr = x;
            continue;
        }
        cplx<T> r = apply_mul(v, op, c, e, n);
        if (op.flags & F_NORMALIZE) {
            const cplx<T> x = (op.flags & F_CONJ_OUT) ? cconj(r) : r;
            const T k = T(1) / sqrt(x.x * x.x + x.y * x.y);
            r.x *= k;
            r.y *= k;
        }
        *ptr = r;
    }
}

// Even-N R2C post-processing (real_ir.rs:1002-1013), in place on the src region:
// from Z = FFT_{h}(x[2n] + i x[2n+1]), h = N/2,
// X[k] = 1/2 ((Z[k] + conj Z[h-k]) - i W_N^k (Z[k] - conj Z[h-k])), k = 0..h.
template <typename T>
__device__ __forceinline__ void op_r2c_post(const PassShape &p, const Op &op, cplx<T> *sm) {
    const int h = op.len;
    const int per = h / 2 + 1;
    const int total = p.G * per;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int g = f / per;
        const int k = f - g * per;
        cplx<T> *z = sm + op.src_base + g * op.sub_stride;
        const int k2 = (h - k) % h;
        const cplx<T> zk = z[spad(k % h, op.pad_shift)], zk2 = z[spad(k2, op.pad_shift)];
        auto post = [&](cplx<T> a, cplx<T> bc, int kk) {
            const cplx<T> b = cconj(bc);
            const cplx<T> w = ld_ro<T>(op.lut2, kk);
            const cplx<T> d = {a.x - b.x, a.y - b.y};
            const cplx<T> r = cmul(w, d);
            return cplx<T>{T(0.5) * (a.x + b.x + r.y), T(0.5) * (a.y + b.y - r.x)};
        };
        const cplx<T> xk = post(zk, zk2, k);
        if (k == 0) {
            z[spad(0, op.pad_shift)] = xk;
            z[spad(h, op.pad_shift)] = post(zk, zk, h);
        } else if (k != h - k) {
            const cplx<T> xk2 = post(zk2, zk, h - k);
            z[spad(k, op.pad_shift)] = xk;
            z[spad(h - k, op.pad_shift)] = xk2;
        } else {
            z[spad(k, op.pad_shift)] = xk;
        }
    }
}

// Even-N C2R pre-processing (real_ir.rs:1087-1100), in place on the src region:
// Z[k] = s (X[k] + conj X[h-k] + i conj(W_N^k) (X[k] - conj X[h-k])), k = 0..h-1.
template <typename T>
__device__ __forceinline__ void op_c2r_pre(const PassShape &p, const Op &op, cplx<T> *sm) {
    const int h = op.len;
    const int per = h / 2 + 1;
    const int total = p.G * per;
    const T sc = (op.flags & F_SCALE) ? kc<T>(op.scale, op.scale_lo) : T(1);
    const bool conj_out = op.flags & F_CONJ_OUT;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int g = f / per;
        const int k = f - g * per;
        cplx<T> *z = sm + op.src_base + g * op.sub_stride;
        const cplx<T> xa = z[spad(k, op.pad_shift)], xb = z[spad(h - k, op.pad_shift)];
        auto pre = [&](cplx<T> x, cplx<T> mc, int kk) {
            const cplx<T> m = cconj(mc);
            const cplx<T> w = cconj(ld_ro<T>(op.lut2, kk));
            const cplx<T> d = {x.x - m.x, x.y - m.y};
            const cplx<T> r = cmul(w, d);
            cplx<T> o = {sc * (x.x + m.x - r.y), sc * (x.y + m.y + r.x)};
            if (conj_out) o.y = -o.y;
            return o;
        };
        const cplx<T> za = pre(xa, xb, k);
        if (k == 0) {
            z[spad(0, op.pad_shift)] = za;
        } else if (k != h - k) {
            const cplx<T> zb = pre(xb, xa, h - k);
            z[spad(k, op.pad_shift)] = za;
            z[spad(h - k, op.pad_shift)] = zb;
        } else {
            z[spad(k, op.pad_shift)] = za;
        }
    }
}

// Rader radix-p step, gather half: for butterfly b = (s, bb), j = bb mod P,
// x[q] = src[bb + q*len/p] * W_{P*p}^{j*q}; X0[b] = x[0]; W[b][m] = x[g^m mod p].
template <typename T>
__device__ __forceinline__ void op_rader_gather(const Op &op, cplx<T> *sm) {
    const int pr = op.radix;
    const int NBL = op.len / pr;
    const int NB = op.nsub * NBL;
    const int P = op.P;
    const int tstep = op.len / (P * pr);
    const int *perm = reinterpret_cast<const int *>(op.lut2);
    const int total = NB * pr;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int b = fdiv(f, op.div_c);
        const int m = f - b * pr;
        const int s = op.nsub == 1 ? 0 : (int)fdiv(b, op.div_a);
        const int bb = b - s * NBL;
        const int j = bb - (int)fdiv(bb, op.div_b) * P;
        const int q = m < pr - 1 ? __ldg(perm + m) : 0;
        cplx<T> v = sm[op.src_base + s * op.sub_stride + spad(bb + q * NBL, op.pad_shift)];
        if (P > 1 && q > 0) v = cmul(v, ld_ro<T>(op.lut, j * q * tstep));
        if (m < pr - 1)
            sm[op.w_base + b * op.w_stride + spad(m, op.pad_shift)] = v;
        else
            sm[op.x0_base + 2 * b] = v;
    }
}

// Rader radix-p step, scatter half: y[g^-m] = x0 + c[m], y[0] = x0 + sum(a), written to
// the Stockham output position (bb - j)*p + j + k*P of the dst region.  c is the cyclic
// convolution of a with b[m] = W_p^{g^-m}: read from the W region (FFT mode, after the
// inverse sub-transform; conjugated when F_CONJ_IN) or summed here (F_DIRECT, lut = b).
template <typename T>
__device__ __forceinline__ void op_rader_scatter(const Op &op, cplx<T> *sm) {
    const int pr = op.radix;
    const int NBL = op.len / pr;
    const int NB = op.nsub * NBL;
    const int P = op.P;
    const int *ginv = reinterpret_cast<const int *>(op.lut3);
    const int total = NB * pr;
    const bool direct = op.flags & F_DIRECT;
    const bool conj_in = op.flags & F_CONJ_IN;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int b = fdiv(f, op.div_c);
        const int m = f - b * pr;
        const int s = op.nsub == 1 ? 0 : (int)fdiv(b, op.div_a);
        const int bb = b - s * NBL;
        const int j = bb - (int)fdiv(bb, op.div_b) * P;
        const cplx<T> x0 = sm[op.x0_base + 2 * b];
        const cplx<T> *w = sm + op.w_base + b * op.w_stride;
        cplx<T> acc = {T(0), T(0)};
        int k;
        if (m == pr - 1) {
            k = 0;
            if (direct) {
                for (int q = 0; q < pr - 1; q++) {
                    const cplx<T> a = w[spad(q, op.pad_shift)];
                    acc.x += a.x;
                    acc.y += a.y;
                }
            } else {
                acc = sm[op.x0_base + 2 * b + 1];
            }
        } else {
            k = __ldg(ginv + m);
            if (direct) {
                const int L1 = pr - 1;
                int idx = m;
                for (int q = 0; q < L1; q++) {
                    const cplx<T> a = w[spad(q, op.pad_shift)];
                    const cplx<T> bt = ld_ro<T>(op.lut, idx);
                    acc.x += a.x * bt.x - a.y * bt.y;
                    acc.y += a.x * bt.y + a.y * bt.x;
                    idx = idx == 0 ? L1 - 1 : idx - 1;
                }
            } else {
                acc = w[spad(m, op.pad_shift)];
                if (conj_in) acc = cconj(acc);
            }
        }
        sm[op.dst_base + s * op.sub_stride + spad((bb - j) * pr + j + k * P, op.pad_shift)] = {x0.x + acc.x, x0.y + acc.y};
    }
}

// Hermitian expansion of the src region (lines of length nfull): X[k] = conj(X[N-k])
// for k = N/2+1 .. N-1.
template <typename T>
__device__ __forceinline__ void op_herm_expand(const PassShape &p, const Op &op, cplx<T> *sm) {
    const int n = op.nfull;
    const int lo = n / 2 + 1;
    const int per = n - lo;
    if (per <= 0) return;
    const int total = p.G * per;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int g = f / per;
        const int k = lo + (f - g * per);
        cplx<T> *z = sm + op.src_base + g * op.sub_stride;
        z[spad(k, op.pad_shift)] = cconj(z[spad(n - k, op.pad_shift)]);
    }
}

// Pass-level Rader gather: dst[m] = src[g^m mod p] for m < p-1 and dst[p-1] = src[0]
// (the line layout of the convolution scratch is [a_0 .. a_{p-2}, x0, A0]).
template <typename T>
__device__ __forceinline__ void op_permute_gather(const Op &op, cplx<T> *sm) {
    const int pr = op.radix;
    const int *perm = reinterpret_cast<const int *>(op.lut2);
    const int total = op.nsub * pr;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int g = fdiv(f, op.div_c);
        const int m = f - g * pr;
        const int q = m < pr - 1 ? __ldg(perm + m) : 0;
        sm[op.dst_base + g * op.sub_stride + spad(m, op.pad_shift)] = sm[op.src_base + g * op.sub_stride + spad(q, op.pad_shift)];
    }
}

// line[slot] = line[0] for every line of the src region.
template <typename T>
__device__ __forceinline__ void op_save_dc(const Op &op, cplx<T> *sm) {
    for (int g = threadIdx.x; g < op.nsub; g += B200FFT_NT)
        sm[op.src_base + g * op.sub_stride + spad(op.nfull, op.pad_shift)] = sm[op.src_base + g * op.sub_stride];
}

// Pass-level Rader scatter: from [c_0 .. c_{p-2}, x0, A0] (c conjugated when F_CONJ_IN),
// dst[g^-m] = x0 + c[m], dst[0] = x0 + A0, then F_SCALE / F_CONJ_OUT.
template <typename T>
__device__ __forceinline__ void op_permute_scatter(const Op &op, cplx<T> *sm) {
    const int pr = op.radix;
    const int *ginv = reinterpret_cast<const int *>(op.lut3);
    const int total = op.nsub * pr;
    for (int f = threadIdx.x; f < total; f += B200FFT_NT) {
        const int g = fdiv(f, op.div_c);
        const int m = f - g * pr;
        const cplx<T> *src = sm + op.src_base + g * op.sub_stride;
        const cplx<T> x0 = src[spad(pr - 1, op.pad_shift)];
        cplx<T> acc;
        int k;
        if (m < pr - 1) {
            acc = src[spad(m, op.pad_shift)];
            if (op.flags & F_CONJ_IN) acc = cconj(acc);
            k = __ldg(ginv + m);
        } else {
            acc = src[spad(pr, op.pad_shift)];
            k = 0;
        }
        cplx<T> y = {x0.x + acc.x, x0.y + acc.y};
        if (op.flags & F_SCALE) {
            y.x *= kc<T>(op.scale, op.scale_lo);
            y.y *= kc<T>(op.scale, op.scale_lo);
        }
        if (op.flags & F_CONJ_OUT) y = cconj(y);
        sm[op.dst_base + g * op.sub_stride + spad(k, op.pad_shift)] = y;
    }
}

// Per-thread prologue: copy the op program into shared memory (after the line
// metadata, so the dynamic op index below reads shared memory rather than the
// parameter block) and resolve every line's global base addresses.
template <typename T>
__device__ __forceinline__ LineMeta pass_prologue(const PassShape &p, unsigned char *smem_raw) {
    int64_t *ib = reinterpret_cast<int64_t *>(smem_raw + p.meta_off);
    int64_t *ob = ib + p.G;
    int *col = reinterpret_cast<int *>(ob + p.G);
    int *oidx = col + ((p.G + 3) & ~3);
    const int64_t l0 = (int64_t)blockIdx.x * p.G;
    const int64_t rem = p.nlines - l0;
    LineMeta lm{ib, ob, col, oidx, (int)(rem < p.G ? rem : p.G)};
    for (int g = threadIdx.x; g < p.G; g += B200FFT_NT) {
        int64_t l = l0 + g;
        if (g >= lm.nl) l = l0;  // padding lines: any valid address, never read or written
        const int64_t i = l % p.ni;
        const int64_t t = l / p.ni;
        const int64_t c = t % p.nc;
        const int64_t o = t / p.nc;
        ib[g] = o * p.in.os + i * p.in.is + c * p.in.cs;
        ob[g] = o * p.out.os + i * p.out.is + c * p.out.cs;
        col[g] = (int)c;
        oidx[g] = (int)o;
    }
    return lm;
}

// One op of the program, this thread's share (threads synchronise between ops).
template <typename T>
__device__ __forceinline__ void run_op(const PassShape &p, const Op &op, cplx<T> *sm, const LineMeta &lm) {
    switch (op.type) {
        case OP_LOAD: op_load<T>(p, op, sm, lm); break;
        case OP_STORE: op_store<T>(p, op, sm, lm); break;
        case OP_STAGE: op_stage_dispatch<T>(op, sm, p.err); break;
        case OP_MUL: op_mul<T>(op, sm, lm); break;
        case OP_R2C_POST: op_r2c_post<T>(p, op, sm); break;
        case OP_C2R_PRE: op_c2r_pre<T>(p, op, sm); break;
        case OP_RADER_GATHER: op_rader_gather<T>(op, sm); break;
        case OP_RADER_SCATTER: op_rader_scatter<T>(op, sm); break;
        case OP_HERM_EXPAND: op_herm_expand<T>(p, op, sm); break;
        case OP_PERMUTE_GATHER: op_permute_gather<T>(op, sm); break;
        case OP_PERMUTE_SCATTER: op_permute_scatter<T>(op, sm); break;
        case OP_SAVE_DC: op_save_dc<T>(op, sm); break;
        default: raise_error(p.err, 4); break;
    }
}

}  // namespace b200fft
