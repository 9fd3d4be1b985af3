// Device routines of the element-wise passes: convolution multiply, boundary copy
// (zero padding, formatted strides, storage <-> compute precision) and the DCT/DST
// pre/post passes.  Included by boundary.cu and by the CPU emulator.
#pragma once

#include <cuda_fp16.h>

#include <cmath>

#include "pass_device.cuh"

namespace b200fft {

// Kernel plane of a (output, input) coordinate pair (convolution_ir.rs:127-149).
B200FFT_HD int conv_plane(int M, bool symmetric, int oc, int ic) {
    if (!symmetric) return oc * M + ic;
    return ic < oc ? ic * M - ic * ic + oc : oc * M - oc * oc + ic;
}

// One output element of a convolution multiply (pass_desc.hpp ConvMultiply).
template <typename T>
B200FFT_HD void conv_multiply_one(const ConvMultiply &m, int64_t L) {
    const int64_t i = L % m.T;
    const int64_t sc = L / m.T;
    const int oc = (int)(sc % m.C);
    const int64_t s = sc / m.C;
    const int64_t in_s = m.K > 1 ? 0 : s, kid = m.K > 1 ? s : 0;
    const cplx<T> *spec = reinterpret_cast<const cplx<T> *>(m.src);
    const cplx<T> *ker = reinterpret_cast<const cplx<T> *>(m.ker);
    auto prep = [&](cplx<T> v) { return m.conj_seq ? cplx<T>{v.x, -v.y} : v; };
    auto mul = [](cplx<T> a, cplx<T> b) { return cplx<T>{a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x}; };
    cplx<T> r;
    if (m.matrix) {
        r = {T(0), T(0)};
        for (int ic = 0; ic < m.C; ic++) {
            const cplx<T> p = mul(prep(spec[(in_s * m.C + ic) * m.T + i]),
                                  ker[(kid * m.planes + conv_plane(m.matrix, m.symmetric != 0, oc, ic)) * m.T + i]);
            r.x += p.x;
            r.y += p.y;
        }
    } else {
        const int64_t kt = m.shared_kernel ? 0 : kid * m.C + oc;
        r = mul(prep(spec[(in_s * m.C + oc) * m.T + i]), ker[kt * m.T + i]);
    }
    if (m.cross_power) {
        const T k = T(1) / sqrt(r.x * r.x + r.y * r.y);
        r.x *= k;
        r.y *= k;
    }
    reinterpret_cast<cplx<T> *>(m.dst)[L] = r;
}

// One stored scalar as a double-double value (lo = 0 unless the storage is
// double-double, 16 bytes: hi then lo) and its store, rounded to the storage type.
B200FFT_HD dd load_scalar(const void *base, int64_t idx, int bytes) {
    if (bytes == 16) {
        const double *q = reinterpret_cast<const double *>(base) + 2 * idx;
        return dd(q[0], q[1]);
    }
    if (bytes == 8) return dd(reinterpret_cast<const double *>(base)[idx]);
    if (bytes == 4) return dd((double)reinterpret_cast<const float *>(base)[idx]);
    return dd((double)__half2float(reinterpret_cast<const __half *>(base)[idx]));
}

B200FFT_HD void store_scalar(void *base, int64_t idx, int bytes, dd v) {
    if (bytes == 16) {
        double *q = reinterpret_cast<double *>(base) + 2 * idx;
        q[0] = v.hi;
        q[1] = v.lo;
    } else if (bytes == 8) {
        reinterpret_cast<double *>(base)[idx] = v.hi + v.lo;
    } else if (bytes == 4) {
        reinterpret_cast<float *>(base)[idx] = (float)v.hi;
    } else {
        reinterpret_cast<__half *>(base)[idx] = __float2half_rn((float)v.hi);
    }
}

// One element of a boundary copy (pass_desc.hpp BoundaryCopy).
B200FFT_HD void boundary_copy_one(const BoundaryCopy &b, int64_t L) {
    int64_t so = 0, dof = 0;
    bool zero = false;
    for (int a = b.rank - 1; a >= 0; a--) {
        const int64_t c = L % b.dims[a];
        L /= b.dims[a];
        so += c * b.src_stride[a];
        dof += c * b.dst_stride[a];
        zero |= c >= b.pad_lo[a] && c < b.pad_hi[a];
    }
    so += L * b.src_batch;
    dof += L * b.dst_batch;
    const int eb = b.src_bytes * b.scalars;
    if (b.src_bytes == b.dst_bytes && eb >= 4) {  // plain copy
        if (eb == 16) {
            double2 v = zero ? double2{0.0, 0.0} : reinterpret_cast<const double2 *>(b.src)[so];
            reinterpret_cast<double2 *>(b.dst)[dof] = v;
        } else if (eb == 8) {
            unsigned long long v = zero ? 0ull : reinterpret_cast<const unsigned long long *>(b.src)[so];
            reinterpret_cast<unsigned long long *>(b.dst)[dof] = v;
        } else {
            unsigned v = zero ? 0u : reinterpret_cast<const unsigned *>(b.src)[so];
            reinterpret_cast<unsigned *>(b.dst)[dof] = v;
        }
        return;
    }
    for (int k = 0; k < b.scalars; k++) {  // storage <-> compute precision
        const dd v = zero ? dd(0.0) : load_scalar(b.src, so * b.scalars + k, b.src_bytes);
        store_scalar(b.dst, dof * b.scalars + k, b.dst_bytes, v);
    }
}

template <typename T>
B200FFT_HD cplx<T> r2r_cmul(cplx<T> a, cplx<T> b) {
    return cplx<T>{a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x};
}

template <typename T>
B200FFT_HD cplx<T> r2r_tab(const R2rPass &r, int64_t idx) {
    return reinterpret_cast<const cplx<T> *>(r.tb)[idx];
}

// One element of an R2R pre pass (real tensor -> complex work array) or post pass
// (FFT output -> real tensor); the algebra of reg_kernels.cu r2r_load_all /
// r2r_store_all, with the twiddles from the per-position table r.tb = [A | B].
template <typename T>
B200FFT_HD void r2r_one(const R2rPass &r, int64_t t) {
    const int64_t n = r.n, L = r.L, inner = r.inner;
    const int64_t i = t % inner;
    const int64_t rest = t / inner;
    const bool dst = r.kind >= 4;
    const int type = r.kind & 3;  // 0..3 = I..IV
    if (r.pre) {
        const int64_t m = rest % L, o = rest / L;
        const T *x = reinterpret_cast<const T *>(r.src) + o * n * inner + i;
        auto at = [&](int64_t j) { return x[j * inner]; };
        cplx<T> v{T(0), T(0)};
        if (type == 0) {
            if (!dst)
                v.x = m < n ? at(m) : at(L - m);
            else if (m != 0 && m != n + 1)
                v.x = m <= n ? at(m - 1) : -at(L - m - 1);
        } else if (type == 1) {
            const int64_t split = (n + 1) / 2;
            const int64_t s = m < split ? 2 * m : 2 * (n - m) - 1;
            v.x = (dst && (s & 1)) ? -at(s) : at(s);
        } else if (type == 2) {
            const T a = dst ? at(n - 1 - m) : at(m);
            const T b = m == 0 ? T(0) : (dst ? at(m - 1) : at(n - m));
            v = r2r_cmul(cplx<T>{a, -b}, r2r_tab<T>(r, m));
        } else if ((n & 1) == 0) {
            const T a = at(2 * m), b = at(n - 1 - 2 * m);
            v = r2r_cmul(cplx<T>{a, dst ? b : -b}, r2r_tab<T>(r, m));
        } else if (m < n) {
            const cplx<T> w = r2r_tab<T>(r, m);
            const T a = at(m);
            v = cplx<T>{a * w.x, a * w.y};
        }
        reinterpret_cast<cplx<T> *>(r.dst)[(o * L + m) * inner + i] = v;
    } else {
        const int64_t k = rest % n, o = rest / n;
        const cplx<T> *Y = reinterpret_cast<const cplx<T> *>(r.src) + o * L * inner + i;
        auto at = [&](int64_t j) { return Y[j * inner]; };
        T v;
        if (type == 0) {
            v = dst ? -at(k + 1).y : at(k).x;
        } else if (type == 1) {
            const int64_t q = dst ? n - 1 - k : k;
            v = T(2) * r2r_cmul(at(q), r2r_tab<T>(r, q)).x;
        } else if (type == 2) {
            v = at((k & 1) == 0 ? k / 2 : n - 1 - k / 2).x;
            if (dst && (k & 1)) v = -v;
        } else if ((n & 1) == 0) {
            // k even: Y[k/2] conj(B[k/2]); k odd: conj(Y[p]) i B[p], p = L - (k+1)/2
            cplx<T> rot;
            if ((k & 1) == 0) {
                const cplx<T> z = r2r_tab<T>(r, L + k / 2);
                rot = r2r_cmul(at(k / 2), cplx<T>{z.x, -z.y});
            } else {
                const int64_t p = L - (k + 1) / 2;
                const cplx<T> z = r2r_tab<T>(r, L + p);
                const cplx<T> y = at(p);
                rot = r2r_cmul(cplx<T>{y.x, -y.y}, cplx<T>{-z.y, z.x});
            }
            v = T(2) * (dst ? rot.y : rot.x);
        } else {
            const cplx<T> rot = r2r_cmul(at(k), r2r_tab<T>(r, L + k));
            v = T(2) * (dst ? -rot.y : rot.x);
        }
        reinterpret_cast<T *>(r.dst)[(o * n + k) * inner + i] = v * kc<T>(r.scale, r.scale_lo);
    }
}

}  // namespace b200fft
