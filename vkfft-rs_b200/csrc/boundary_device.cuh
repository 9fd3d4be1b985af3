// Device routines of the element-wise passes: convolution multiply and boundary copy
// (zero padding, formatted strides, storage <-> compute precision).  Included by
// boundary.cu and by the CPU emulator.
#pragma once

#include <cuda_fp16.h>

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
        r = mul(prep(spec[in_s * m.T + i]), ker[kid * m.T + i]);
    }
    if (m.cross_power) {
        const T k = T(1) / sqrt(r.x * r.x + r.y * r.y);
        r.x *= k;
        r.y *= k;
    }
    reinterpret_cast<cplx<T> *>(m.dst)[L] = r;
}

B200FFT_HD double load_scalar(const void *base, int64_t idx, int bytes) {
    if (bytes == 8) return reinterpret_cast<const double *>(base)[idx];
    if (bytes == 4) return reinterpret_cast<const float *>(base)[idx];
    return (double)__half2float(reinterpret_cast<const __half *>(base)[idx]);
}

B200FFT_HD void store_scalar(void *base, int64_t idx, int bytes, double v) {
    if (bytes == 8)
        reinterpret_cast<double *>(base)[idx] = v;
    else if (bytes == 4)
        reinterpret_cast<float *>(base)[idx] = (float)v;
    else
        reinterpret_cast<__half *>(base)[idx] = __float2half_rn((float)v);
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
        const double v = zero ? 0.0 : load_scalar(b.src, so * b.scalars + k, b.src_bytes);
        store_scalar(b.dst, dof * b.scalars + k, b.dst_bytes, v);
    }
}

}  // namespace b200fft
