"""numpy front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Wraps ``liboracle.so`` (a C restatement of vkfft-rs ``src/reference.rs``; see
``reference_oracle.c`` for the line-by-line citations).  Imported by the test
suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
arm, always as the checker or the timed CPU reference, never by the product.

ND transforms apply the 1D oracle along every axis, fastest axis first, as the
reference's separable ND path does (nd_ir.rs:671-673, :1303-1338).  R2C keeps
the first n/2+1 bins of the complex FFT of (x, 0); C2R expands the Hermitian
half spectrum and keeps the real part (real_ir.rs:1037-1053).
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build():
    """Compile liboracle.so with the committed Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        l = ctypes.CDLL(_LIB_PATH)
        dp = ctypes.POINTER(ctypes.c_double)
        sz = ctypes.c_size_t
        ci = ctypes.c_int
        l.oracle_fft.argtypes = [dp, dp, sz, ci, ci]
        l.oracle_dft.argtypes = [dp, dp, sz, ci, ci]
        l.oracle_fft_axis.argtypes = [dp, dp, sz, sz, sz, ci, ci, ci]
        l.oracle_fft_batch.argtypes = [dp, dp, sz, sz, ci, ci, ci]
        l.oracle_r2c_batch.argtypes = [dp, dp, sz, sz, ci]
        l.oracle_c2r_batch.argtypes = [dp, dp, sz, sz, ci, ci]
        l.oracle_dd_dft_lines.argtypes = [dp, dp, sz, sz, ci, ci, ci]
        l.oracle_dd_r2r_lines.argtypes = [dp, dp, sz, sz, ci, ci, ci, ci]
        l.oracle_dd_dft_lines.restype = ci
        l.oracle_dd_r2r_lines.restype = ci
        l.oracle_next_smooth_at_least.argtypes = [sz]
        l.oracle_next_smooth_at_least.restype = sz
        for f in (l.oracle_fft, l.oracle_dft, l.oracle_fft_axis, l.oracle_fft_batch,
                  l.oracle_r2c_batch, l.oracle_c2r_batch):
            f.restype = ci
        _lib = l
    return _lib


def _dp(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def default_threads():
    return max(1, os.cpu_count() or 1)


def fft(x, inverse=False, normalize=False):
    """1D C2C of one sequence, complex128 in/out (reference::fft)."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    out = np.empty_like(x)
    if lib().oracle_fft(_dp(x), _dp(out), x.size, int(inverse), int(normalize)) != 0:
        raise RuntimeError("oracle fft failed")
    return out


def dft(x, inverse=False, normalize=False):
    """O(n^2) direct DFT (reference::dft)."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    out = np.empty_like(x)
    lib().oracle_dft(_dp(x), _dp(out), x.size, int(inverse), int(normalize))
    return out


def fft_axis(x, axis, inverse=False, normalize=False, threads=None):
    """C2C along one axis of a dense complex128 array (returns a new array)."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    out = np.empty_like(x)
    shape = x.shape
    outer = int(np.prod(shape[:axis], dtype=np.int64))
    inner = int(np.prod(shape[axis + 1:], dtype=np.int64))
    rc = lib().oracle_fft_axis(_dp(x), _dp(out), outer, shape[axis], inner, int(inverse),
                               int(normalize), threads or default_threads())
    if rc != 0:
        raise RuntimeError("oracle fft_axis failed")
    return out


def fft_nd(x, ndim, inverse=False, normalize=False, threads=None):
    """Separable C2C over the last ``ndim`` axes (leading axes are batch)."""
    y = np.ascontiguousarray(x, dtype=np.complex128)
    for axis in range(y.ndim - 1, y.ndim - 1 - ndim, -1):
        y = fft_axis(y, axis, inverse, normalize, threads)
    return y


def r2c(x, threads=None):
    """Batched R2C along the last axis: (..., n) float64 -> (..., n//2+1) complex128."""
    x = np.ascontiguousarray(x, dtype=np.float64)
    n = x.shape[-1]
    batch = x.size // n
    out = np.empty(x.shape[:-1] + (n // 2 + 1,), dtype=np.complex128)
    if lib().oracle_r2c_batch(_dp(x), _dp(out), n, batch, threads or default_threads()) != 0:
        raise RuntimeError("oracle r2c failed")
    return out


def c2r(x, n, normalize=False, threads=None):
    """Batched C2R along the last axis: (..., n//2+1) complex128 -> (..., n) float64."""
    x = np.ascontiguousarray(x, dtype=np.complex128)
    batch = x.size // (n // 2 + 1)
    out = np.empty(x.shape[:-1] + (n,), dtype=np.float64)
    if lib().oracle_c2r_batch(_dp(x), _dp(out), n, batch, int(normalize),
                              threads or default_threads()) != 0:
        raise RuntimeError("oracle c2r failed")
    return out


def r2c_nd(x, ndim, threads=None):
    """ND R2C: real axis on the fastest dim, then complex axes on the compact shape
    (nd_real_ir.rs:21-41)."""
    y = r2c(x, threads)
    for axis in range(y.ndim - 2, y.ndim - 1 - ndim, -1):
        y = fft_axis(y, axis, False, False, threads)
    return y


def c2r_nd(x, shape_last, ndim, normalize=False, threads=None):
    """ND C2R: complex inverse axes on the compact shape, then C2R on the fastest."""
    y = np.ascontiguousarray(x, dtype=np.complex128)
    for axis in range(y.ndim - 1 - ndim + 1, y.ndim - 1):
        y = fft_axis(y, axis, True, normalize, threads)
    return c2r(y, shape_last, normalize, threads)


def next_smooth_at_least(target):
    return int(lib().oracle_next_smooth_at_least(target))


def convolve_nd(x, kernel_spectrum, dims, coordinates=1, kernels=1, conjugate_sequence=False,
                cross_power=False, matrix=0, symmetric=False, pads=None, threads=None):
    """ND real FFT convolution (NdRealConvolutionIr, execute_nd_real_convolution_ir,
    convolution_ir.rs:4192-4250): R2C of the ``coordinates`` images (each masked to zero on
    the padding intervals ``pads`` {axis: (lo, hi)} first, the forward zero-pad pass), per
    output system the product -- independent / scalar: policy(seq[c]) * kernel[k*C + c];
    matrix (``matrix`` = 2 or 3 coordinates): sum over ic of prep(seq[ic]) *
    kernel[k*planes + plane(oc, ic)] then the cross-power normalisation -- then a normalised
    C2R of the K*C systems, masked on the padding intervals (the inverse zero-pad pass).
    Sequence conjugation and cross-power normalisation p / |p| as vulkan.rs:17846-17873
    emits them.  ``kernel_spectrum`` holds the reference layout (K*C, or K*planes for a
    matrix, compact spectra) or, for independent coordinates, one spectrum every system
    shares."""
    dims = tuple(dims)
    C, K = coordinates, kernels
    mask = None
    if pads:
        mask = np.zeros(dims, dtype=bool)
        for axis, (lo, hi) in pads.items():
            idx = [slice(None)] * len(dims)
            idx[int(axis)] = slice(lo, hi)
            mask[tuple(idx)] = True
    xr = np.asarray(x, dtype=np.float64).reshape((C,) + dims)
    if mask is not None:
        xr = np.where(mask, 0.0, xr)
    seq = r2c_nd(xr, len(dims), threads=threads)
    seq = seq.reshape(C, -1)
    L = seq.shape[1]
    ker = np.asarray(kernel_spectrum, dtype=np.complex128).reshape(-1, L)
    prep = (lambda v: np.conj(v)) if conjugate_sequence else (lambda v: v)
    norm = (lambda p: p / np.sqrt(p.real * p.real + p.imag * p.imag)) if cross_power else (lambda p: p)
    out = np.empty((K * C, L), dtype=np.complex128)
    if matrix:
        planes = matrix * (matrix + 1) // 2 if symmetric else matrix * matrix
        for k in range(K):
            for oc in range(matrix):
                acc = np.zeros(L, dtype=np.complex128)
                for ic in range(matrix):
                    acc += prep(seq[ic]) * ker[k * planes + conv_plane(matrix, symmetric, oc, ic)]
                out[k * matrix + oc] = norm(acc)
    else:
        for k in range(K):
            for c in range(C):
                out[k * C + c] = norm(prep(seq[c]) * (ker[k * C + c] if ker.shape[0] > 1 else ker[0]))
    half = dims[:-1] + (dims[-1] // 2 + 1,)
    y = c2r_nd(out.reshape((K * C,) + half), dims[-1], len(dims), normalize=True, threads=threads)
    if mask is not None:
        y = np.where(mask, 0.0, y)
    return y


def conv_plane(m, symmetric, oc, ic):
    """ConvolutionMatrixLayout::kernel_plane_index (convolution_ir.rs:127-149)."""
    if not symmetric:
        return oc * m + ic
    return ic * m - ic * ic + oc if ic < oc else oc * m - oc * oc + ic


def convolve_c2c(x, kernel_spectrum, dims, batch=1, coordinates=1, kernels=1, matrix=0, symmetric=False,
                 conjugate_sequence=False, cross_power=False, threads=None):
    """C2C FFT convolution (execute_convolution_ir / execute_nd_convolution_ir,
    convolution_ir.rs:4252-4440): forward FFT of the batch x coordinate systems, the
    scalar / K-kernel / matrix multiply with the sequence-conjugation and cross-power
    policy, normalised inverse FFT of the output systems."""
    dims = tuple(dims)
    T = int(np.prod(dims))
    C = matrix if matrix else coordinates
    spec = fft_nd(np.asarray(x, dtype=np.complex128).reshape((batch * C,) + dims), len(dims), threads=threads)
    spec = spec.reshape(batch * C, T)
    ker = np.asarray(kernel_spectrum, dtype=np.complex128).reshape(-1, T)
    planes = (matrix * (matrix + 1) // 2 if symmetric else matrix * matrix) if matrix else 1
    out_systems = kernels if kernels > 1 else batch
    prep = (lambda v: np.conj(v)) if conjugate_sequence else (lambda v: v)
    norm = (lambda p: p / np.sqrt(p.real * p.real + p.imag * p.imag)) if cross_power else (lambda p: p)
    out = np.empty((out_systems * C, T), dtype=np.complex128)
    for s in range(out_systems):
        in_s, kid = (0, s) if kernels > 1 else (s, 0)
        for oc in range(C):
            if matrix:
                acc = np.zeros(T, dtype=np.complex128)
                for ic in range(C):
                    acc += prep(spec[in_s * C + ic]) * ker[kid * planes + conv_plane(matrix, symmetric, oc, ic)]
                out[s * C + oc] = norm(acc)
            else:
                out[s * C + oc] = norm(prep(spec[in_s * C + oc]) * ker[kid])
    return fft_nd(out.reshape((out_systems * C,) + dims), len(dims), inverse=True, normalize=True, threads=threads)


# ---- DCT / DST ----------------------------------------------------------------------
# The eight FFTW real-to-real kinds as the reference's direct evaluator states them
# (r2r_ir.rs:2351-2433, evaluate_bin): REDFT00/10/01/11 = DCT-I..IV, RODFT00/10/01/11 =
# DST-I..IV, unnormalised.  The inverse direction evaluates the inverse partner
# (II <-> III, the others self, r2r_ir.rs:2317-2325) and, with normalisation, scales
# by inverse_pair_scale (r2r_ir.rs:2327-2349).  Each bin is a direct O(N) sum; the
# trigonometric arguments are reduced exactly in integers before the cosine/sine.
R2R_KINDS = ("DCT1", "DCT2", "DCT3", "DCT4", "DST1", "DST2", "DST3", "DST4")


def _trig(fn, num, den):
    """fn(pi * num / den) with num reduced modulo 2 * den first."""
    num = np.mod(num, 2 * den)
    return fn(np.pi * num / den)


def r2r_matrix(kind, n):
    """n x n matrix of one unnormalised FFTW R2R kind (r2r_ir.rs:2351-2433)."""
    k = np.arange(n, dtype=np.int64)[:, None]
    j = np.arange(n, dtype=np.int64)[None, :]
    alt = np.where(k % 2 == 0, 1.0, -1.0)[:, 0]
    if kind == "DCT1":
        if n < 2:
            raise ValueError("DCT-I needs n >= 2")
        m = 2.0 * _trig(np.cos, j * k, n - 1)
        m[:, 0] = 1.0
        m[:, n - 1] = alt
    elif kind == "DCT2":
        m = 2.0 * _trig(np.cos, (2 * j + 1) * k, 2 * n)
    elif kind == "DCT3":
        m = 2.0 * _trig(np.cos, j * (2 * k + 1), 2 * n)
        m[:, 0] = 1.0
    elif kind == "DCT4":
        m = 2.0 * _trig(np.cos, (2 * j + 1) * (2 * k + 1), 4 * n)
    elif kind == "DST1":
        m = 2.0 * _trig(np.sin, (j + 1) * (k + 1), n + 1)
    elif kind == "DST2":
        m = 2.0 * _trig(np.sin, (2 * j + 1) * (k + 1), 2 * n)
    elif kind == "DST3":
        m = 2.0 * _trig(np.sin, (j + 1) * (2 * k + 1), 2 * n)
        m[:, n - 1] = alt
    elif kind == "DST4":
        m = 2.0 * _trig(np.sin, (2 * j + 1) * (2 * k + 1), 4 * n)
    else:
        raise ValueError(kind)
    return m


def r2r_inverse_partner(kind):
    return {"DCT2": "DCT3", "DCT3": "DCT2", "DST2": "DST3", "DST3": "DST2"}.get(kind, kind)


def r2r_inverse_pair_scale(kind, n):
    if kind == "DCT1":
        return 1.0 / (2 * (n - 1))
    if kind == "DST1":
        return 1.0 / (2 * (n + 1))
    return 1.0 / (2 * n)


def r2r_nd(x, kind, ndim, inverse=False, normalize=False, omitted=()):
    """DCT/DST over the last ``ndim`` axes of ``x`` (leading axes are batch): the 1D
    definition applied along every non-omitted axis (NdR2rIr, r2r_ir.rs:1795-2017)."""
    x = np.asarray(x, dtype=np.float64)
    eff = r2r_inverse_partner(kind) if inverse else kind
    for a in range(ndim):
        if a in omitted:
            continue
        axis = x.ndim - ndim + a
        n = x.shape[axis]
        m = r2r_matrix(eff, n)
        if inverse and normalize:
            m = m * r2r_inverse_pair_scale(kind, n)
        x = np.moveaxis(np.tensordot(m, np.moveaxis(x, axis, 0), axes=(1, 0)), 0, axis)
    return x


# ---- double-double ---------------------------------------------------------------------
# Double-double arrays are float64 words: (..., 2) = (hi, lo) per real value and
# (..., 4) = (re.hi, re.lo, im.hi, im.lo) per complex value, the crate's DD buffer layout
# (double_double.rs encode_complex_double_double).  The transforms are direct binary128
# DFTs / DCT-DST sums with Kahan summation, rounded to hi + lo (dd_oracle.c), the method
# the crate's double-double golden vectors were generated with.

def _dd_along(words, axis, ndim_words, fn):
    """Apply fn(lines_array (lines, n, W)) along `axis` of a (..., n, ..., W) word array."""
    x = np.moveaxis(np.asarray(words, dtype=np.float64), axis, -2)
    shape = x.shape
    lines = int(np.prod(shape[:-2])) if len(shape) > 2 else 1
    y = fn(np.ascontiguousarray(x.reshape(lines, shape[-2], ndim_words)))
    return np.moveaxis(y.reshape(shape[:-2] + y.shape[-2:]), -2, axis)


def dd_fft_nd(words, ndim, inverse=False, normalize=False, threads=None):
    """Complex double-double DFT over the last `ndim` tensor axes of words (..., 4)."""
    x = np.asarray(words, dtype=np.float64)
    t = threads or default_threads()
    for a in range(ndim):
        axis = x.ndim - 1 - ndim + a

        def run(lines):
            out = np.empty_like(lines)
            rc = lib().oracle_dd_dft_lines(_dp(lines), _dp(out), lines.shape[1], lines.shape[0], int(inverse),
                                           int(normalize), t)
            assert rc == 0
            return out
        x = _dd_along(x, axis, 4, run)
    return x


def dd_r2c_nd(words, ndim, threads=None):
    """R2C of real double-double words (..., 2): the first n/2+1 bins of the last axis of
    the complex DFT of (x, 0)."""
    r = np.asarray(words, dtype=np.float64)
    c = np.zeros(r.shape[:-1] + (4,))
    c[..., 0:2] = r
    full = dd_fft_nd(c, ndim, threads=threads)
    n = r.shape[-2]
    return full[..., : n // 2 + 1, :]


def dd_r2r_nd(words, kind, ndim, inverse=False, normalize=False, threads=None):
    """DCT/DST of real double-double words (..., 2) over the last `ndim` axes."""
    x = np.asarray(words, dtype=np.float64)
    t = threads or default_threads()
    k = R2R_KINDS.index(kind)
    for a in range(ndim):
        axis = x.ndim - 1 - ndim + a

        def run(lines):
            out = np.empty_like(lines)
            rc = lib().oracle_dd_r2r_lines(_dp(lines), _dp(out), lines.shape[1], lines.shape[0], k, int(inverse),
                                           int(normalize), t)
            assert rc == 0
            return out
        x = _dd_along(x, axis, 2, run)
    return x


def dd_max_abs_diff(a, b):
    """max |a - b| over double-double words (pairs (hi, lo) on the last axis, any width)."""
    a = np.asarray(a, dtype=np.float64).reshape(-1, 2)
    b = np.asarray(b, dtype=np.float64).reshape(-1, 2)
    return float(np.max(np.abs((a[:, 0] - b[:, 0]) + (a[:, 1] - b[:, 1])))) if a.size else 0.0
