"""Child-process runner of emulated cases (loaded with the ASan runtime preloaded).

stdin: JSON list of cases {"kind": "c2c"|"r2c"|"c2r", "dims": [...], "batch": b,
"prec": "F32"|"F64", "inverse": bool, "normalize": bool, "tuning": {...}|null,
"seed": s}.  stdout (last line): JSON list of {"err": relL2 vs oracle, "launches": n}
or {"error": "<variant>: message"}."""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

import oracle  # noqa: E402
from __init__ import _load, emulate  # noqa: E402


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.complex128).ravel()
    b = np.asarray(b, dtype=np.complex128).ravel()
    d = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (d if d > 0 else 1.0))


def b200_profile(V):
    return V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA).replace(
        shared_memory_bytes=49152, shared_memory_pow2_bytes=32768, max_threads_per_block=1024,
        max_workgroup_size=[1024, 1024, 64])


def run(case, V, lib):
    if case["kind"] == "dd":
        return run_dd(case, V, lib, b200_profile(V), np.random.default_rng(case.get("seed", 0)))
    dims, batch, prec = case["dims"], case["batch"], case["prec"]
    cdt, rdt = (np.complex64, np.float32) if prec == "F32" else (np.complex128, np.float64)
    dev = b200_profile(V)
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    cfg = cfg.with_inverse_normalization(case.get("normalize", False))
    if case.get("tuning"):
        cfg = cfg.with_tuning(V.PlannerTuning(**case["tuning"]))
    rng = np.random.default_rng(case.get("seed", 0))
    shape = (batch,) + tuple(dims)
    kind = case["kind"]
    if kind == "c2c":
        x = (rng.uniform(-1, 1, shape) + 1j * rng.uniform(-1, 1, shape)).astype(cdt)
        d = V.Direction.INVERSE if case.get("inverse") else V.Direction.FORWARD
        y, n = emulate(V, lib, cfg, d, dev, x, x.size, cdt)
        ref = oracle.fft_nd(x.astype(np.complex128), len(dims), inverse=case.get("inverse", False),
                            normalize=case.get("normalize", False), threads=4)
    elif kind == "r2c":
        x = rng.uniform(-1, 1, shape).astype(rdt)
        cfg = cfg.with_transform(V.TransformKind.R2C)
        ref = oracle.r2c_nd(x.astype(np.float64), len(dims), threads=4)
        y, n = emulate(V, lib, cfg, V.Direction.FORWARD, dev, x, ref.size, cdt)
    elif kind == "conv":
        return run_conv(case, V, lib, dev, cfg, rng, cdt, rdt)
    elif kind == "slab":
        return run_slab(case, V, lib, dev, cfg, rng, cdt, rdt)
    elif kind == "bnd":
        return run_boundary(case, V, lib, dev, cfg, rng, cdt, rdt)
    elif kind == "cconv":
        return run_cconv(case, V, lib, dev, cfg, rng, cdt, rdt)
    elif kind == "mixed":
        # F16 storage / F32 compute, F64 compute / F32 storage: the caller's buffers hold
        # the storage type; results are the compute-precision transform of the quantised
        # input, quantised to the storage type
        store = np.float16 if case["precision"] == "F16_STORAGE_F32_COMPUTE" else np.float32
        cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[case["precision"]])
        real = case.get("real", False)
        if real:
            cfg = cfg.with_transform(V.TransformKind.R2C)
            x = rng.uniform(-1, 1, (batch,) + tuple(dims)).astype(store)
            ref = oracle.r2c_nd(x.astype(np.float64), len(dims), threads=4)
        else:
            x = rng.uniform(-1, 1, (batch,) + tuple(dims) + (2,)).astype(store)
            ref = oracle.fft_nd(x[..., 0].astype(np.float64) + 1j * x[..., 1].astype(np.float64), len(dims),
                                threads=4)
        ref_q = ref.view(np.float64).astype(store).astype(np.float64).view(np.complex128)
        y, n = emulate(V, lib, cfg, V.Direction.FORWARD, dev, x, ref.size * 2, store)
        return {"err": rel_l2(y.astype(np.float64).view(np.complex128), ref_q), "launches": n}
    elif kind == "r2r":
        # DCT / DST (r2r_ir.rs): real in, real out; inverse = partner kind x pair scale
        x = rng.uniform(-1, 1, shape).astype(rdt)
        inverse = case.get("inverse", False)
        cfg = cfg.with_transform(V.TransformKind[case["r2r"]])
        for a, (lo, hi) in case.get("pad", {}).items():
            cfg = cfg.with_zero_padding(int(a), lo, hi)
        for a in case.get("omit", []):
            cfg = cfg.with_omit_dimension(a, True)
        d = V.Direction.INVERSE if inverse else V.Direction.FORWARD
        xin = x.astype(np.float64)
        pads = {int(a): v for a, v in case.get("pad", {}).items()}
        if pads and not inverse:
            xin = xin * _pad_keep(dims, pads)
        ref = oracle.r2r_nd(xin, case["r2r"], len(dims), inverse=inverse, normalize=case.get("normalize", False),
                            omitted=tuple(case.get("omit", [])))
        if pads and inverse:
            ref = ref * _pad_keep(dims, pads)
        y, n = emulate(V, lib, cfg, d, dev, x, ref.size, rdt)
        return {"err": rel_l2(y, ref), "launches": n}
    elif kind == "kprep":
        # kernelConvolution preparation: the forward transform of batch x coordinate systems
        C = case["coords"]
        cfg = cfg.with_kernel_convolution(True).with_coordinate_features(C)
        n = int(np.prod(dims))
        if case.get("real"):
            x = rng.uniform(-1, 1, (batch * C,) + tuple(dims)).astype(rdt)
            cfg = cfg.with_transform(V.TransformKind.R2C)
            ref = oracle.r2c_nd(x.astype(np.float64), len(dims), threads=4)
        else:
            x = (rng.uniform(-1, 1, (batch * C,) + tuple(dims))
                 + 1j * rng.uniform(-1, 1, (batch * C,) + tuple(dims))).astype(cdt)
            ref = oracle.fft_nd(x.astype(np.complex128), len(dims), threads=4)
        y, n = emulate(V, lib, cfg, V.Direction.FORWARD, dev, x, ref.size, cdt)
        return {"err": rel_l2(y, ref), "launches": n}
    else:
        x = rng.uniform(-1, 1, shape)
        spec = oracle.r2c_nd(x, len(dims), threads=4).astype(cdt)
        cfg = cfg.with_transform(V.TransformKind.C2R)
        ref = oracle.c2r_nd(spec.astype(np.complex128), dims[-1], len(dims), normalize=case.get("normalize", False),
                            threads=4)
        y, n = emulate(V, lib, cfg, V.Direction.INVERSE, dev, spec, ref.size, rdt)
    return {"err": rel_l2(y, ref), "launches": n}


def run_conv(case, V, lib, dev, cfg, rng, cdt, rdt):
    import ctypes
    dims = case["dims"]
    C, K = case.get("coords", 1), case.get("kernels", 1)
    copies = case.get("copies", K * C)
    cfg = (cfg.with_transform(V.TransformKind.R2C).with_convolution(True).with_coordinate_features(C)
           .with_convolution_kernel_count(K))
    if case.get("conj"):
        cfg = cfg.with_convolution_conjugation(1)
    if case.get("cross"):
        cfg = cfg.with_cross_power_spectrum_normalization(True)
    x = rng.uniform(-1, 1, (C,) + tuple(dims)).astype(rdt)
    L = int(np.prod(dims[:-1])) * (dims[-1] // 2 + 1)
    ker = (rng.uniform(-1, 1, copies * L) + 1j * rng.uniform(-1, 1, copies * L)).astype(cdt)
    ref = oracle.convolve_nd(x, ker, dims, C, K, case.get("conj", False), case.get("cross", False), threads=4)
    out = np.empty(ref.size, dtype=rdt)
    err = ctypes.create_string_buffer(512)
    launches = ctypes.c_int(0)
    fn = lib.b200fft_emu_convolution_run
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p,
                   ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t,
                   ctypes.c_void_p]
    d = dev._c()
    st = fn(ctypes.addressof(cfg._s), ctypes.addressof(d), ker.ctypes.data, copies, x.ctypes.data, x.nbytes,
            out.ctypes.data, out.nbytes, err, 512, ctypes.addressof(launches))
    if st != 0:
        raise V.VkFftError(st, err.value.decode())
    return {"err": rel_l2(out, ref), "launches": launches.value}


def slab_case_arrays(case, rng, cdt, rdt):
    """Global input / expected output of a slab case, split into the per-rank layouts:
    slabs [D0/P, D1, ...] and pencils [D0, D1/P, ...]."""
    dims, P, mode = case["dims"], case["nranks"], case["mode"]
    norm = case.get("normalize", False)
    D0, D1 = dims[0], dims[1]
    L0, C1 = D0 // P, D1 // P
    slabs = lambda a: np.concatenate([a[g * L0:(g + 1) * L0].ravel() for g in range(P)])
    pencils = lambda a: np.concatenate([a[:, g * C1:(g + 1) * C1].ravel() for g in range(P)])
    if mode == "c2c":
        x = rng.uniform(-1, 1, dims) + 1j * rng.uniform(-1, 1, dims)
        return slabs(x).astype(cdt), pencils(oracle.fft_nd(x, len(dims), threads=4))
    if mode == "c2c_inv":
        x = rng.uniform(-1, 1, dims) + 1j * rng.uniform(-1, 1, dims)
        return pencils(x).astype(cdt), slabs(oracle.fft_nd(x, len(dims), inverse=True, normalize=norm, threads=4))
    if mode == "r2c":
        x = rng.uniform(-1, 1, dims)
        return slabs(x).astype(rdt), pencils(oracle.r2c_nd(x, len(dims), threads=4))
    x = rng.uniform(-1, 1, dims)
    spec = oracle.r2c_nd(x, len(dims), threads=4)
    return (pencils(spec).astype(cdt),
            slabs(oracle.c2r_nd(spec, dims[-1], len(dims), normalize=norm, threads=4)))


def run_slab(case, V, lib, dev, cfg, rng, cdt, rdt):
    import ctypes
    mode = case["mode"]
    direction = V.Direction.INVERSE if mode in ("c2c_inv", "c2r") else V.Direction.FORWARD
    if mode == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
    elif mode == "c2r":
        cfg = cfg.with_transform(V.TransformKind.C2R)
    x, ref = slab_case_arrays(case, rng, cdt, rdt)
    P = case["nranks"]
    out_dt = rdt if mode == "c2r" else cdt
    out = np.empty(ref.size, dtype=out_dt)
    err = ctypes.create_string_buffer(512)
    launches = ctypes.c_int(0)
    fn = lib.b200fft_emu_slab_run
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                   ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_void_p]
    d = dev._c()
    st = fn(ctypes.addressof(cfg._s), int(direction), ctypes.addressof(d), P, x.ctypes.data, x.nbytes // P,
            out.ctypes.data, out.nbytes // P, err, 512, ctypes.addressof(launches))
    if st != 0:
        raise V.VkFftError(st, err.value.decode())
    return {"err": rel_l2(out, ref), "launches": launches.value}


def dd_words(rng, shape, complex_):
    """Random double-double words: hi uniform in [-1, 1], lo a canonical residual."""
    w = 4 if complex_ else 2
    x = np.zeros(tuple(shape) + (w,))
    for k in range(0, w, 2):
        hi = rng.uniform(-1, 1, shape)
        x[..., k] = hi
        x[..., k + 1] = hi * np.ldexp(rng.uniform(-1, 1, shape), -55)
    return x


def run_dd(case, V, lib, dev, rng):
    """Double-double (kind "dd"): mode c2c | r2c | c2r (round trip through r2c) | r2r;
    precision DOUBLE_DOUBLE (float64 words) or DOUBLE_DOUBLE_F64_STORAGE (f64 arrays).
    err = max abs error / (2e-30 * N), the crate's GPU gate (must be <= 1); with f64
    storage the outputs are compared to the oracle rounded to binary64 (relative L2)."""
    dims, batch = case["dims"], case["batch"]
    mode = case.get("mode", "c2c")
    prec = case.get("precision", "DOUBLE_DOUBLE")
    f64s = prec == "DOUBLE_DOUBLE_F64_STORAGE"
    inverse, normalize = case.get("inverse", False), case.get("normalize", False)
    cfg = (V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
           .with_inverse_normalization(normalize))
    if case.get("tuning"):
        cfg = cfg.with_tuning(V.PlannerTuning(**case["tuning"]))
    shape = (batch,) + tuple(dims)
    nd, N = len(dims), int(np.prod(dims))
    half = tuple(dims[:-1]) + (dims[-1] // 2 + 1,)
    d = V.Direction.INVERSE if inverse else V.Direction.FORWARD
    launches = 0

    def run(c, direction, x_words, out_words_shape, complex_in, complex_out):
        nonlocal launches
        if f64s:
            x = x_words[..., 0::2] if complex_in else x_words[..., 0]
            x = np.ascontiguousarray(x)
            y, n = emulate(V, lib, c, direction, dev, x, int(np.prod(out_words_shape)) // 2, np.float64)
            launches += n
            w = np.zeros(out_words_shape)
            w[..., 0::2] = y.reshape(out_words_shape[:-1] + (out_words_shape[-1] // 2,))
            return w
        y, n = emulate(V, lib, c, direction, dev, x_words, int(np.prod(out_words_shape)), np.float64)
        launches += n
        return y.reshape(out_words_shape)

    def quantise(w):  # f64 storage: inputs are binary64
        if f64s:
            w = w.copy()
            w[..., 1::2] = 0.0
        return w

    if mode == "c2c":
        x = quantise(dd_words(rng, shape, True))
        y = run(cfg, d, x, shape + (4,), True, True)
        ref = oracle.dd_fft_nd(x, nd, inverse=inverse, normalize=normalize, threads=4)
    elif mode == "r2c":
        x = quantise(dd_words(rng, shape, False))
        y = run(cfg.with_transform(V.TransformKind.R2C), V.Direction.FORWARD, x, (batch,) + half + (4,), False, True)
        ref = oracle.dd_r2c_nd(x, nd, threads=4)
    elif mode == "c2r":
        x = quantise(dd_words(rng, shape, False))
        spec = run(cfg.with_transform(V.TransformKind.R2C), V.Direction.FORWARD, x, (batch,) + half + (4,), False,
                   True)
        c = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        y = run(c, V.Direction.INVERSE, quantise(spec), shape + (2,), True, False)
        ref = x
    else:
        x = quantise(dd_words(rng, shape, False))
        c = cfg.with_transform(V.TransformKind[case["r2r"]])
        y = run(c, d, x, shape + (2,), False, False)
        ref = oracle.dd_r2r_nd(x, case["r2r"], nd, inverse=inverse, normalize=normalize, threads=4)
    if f64s:
        a = y[..., 0::2].ravel()
        b = ref.reshape(-1, 2).sum(axis=1)
        return {"err": rel_l2(a, b) / 1e-15, "launches": launches}
    return {"err": oracle.dd_max_abs_diff(y, ref) / (2e-30 * N), "launches": launches}


def _pad_keep(dims, pads):
    """1 outside and 0 inside the zero-padding ranges [lo, hi) of the given axes."""
    keep = np.ones(tuple(dims))
    for a, (lo, hi) in pads.items():
        idx = [slice(None)] * len(dims)
        idx[a] = slice(lo, hi)
        keep[tuple(idx)] = 0.0
    return keep


def _pad_mask(dims, pads):
    """True where any padded axis coordinate lies in its [left, right) interval."""
    mask = np.zeros(dims, dtype=bool)
    for axis, (lo, hi) in pads.items():
        idx = [slice(None)] * len(dims)
        idx[int(axis)] = slice(lo, hi)
        mask[tuple(idx)] = True
    return mask


def _resolve(dims, strides, batch_stride):
    """config.rs:1463-1522: per-axis strides (None = dense minimum) and batch stride."""
    st = [1] * len(dims)
    for a in range(len(dims) - 2, -1, -1):
        minimum = st[a + 1] * dims[a + 1]
        st[a] = (strides or {}).get(str(a), minimum)
    return st, (batch_stride or st[0] * dims[0])


def _pack(x, dims, strides, batch_stride, fill):
    st, bs = _resolve(dims, strides, batch_stride)
    batch = x.shape[0]
    phys = np.full(bs * batch, fill, dtype=x.dtype)
    idx = np.indices(dims).reshape(len(dims), -1)
    off = sum(idx[a] * st[a] for a in range(len(dims)))
    for b in range(batch):
        phys[b * bs + off] = x[b].reshape(-1)
    return phys


def _unpack(phys, dims, strides, batch_stride, batch):
    st, bs = _resolve(dims, strides, batch_stride)
    idx = np.indices(dims).reshape(len(dims), -1)
    off = sum(idx[a] * st[a] for a in range(len(dims)))
    return np.stack([phys[b * bs + off].reshape(dims) for b in range(batch)])


def run_boundary(case, V, lib, dev, cfg, rng, cdt, rdt):
    """Zero padding / formatted strides (kind "bnd"): mode c2c | c2c_inv | r2c | c2r."""
    dims, batch, mode = case["dims"], case["batch"], case["mode"]
    pads = case.get("pad", {})
    freq = case.get("domain") == "frequency"
    for axis, (lo, hi) in pads.items():
        cfg = cfg.with_zero_padding(int(axis), lo, hi)
    if freq:
        cfg = cfg.with_zero_padding_domain(V.ZeroPaddingDomain.FREQUENCY)
    for axis, st in (case.get("in_strides") or {}).items():
        cfg = cfg.with_input_buffer_axis_stride(int(axis), st)
    for axis, st in (case.get("out_strides") or {}).items():
        cfg = cfg.with_output_buffer_axis_stride(int(axis), st)
    if case.get("in_batch_stride"):
        cfg = cfg.with_input_buffer_batch_stride(case["in_batch_stride"])
    if case.get("out_batch_stride"):
        cfg = cfg.with_output_buffer_batch_stride(case["out_batch_stride"])
    half = list(dims[:-1]) + [dims[-1] // 2 + 1]
    nd = len(dims)
    shape = (batch,) + tuple(dims)
    mask = _pad_mask(dims, pads) if pads else np.zeros(dims, dtype=bool)
    direction = V.Direction.FORWARD
    if mode in ("c2c", "c2c_inv"):
        x = rng.uniform(-1, 1, shape) + 1j * rng.uniform(-1, 1, shape)
        inv = mode == "c2c_inv"
        direction = V.Direction.INVERSE if inv else V.Direction.FORWARD
        pad_in = bool(pads) and (freq == inv)
        xi = np.where(mask, 0, x) if pad_in else x
        ref = oracle.fft_nd(xi, nd, inverse=inv, normalize=case.get("normalize", False), threads=4)
        if pads and not pad_in:
            ref = np.where(mask, 0, ref)
        in_dims, out_dims, in_dt, out_dt = dims, dims, cdt, cdt
    elif mode == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
        x = rng.uniform(-1, 1, shape)
        ref = oracle.r2c_nd(np.where(mask, 0, x), nd, threads=4)
        in_dims, out_dims, in_dt, out_dt = dims, half, rdt, cdt
    else:
        cfg = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        direction = V.Direction.INVERSE
        x = oracle.r2c_nd(rng.uniform(-1, 1, shape), nd, threads=4)
        ref = np.where(mask, 0, oracle.c2r_nd(x, dims[-1], nd, normalize=True, threads=4))
        in_dims, out_dims, in_dt, out_dt = half, dims, cdt, rdt
    phys_in = _pack(np.asarray(x).astype(in_dt), in_dims, case.get("in_strides"), case.get("in_batch_stride"),
                    in_dt(7.0))
    st, bs = _resolve(out_dims, case.get("out_strides"), case.get("out_batch_stride"))
    y, n = emulate(V, lib, cfg, direction, dev, phys_in, bs * batch, out_dt)
    got = _unpack(y, out_dims, case.get("out_strides"), case.get("out_batch_stride"), batch)
    return {"err": rel_l2(got, ref), "launches": n}


def run_cconv(case, V, lib, dev, cfg, rng, cdt, rdt):
    """C2C convolution (kind "cconv"): batch, coords, kernels, matrix, symmetric, conj, cross."""
    import ctypes
    dims, B = case["dims"], case["batch"]
    M, K = case.get("matrix", 0), case.get("kernels", 1)
    C = M if M else case.get("coords", 1)
    sym = case.get("symmetric", False)
    cfg = cfg.with_convolution(True).with_convolution_kernel_count(K)
    if M:
        cfg = cfg.with_matrix_convolution(M)
        if sym:
            cfg = cfg.with_symmetric_convolution_kernel(True)
    elif C > 1:
        cfg = cfg.with_coordinate_features(C)
    if case.get("conj"):
        cfg = cfg.with_convolution_conjugation(1)
    if case.get("cross"):
        cfg = cfg.with_cross_power_spectrum_normalization(True)
    T = int(np.prod(dims))
    planes = (M * (M + 1) // 2 if sym else M * M) if M else 1
    x = (rng.uniform(-1, 1, (B * C,) + tuple(dims)) + 1j * rng.uniform(-1, 1, (B * C,) + tuple(dims))).astype(cdt)
    ker = (rng.uniform(-1, 1, planes * K * T) + 1j * rng.uniform(-1, 1, planes * K * T)).astype(cdt)
    ref = oracle.convolve_c2c(x, ker, dims, B, C, K, M, sym, case.get("conj", False), case.get("cross", False),
                              threads=4)
    out = np.empty(ref.size, dtype=cdt)
    err = ctypes.create_string_buffer(512)
    launches = ctypes.c_int(0)
    fn = lib.b200fft_emu_convolution_run
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p,
                   ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_char_p, ctypes.c_size_t,
                   ctypes.c_void_p]
    d = dev._c()
    st = fn(ctypes.addressof(cfg._s), ctypes.addressof(d), ker.ctypes.data, planes * K, x.ctypes.data, x.nbytes,
            out.ctypes.data, out.nbytes, err, 512, ctypes.addressof(launches))
    if st != 0:
        raise V.VkFftError(st, err.value.decode())
    return {"err": rel_l2(out, ref), "launches": launches.value}


def main():
    cases = json.loads(sys.stdin.read())
    V, lib = _load()
    out = []
    for c in cases:
        try:
            out.append(run(c, V, lib))
        except V.VkFftError as e:
            out.append({"error": f"{e.variant}: {e}"})
    print(json.dumps(out))


if __name__ == "__main__":
    main()
