"""GPU parity: the B200 kernels, called through the C ABI, against the CPU oracle
(a restatement of vkfft-rs src/reference.rs) on identical seeded inputs.

Tolerances: relative L2 <= 2e-6 for f32 compute, <= 1e-13 for f64.
FFTW golden vectors are also checked at the reference's own GPU tolerances
(tests/fftw_medium_golden.rs:161-171: f64 1e-8*n, f32 1e-4*n max abs)."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2, uniform_complex

pytestmark = pytest.mark.gpu

TOL = {"F32": 2e-6, "F64": 1e-13}
NP = {"F32": (np.complex64, np.float32), "F64": (np.complex128, np.float64)}


def run_c2c(V, ctx, dims, batch, prec, direction, normalize=False, tuning=None, seed=0):
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    cfg = cfg.with_inverse_normalization(normalize)
    if tuning is not None:
        cfg = cfg.with_tuning(tuning)
    ir = V.TransformIr.build(cfg, direction, ctx.device_profile())
    rng = np.random.default_rng(seed)
    x = uniform_complex(rng, (batch,) + tuple(dims), NP[prec][0])
    y = ctx.execute_transform(ir, x).reshape(x.shape)
    ref = oracle.fft_nd(x.astype(np.complex128), len(dims), inverse=direction == V.Direction.INVERSE,
                        normalize=normalize)
    return ir, rel_l2(y, ref)


C2C_1D = [
    # (N, batch): BASELINE config 1 (1024 x 8) plus radix / Rader / Bluestein coverage
    (1024, 8), (4096, 64), (8, 16), (16, 8), (64, 33), (100, 7), (360, 5), (1000, 3), (1536, 4), (2048, 4),
    (3 ** 7, 2), (5 ** 5, 2), (7 ** 4, 2), (11 * 13 * 16, 2), (17, 64), (47, 32), (257, 8), (89, 16),
    (4099, 6), (83 * 4, 4), (17 * 17, 3), (1, 5), (2, 9),
]


@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("n,batch", C2C_1D)
def test_c2c_1d_forward(V, ctx, n, batch, prec):
    ir, err = run_c2c(V, ctx, [n], batch, prec, V.Direction.FORWARD, seed=n)
    assert err <= TOL[prec], (ir.axis_child(0), err)


@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("n,batch", [(1024, 8), (17, 16), (4099, 3), (360, 4), (47, 8), (131072, 2)])
def test_c2c_1d_inverse_normalized(V, ctx, n, batch, prec):
    ir, err = run_c2c(V, ctx, [n], batch, prec, V.Direction.INVERSE, normalize=True, seed=n + 1)
    assert err <= TOL[prec], (ir.axis_child(0), err)


@pytest.mark.parametrize("prec", ["F32", "F64"])
def test_c2c_large_four_step_and_bluestein_multipass(V, ctx, prec):
    # 2^17 and 2^19 (four-step; 2^19 is the reference's published large case) and the
    # BASELINE Bluestein N=65537 (device M=131220, three passes)
    for n, batch in ((131072, 3), (524288, 2), (65537, 2)):
        ir, err = run_c2c(V, ctx, [n], batch, prec, V.Direction.FORWARD, seed=7)
        assert err <= TOL[prec], (n, ir.axis_child(0), err)


def check_against_oracle_and_exact(y, x, prec, inverse=False, normalize=False, ndim=1):
    """f64 lengths whose prime-free part the reference's CPU path computes by Bluestein
    carry that path's unreduced-chirp error (8e-13 at 4099, 1e-11 at 83*1009); an exact
    planned algorithm (Rader) cannot reproduce it.  Check the result against an exact DFT
    at the f64 tolerance and against the oracle within the oracle's own measured error."""
    ref = oracle.fft_nd(x.astype(np.complex128), ndim, inverse=inverse, normalize=normalize)
    axes = tuple(range(x.ndim - ndim, x.ndim))
    exact = (np.fft.ifftn(x.astype(np.complex128), axes=axes, norm="backward" if normalize else "forward")
             if inverse else np.fft.fftn(x.astype(np.complex128), axes=axes))
    oracle_err = rel_l2(ref, exact)
    assert rel_l2(y, exact) <= TOL[prec]
    assert rel_l2(y, ref) <= TOL[prec] + 1.05 * oracle_err


@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("inverse", [False, True])
def test_recursive_rader_tuning_executes_rader_for_4099(V, ctx, prec, inverse):
    # BASELINE config 4, recursive-Rader variant: FFT-Rader 4099 -> conv 2*3*683, 683 nested
    rec = V.PlannerTuning.portable().with_recursive_fft_rader(True)
    cfg = (V.FftConfig([4099]).with_batch_count(3).with_precision(V.Precision[prec]).with_tuning(rec)
           .with_inverse_normalization(True))
    d = V.Direction.INVERSE if inverse else V.Direction.FORWARD
    ir = V.TransformIr.build(cfg, d, ctx.device_profile())
    assert ir.axis_child(0).kind == V.AlgorithmKind.RADER
    x = uniform_complex(np.random.default_rng(5), (3, 4099), NP[prec][0])
    y = ctx.execute_transform(ir, x).reshape(x.shape)
    check_against_oracle_and_exact(y, x, prec, inverse=inverse, normalize=inverse)


@pytest.mark.parametrize("prec", ["F32", "F64"])
def test_mixed_direct_and_fft_rader_axis(V, ctx, prec):
    # 83 * 1009: direct Rader (83 fails the safe-prime gate) and FFT-Rader 1009
    n = 83 * 1009
    cfg = V.FftConfig([n]).with_batch_count(2).with_precision(V.Precision[prec])
    ir = V.TransformIr.build(cfg, V.Direction.FORWARD, ctx.device_profile())
    x = uniform_complex(np.random.default_rng(9), (2, n), NP[prec][0])
    y = ctx.execute_transform(ir, x).reshape(x.shape)
    if ir.axis_child(0).kind == V.AlgorithmKind.RADER:
        check_against_oracle_and_exact(y, x, prec)
    else:
        assert rel_l2(y, oracle.fft_nd(x.astype(np.complex128), 1)) <= TOL[prec]


@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("dims,batch", [([8, 16], 3), ([64, 64, 64], 1), ([32, 17, 100], 2), ([5, 47, 12], 2),
                                        ([2, 17, 4099], 1), ([16, 1, 64], 2), ([512, 512], 3), ([3, 512, 512], 1)])
def test_c2c_nd(V, ctx, dims, batch, prec):
    for direction, norm in ((V.Direction.FORWARD, False), (V.Direction.INVERSE, True)):
        ir, err = run_c2c(V, ctx, dims, batch, prec, direction, normalize=norm, seed=len(dims))
        assert err <= TOL[prec], (dims, direction, err)


@pytest.mark.parametrize("prec", ["F32", "F64"])
def test_c2c_3d_stockham_rader_bluestein_small_batch(V, ctx, prec):
    # BASELINE config 4 shape family [.., 17, 65537] with the outer axis shortened
    ir, err = run_c2c(V, ctx, [2, 17, 65537], 1, prec, V.Direction.FORWARD, seed=3)
    assert [ir.axis_child(k).kind.name for k in range(3)] == ["STOCKHAM", "RADER", "BLUESTEIN"]
    assert err <= TOL[prec]


def run_real(V, ctx, dims, batch, prec, seed=0):
    cdt, rdt = NP[prec]
    p = V.Precision[prec]
    dev = ctx.device_profile()
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, size=(batch,) + tuple(dims)).astype(rdt)
    fwd = V.TransformIr.build(V.FftConfig(dims).with_batch_count(batch).with_precision(p)
                              .with_transform(V.TransformKind.R2C), V.Direction.FORWARD, dev)
    spec = ctx.execute_transform(fwd, x)
    ref = oracle.r2c_nd(x.astype(np.float64), len(dims))
    e1 = rel_l2(spec, ref)
    inv = V.TransformIr.build(V.FftConfig(dims).with_batch_count(batch).with_precision(p)
                              .with_transform(V.TransformKind.C2R).with_inverse_normalization(True),
                              V.Direction.INVERSE, dev)
    back = ctx.execute_transform(inv, ref.astype(cdt))
    ref_back = oracle.c2r_nd(ref.astype(cdt).astype(np.complex128), dims[-1], len(dims), normalize=True)
    e2 = rel_l2(back, ref_back)
    return fwd, e1, e2


@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("dims,batch", [([4096], 16), ([30], 7), ([94], 5), ([206], 3), ([45], 4), ([2048], 3),
                                        ([8704], 2), ([4106], 2), ([17, 34], 2), ([64, 64], 2), ([16, 32, 30], 1),
                                        ([1, 64], 3)])
def test_r2c_c2r(V, ctx, dims, batch, prec):
    ir, e1, e2 = run_real(V, ctx, dims, batch, prec, seed=dims[-1])
    assert e1 <= TOL[prec], (dims, ir.real_algorithm, e1)
    assert e2 <= TOL[prec], (dims, ir.real_algorithm, e2)


@pytest.mark.gpu
@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("dims,batch", [([4096], 8), ([2048], 4), ([256], 16), ([64, 64], 2), ([32, 16, 128], 1)])
def test_c2r_of_arbitrary_bins_matches_full_complex(V, ctx, dims, batch, prec):
    """C2R of bins that are not the spectrum of a real signal (imaginary DC / Nyquist parts,
    as a convolution product has): a FullComplex plan's result is the real part of the
    Hermitian expansion (real_ir.rs:1037-1053), whatever kernel computes it."""
    cdt, rdt = NP[prec]
    rng = np.random.default_rng(sum(dims))
    shape = (batch,) + tuple(dims[:-1]) + (dims[-1] // 2 + 1,)
    bins = (rng.uniform(-1, 1, shape) + 1j * rng.uniform(-1, 1, shape)).astype(cdt)
    inv = V.TransformIr.build(V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
                              .with_transform(V.TransformKind.C2R).with_inverse_normalization(True),
                              V.Direction.INVERSE, ctx.device_profile())
    if inv.real_algorithm != V.RealFftAlgorithm.FULL_COMPLEX:
        pytest.skip("even-half plan: the reference's own even-half algebra defines the result")
    out = ctx.execute_transform(inv, bins)
    ref = oracle.c2r_nd(bins.astype(np.complex128), dims[-1], len(dims), normalize=True)
    assert rel_l2(out, ref) <= TOL[prec]


def _golden_inputs(kind, n, f32):
    x = np.arange(n, dtype=np.float32 if f32 else np.float64)
    if f32:
        if kind == 0:
            return (np.sin(np.float32(0.137) * x) + np.float32(0.0013) * x
                    + 1j * (np.cos(np.float32(0.071) * x) - np.float32(0.0009) * x)).astype(np.complex64)
        return (np.sin(np.float32(0.173) * x) + np.float32(0.003) * x
                - np.float32(0.27) * np.cos(np.float32(0.071) * x)).astype(np.float32)
    if kind == 0:
        return np.sin(0.137 * x) + 0.0013 * x + 1j * (np.cos(0.071 * x) - 0.0009 * x)
    return np.sin(0.173 * x) + 0.003 * x - 0.27 * np.cos(0.071 * x)


@pytest.mark.parametrize("set_name,prec", [("medium", "F64"), ("medium_f32", "F32")])
def test_fftw_golden_vectors_on_gpu(V, ctx, set_name, prec):
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "fftw_golden.npz"))
    names = sorted({k.rsplit("/", 1)[0].split("/", 1)[1] for k in z.files if k.startswith(set_name + "/")})
    dev = ctx.device_profile()
    for name in names:
        shape = [int(v) for v in z[f"{set_name}/{name}/shape"]]
        kind = int(z[f"{set_name}/{name}/kind"])
        n = int(np.prod(shape))
        cfg = V.FftConfig(shape).with_precision(V.Precision[prec])
        if kind == 1:
            cfg = cfg.with_transform(V.TransformKind.R2C)
        elif kind == 2:  # ND DCT-II (FFTW REDFT10 on every axis)
            cfg = cfg.with_transform(V.TransformKind.DCT2)
        if name == "c2c-bluestein-n103":
            t = V.PlannerTuning.portable()
            t.max_rader_fft_prime = 100
            cfg = cfg.with_tuning(t)
        ir = V.TransformIr.build(cfg, V.Direction.FORWARD, dev)
        got = ctx.execute_transform(ir, _golden_inputs(kind, n, prec == "F32"))
        tol = (1e-4 if prec == "F32" else 1e-8) * n
        assert np.abs(got - z[f"{set_name}/{name}/output"]).max() <= tol, name


def test_resident_execution_matches_host_execution(V, ctx):
    torch = pytest.importorskip("torch")
    dev = ctx.device_profile()
    ir = V.TransformIr.build(V.FftConfig([4096]).with_batch_count(32), V.Direction.FORWARD, dev)
    rng = np.random.default_rng(11)
    x = uniform_complex(rng, (32, 4096), np.complex64)
    host = ctx.execute_transform(ir, x)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty_like(xd)
    stream = torch.cuda.current_stream().cuda_stream
    ctx.execute_resident(ir, xd.data_ptr(), yd.data_ptr(), stream=stream)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy().ravel(), host)
    # in place
    ctx.execute_resident(ir, xd.data_ptr(), xd.data_ptr(), stream=stream)
    torch.cuda.synchronize()
    assert np.array_equal(xd.cpu().numpy().ravel(), host)


@pytest.mark.gpu
@pytest.mark.parametrize("dims,batch,prec,kind", [([4096], 16384 + 100, "F32", "c2c"), ([4099], 20000, "F32", "c2c"),
                                                  ([4096], 20000, "F64", "r2c"), ([1024], 100000, "F32", "c2r")])
def test_pipelined_host_execution_matches_resident(V, ctx, dims, batch, prec, kind):
    """Large batched host executions run as overlapped sub-batches (upload / transform /
    download on three streams); the result equals one resident execution of the whole batch."""
    torch = pytest.importorskip("torch")
    cdt, rdt = NP[prec]
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    direction = V.Direction.FORWARD
    if kind == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
    elif kind == "c2r":
        cfg = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        direction = V.Direction.INVERSE
    ir = V.TransformIr.build(cfg, direction, ctx.device_profile())
    rng = np.random.default_rng(batch)
    n_in = ir.input_elements * (1 if kind == "r2c" else 2)
    x = rng.uniform(-1, 1, n_in).astype(rdt)
    host_in = torch.from_numpy(x).pin_memory()
    host_out = torch.empty(ir.output_elements * (1 if kind == "c2r" else 2), dtype=host_in.dtype).pin_memory()
    xin = host_in.numpy().view(np.float32 if prec == "F32" else np.float64)
    out = ctx.execute_transform(ir, xin.view(rdt if kind == "r2c" else cdt),
                                out=host_out.numpy().view(rdt if kind == "c2r" else cdt))
    xd = host_in.cuda()
    yd = torch.empty(host_out.numel(), dtype=host_in.dtype, device="cuda")
    ctx.execute_resident(ir, xd.data_ptr(), yd.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    ref = yd.cpu().numpy().view(rdt if kind == "c2r" else cdt)
    assert rel_l2(out, ref) <= TOL[prec]


def test_input_length_mismatch_is_reported(V, ctx):
    ir = V.TransformIr.build(V.FftConfig([64]).with_batch_count(2), V.Direction.FORWARD, ctx.device_profile())
    import ctypes
    x = np.zeros(100, dtype=np.complex64)
    out = np.zeros(128, dtype=np.complex64)
    lib = V.library()
    st = lib.b200fft_execute_host(ctx._h, ir._h, x.ctypes.data, x.nbytes, out.ctypes.data, out.nbytes)
    assert st == V.Status.InputLengthMismatch


@pytest.mark.gpu
def test_async_submissions_match_synchronous_execution(V, ctx):
    """NativeAsyncRuntime tickets: several submissions in flight, waited for in any order,
    each equal to the synchronous execution of its own input; errors surface at wait()."""
    dev = ctx.device_profile()
    irs = [V.TransformIr.build(V.FftConfig([n]).with_batch_count(b), V.Direction.FORWARD, dev)
           for n, b in ((4096, 256), (4099, 16), (1000, 40))]
    rng = np.random.default_rng(5)
    xs = [uniform_complex(rng, (ir.input_elements,), np.complex64) for ir in irs]
    tickets = [ctx.submit_transform(ir, x) for ir, x in zip(irs, xs)]
    for ir, x, t in reversed(list(zip(irs, xs, tickets))):
        assert np.array_equal(t.wait(), ctx.execute_transform(ir, x))
    bad = ctx.submit_transform(irs[0], xs[0], out=np.empty(irs[0].output_elements - 1, dtype=np.complex64))
    with pytest.raises(V.VkFftError):
        bad.wait()


@pytest.mark.gpu
@pytest.mark.parametrize("precision,real", [("F16_STORAGE_F32_COMPUTE", False), ("F16_STORAGE_F32_COMPUTE", True),
                                            ("F64_COMPUTE_F32_STORAGE", False), ("F64_COMPUTE_F32_STORAGE", True)])
def test_mixed_storage_compute_precision(V, ctx, precision, real):
    """F16 storage / F32 compute and F64 compute / F32 storage (config.rs:107-161): host arrays
    of the API type (f32 / f64) through execute_transform, storage-typed device buffers
    through execute_resident; both equal the compute-precision transform of the input
    quantised to storage, quantised to storage again (the reference's mixed-precision
    expectation, tests/convolution_runtime.rs:116-140)."""
    torch = pytest.importorskip("torch")
    store = np.float16 if precision.startswith("F16") else np.float32
    api = np.float32 if precision.startswith("F16") else np.float64
    dims, batch = ([4096], 16) if not real else ([2048], 8)
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[precision])
    if real:
        cfg = cfg.with_transform(V.TransformKind.R2C)
    ir = V.TransformIr.build(cfg, V.Direction.FORWARD, ctx.device_profile())
    rng = np.random.default_rng(17)
    n_in = ir.input_elements * (1 if real else 2)
    xq = rng.uniform(-1, 1, n_in).astype(store)                     # values representable in storage
    x64 = xq.astype(np.float64)
    ref = (oracle.r2c_nd(x64.reshape(batch, *dims), 1) if real
           else oracle.fft_nd(x64.view(np.complex128).reshape(batch, *dims), 1))
    ref_q = ref.view(np.float64).astype(store).astype(np.float64)
    host_in = xq.astype(api)
    host = ctx.execute_transform(ir, host_in if real else host_in.view(np.complex64 if api == np.float32
                                                                       else np.complex128))
    tol = 2e-3 if store == np.float16 else 1e-6
    assert rel_l2(np.asarray(host).view(api).astype(np.float64), ref_q) <= tol
    tdt = torch.float16 if store == np.float16 else torch.float32
    xd = torch.from_numpy(xq).cuda()
    yd = torch.empty(ir.output_elements * 2, dtype=tdt, device="cuda")
    ctx.execute_resident(ir, xd.data_ptr(), yd.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rel_l2(yd.cpu().numpy().astype(np.float64), ref_q) <= tol
