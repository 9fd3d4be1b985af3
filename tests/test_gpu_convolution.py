"""FFT convolution on the B200 against the oracle: NdRealConvolutionIr
(convolution_ir.rs:3867-4250; R2C -> policy multiply -> normalised C2R), the C2C
ConvolutionIr / NdConvolutionIr (:2520-3866; scalar, K-kernel and matrix multiplies) and the
kernelConvolution preparation transform."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2

TOL = {"F32": 2e-6, "F64": 1e-13}
NP = {"F32": (np.complex64, np.float32), "F64": (np.complex128, np.float64)}


def conv_config(V, dims, prec, coords, kernels, conj=False, cross=False):
    cfg = (V.FftConfig(dims).with_transform(V.TransformKind.R2C).with_precision(V.Precision[prec])
           .with_convolution(True).with_coordinate_features(coords).with_convolution_kernel_count(kernels))
    if conj:
        cfg = cfg.with_convolution_conjugation(V.ConvolutionConjugation.SEQUENCE)
    if cross:
        cfg = cfg.with_cross_power_spectrum_normalization(True)
    return cfg


def run_conv(V, ctx, dims, prec, coords=1, kernels=1, copies=None, conj=False, cross=False, seed=0):
    cdt, rdt = NP[prec]
    copies = kernels * coords if copies is None else copies
    rng = np.random.default_rng(seed)
    L = int(np.prod(dims[:-1])) * (dims[-1] // 2 + 1)
    ker = (rng.uniform(-1, 1, copies * L) + 1j * rng.uniform(-1, 1, copies * L)).astype(cdt)
    x = rng.uniform(-1, 1, (coords,) + tuple(dims)).astype(rdt)
    ir = V.NdRealConvolutionIr.build_from_spectrum(conv_config(V, dims, prec, coords, kernels, conj, cross), ker,
                                                   ctx.device_profile())
    y = ctx.execute_nd_real_convolution(ir, x)
    ref = oracle.convolve_nd(x, ker, dims, coords, kernels, conj, cross)
    return rel_l2(y, ref)


CASES = [
    dict(dims=[32, 48], prec="F32", coords=3),
    dict(dims=[32, 48], prec="F64", coords=3),
    dict(dims=[16, 12, 20], prec="F64", coords=2, copies=1),
    dict(dims=[32, 48], prec="F32", coords=2, kernels=3),
    dict(dims=[30, 34], prec="F64", coords=2, conj=True, cross=True),
    dict(dims=[97, 40], prec="F64"),
    dict(dims=[4099, 6], prec="F32"),
    dict(dims=[8192, 6], prec="F32", kernels=2),
    dict(dims=[256, 256], prec="F32", coords=3),
    dict(dims=[64, 64, 64], prec="F32", coords=2, conj=True),
    dict(dims=[1024, 1024], prec="F32"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_convolution_matches_oracle(V, ctx, case):
    err = run_conv(V, ctx, **case)
    assert err <= TOL[case["prec"]], (case, err)


@pytest.mark.gpu
def test_convolution_resident_matches_host(V, ctx):
    import torch
    dims, C = [64, 96], 2
    rng = np.random.default_rng(3)
    L = 64 * 49
    ker = (rng.uniform(-1, 1, C * L) + 1j * rng.uniform(-1, 1, C * L)).astype(np.complex64)
    x = rng.uniform(-1, 1, (C, 64, 96)).astype(np.float32)
    ir = V.NdRealConvolutionIr.build_from_spectrum(conv_config(V, dims, "F32", C, 1), ker, ctx.device_profile())
    host = ctx.execute_nd_real_convolution(ir, x)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(ir.output_elements, dtype=torch.float32, device="cuda")
    ws = torch.empty(max(ir.workspace_bytes, 1), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream()
    ctx.execute_nd_real_convolution_resident(ir, xd.data_ptr(), yd.data_ptr(), ws.data_ptr(), s.cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), host)


def test_convolution_build_validation(V):
    """Builds are host-only: policy errors match the reference's validation."""
    dev = V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA)
    ker = np.zeros(32 * 25, dtype=np.complex64)
    with pytest.raises(V.VkFftError):
        V.NdRealConvolutionIr.build_from_spectrum(V.FftConfig([32, 48]).with_transform(V.TransformKind.R2C), ker,
                                                  dev)
    cfg = conv_config(V, [32, 48], "F32", 2, 1)
    with pytest.raises(V.VkFftError):  # 3 copies for 2 systems
        V.NdRealConvolutionIr.build_from_spectrum(cfg, np.zeros(3 * 32 * 25, dtype=np.complex64), dev)
    ir = V.NdRealConvolutionIr.build_from_spectrum(cfg, np.zeros(2 * 32 * 25, dtype=np.complex64), dev)
    assert ir.input_elements == 2 * 32 * 48 and ir.output_elements == 2 * 32 * 48


C2C_CASES = [
    dict(dims=[4096], batch=64, prec="F32"),
    dict(dims=[4096], batch=1, prec="F64", kernels=4),
    dict(dims=[1000], batch=1, prec="F64", matrix=2),
    dict(dims=[2048], batch=1, prec="F32", matrix=2, symmetric=True, conj=True),
    dict(dims=[510], batch=1, prec="F64", matrix=3, kernels=2),
    dict(dims=[256, 256], batch=2, prec="F32", cross=True),
    dict(dims=[64, 64, 64], batch=1, prec="F32", matrix=3),
    dict(dims=[4099], batch=2, prec="F64"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", C2C_CASES, ids=[str(c) for c in C2C_CASES])
def test_c2c_convolution_matches_oracle(V, ctx, case):
    """ConvolutionIr / NdConvolutionIr: scalar, K-kernel, matrix (symmetric) and policy variants."""
    dims, B, prec = case["dims"], case["batch"], case["prec"]
    cdt = NP[prec][0]
    M, K, sym = case.get("matrix", 0), case.get("kernels", 1), case.get("symmetric", False)
    C = M if M else 1
    cfg = (V.FftConfig(dims).with_batch_count(B).with_precision(V.Precision[prec]).with_convolution(True)
           .with_convolution_kernel_count(K))
    if M:
        cfg = cfg.with_matrix_convolution(M).with_symmetric_convolution_kernel(sym)
    if case.get("conj"):
        cfg = cfg.with_convolution_conjugation(V.ConvolutionConjugation.SEQUENCE)
    if case.get("cross"):
        cfg = cfg.with_cross_power_spectrum_normalization(True)
    T = int(np.prod(dims))
    planes = (M * (M + 1) // 2 if sym else M * M) if M else 1
    rng = np.random.default_rng(T + B)
    x = (rng.uniform(-1, 1, (B * C, T)) + 1j * rng.uniform(-1, 1, (B * C, T))).astype(cdt)
    ker = (rng.uniform(-1, 1, planes * K * T) + 1j * rng.uniform(-1, 1, planes * K * T)).astype(cdt)
    cls = V.ConvolutionIr if len(dims) == 1 else V.NdConvolutionIr
    ir = cls.build_from_spectrum(cfg, ker, ctx.device_profile())
    y = ctx.execute_convolution(ir, x)
    ref = oracle.convolve_c2c(x, ker, dims, B, C, K, M, sym, case.get("conj", False), case.get("cross", False))
    assert rel_l2(y, ref) <= TOL[prec]


@pytest.mark.gpu
@pytest.mark.parametrize("real", [False, True])
def test_kernel_convolution_preparation(V, ctx, real):
    """kernelConvolution: the forward transform of batch x coordinate kernel systems."""
    B, C = (1, 3) if not real else (2, 2)
    dims = [4096] if not real else [256, 200]
    cfg = V.FftConfig(dims).with_batch_count(B).with_kernel_convolution(True).with_coordinate_features(C)
    rng = np.random.default_rng(9)
    if real:
        cfg = cfg.with_transform(V.TransformKind.R2C)
        x = rng.uniform(-1, 1, (B * C,) + tuple(dims)).astype(np.float32)
        ref = oracle.r2c_nd(x.astype(np.float64), len(dims))
    else:
        x = (rng.uniform(-1, 1, (B * C,) + tuple(dims)) + 1j * rng.uniform(-1, 1, (B * C,) + tuple(dims))).astype(
            np.complex64)
        ref = oracle.fft_nd(x.astype(np.complex128), len(dims))
    ir = V.TransformIr.build(cfg, V.Direction.FORWARD, ctx.device_profile())
    assert rel_l2(ctx.execute_transform(ir, x), ref) <= TOL["F32"]


# ---- ND real convolution: matrix ownership, zero padding, formatted buffers --------------

def real_conv_config(V, dims, prec, coords=1, kernels=1, matrix=0, symmetric=False, conj=False, cross=False,
                     pads=None, in_strides=None, out_strides=None, in_batch_stride=None, out_batch_stride=None):
    cfg = conv_config(V, dims, prec, coords, kernels, conj, cross)
    if matrix:
        cfg = cfg.with_matrix_convolution(matrix).with_symmetric_convolution_kernel(symmetric)
    for axis, (lo, hi) in (pads or {}).items():
        cfg = cfg.with_zero_padding(axis, lo, hi)
    for axis, st in (in_strides or {}).items():
        cfg = cfg.with_input_buffer_axis_stride(axis, st)
    for axis, st in (out_strides or {}).items():
        cfg = cfg.with_output_buffer_axis_stride(axis, st)
    if in_batch_stride:
        cfg = cfg.with_input_buffer_batch_stride(in_batch_stride)
    if out_batch_stride:
        cfg = cfg.with_output_buffer_batch_stride(out_batch_stride)
    return cfg


REAL_CASES = [
    # matrix ownership (C = matrix size), K = 1 and K > 1, symmetric planes, policies
    dict(dims=[32, 48], prec="F32", matrix=2),
    dict(dims=[30, 34], prec="F64", matrix=2, symmetric=True, conj=True, cross=True),
    dict(dims=[16, 12, 20], prec="F64", matrix=3, kernels=2),
    dict(dims=[256, 256], prec="F32", matrix=3),
    # zero padding: independent coordinates, scalar K > 1, nonsymmetric matrix, shared kernel
    dict(dims=[64, 64], prec="F32", coords=2, pads={0: (32, 64), 1: (40, 64)}),
    dict(dims=[48, 40], prec="F64", kernels=3, pads={0: (24, 48)}),
    dict(dims=[32, 32], prec="F64", matrix=2, pads={1: (16, 32)}),
    dict(dims=[128, 100], prec="F32", coords=3, copies=1, pads={1: (50, 100)}, conj=True),
    dict(dims=[16, 20, 24], prec="F32", coords=2, pads={2: (12, 24)}),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", REAL_CASES, ids=[str(c) for c in REAL_CASES])
def test_nd_real_convolution_matrix_and_padding(V, ctx, case):
    """NdRealConvolutionIr matrix ownership and zero padding (convolution_ir.rs:3884-4250)
    against the oracle's R2C -> multiply -> C2R with the padding masks."""
    dims, prec = case["dims"], case["prec"]
    cdt, rdt = NP[prec]
    M, K, sym = case.get("matrix", 0), case.get("kernels", 1), case.get("symmetric", False)
    C = M if M else case.get("coords", 1)
    L = int(np.prod(dims[:-1])) * (dims[-1] // 2 + 1)
    planes = (M * (M + 1) // 2 if sym else M * M) if M else C
    copies = case.get("copies", K * planes)
    rng = np.random.default_rng(L + C)
    ker = (rng.uniform(-1, 1, copies * L) + 1j * rng.uniform(-1, 1, copies * L)).astype(cdt)
    x = rng.uniform(-1, 1, (C,) + tuple(dims)).astype(rdt)
    cfg = real_conv_config(V, dims, prec, C, K, M, sym, case.get("conj", False), case.get("cross", False),
                           case.get("pads"))
    ir = V.NdRealConvolutionIr.build_from_spectrum(cfg, ker, ctx.device_profile())
    y = ctx.execute_nd_real_convolution(ir, x)
    ref = oracle.convolve_nd(x, ker, dims, C, K, case.get("conj", False), case.get("cross", False), matrix=M,
                             symmetric=sym, pads=case.get("pads"))
    assert rel_l2(y, ref) <= TOL[prec], (case, rel_l2(y, ref))


FORMATTED_CASES = [
    dict(dims=[64, 96], prec="F32", in_strides={0: 100}, in_batch_stride=7000, out_strides={0: 104}),
    dict(dims=[32, 20, 24], prec="F64", in_strides={1: 30}, out_strides={0: 700, 1: 25}, out_batch_stride=23000,
         pads={2: (12, 24)}),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", FORMATTED_CASES, ids=[str(c) for c in FORMATTED_CASES])
def test_nd_real_convolution_formatted_buffers(V, ctx, case):
    """Scalar batch-1 K = 1 convolution with formatted buffer strides: the host API takes
    and returns logical tensors, device buffers are the formatted layouts (elements outside
    the tensor are left untouched)."""
    import torch
    from boundary_layout import pack, resolve, unpack
    dims, prec = case["dims"], case["prec"]
    cdt, rdt = NP[prec]
    L = int(np.prod(dims[:-1])) * (dims[-1] // 2 + 1)
    rng = np.random.default_rng(sum(dims))
    ker = (rng.uniform(-1, 1, L) + 1j * rng.uniform(-1, 1, L)).astype(cdt)
    x = rng.uniform(-1, 1, (1,) + tuple(dims)).astype(rdt)
    cfg = real_conv_config(V, dims, prec, pads=case.get("pads"), in_strides=case.get("in_strides"),
                           out_strides=case.get("out_strides"), in_batch_stride=case.get("in_batch_stride"),
                           out_batch_stride=case.get("out_batch_stride"))
    ir = V.NdRealConvolutionIr.build_from_spectrum(cfg, ker, ctx.device_profile())
    ref = oracle.convolve_nd(x, ker, dims, pads=case.get("pads"))
    assert ir.input_elements == x.size and ir.output_elements == x.size
    host = ctx.execute_nd_real_convolution(ir, x)
    assert rel_l2(host, ref) <= TOL[prec]
    phys = pack(x, dims, case.get("in_strides"), case.get("in_batch_stride"))
    st, bs = resolve(dims, case.get("out_strides"), case.get("out_batch_stride"))
    assert ir.input_buffer_elements == phys.size and ir.output_buffer_elements == bs
    xd = torch.from_numpy(np.ascontiguousarray(phys)).cuda()
    yd = torch.full((bs,), 3.0, dtype=xd.dtype, device="cuda")
    ws = torch.empty(max(ir.workspace_bytes, 1), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    ctx.execute_nd_real_convolution_resident(ir, xd.data_ptr(), yd.data_ptr(), ws.data_ptr(), s)
    ctx.synchronize(s)
    out = yd.cpu().numpy()
    got = unpack(out, dims, case.get("out_strides"), case.get("out_batch_stride"), 1)
    assert rel_l2(got, ref) <= TOL[prec]
    touched = pack(np.ones((1,) + tuple(dims), dtype=bool), dims, case.get("out_strides"),
                   case.get("out_batch_stride"), False)
    assert np.all(out[~touched] == 3.0)


def test_nd_real_convolution_ownership_errors(V):
    """The reference's ownership rules (convolution_ir.rs:3899-3937), host only."""
    dev = V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA)
    L = 32 * 25

    def build(cfg, copies):
        return V.NdRealConvolutionIr.build_from_spectrum(cfg, np.zeros(copies * L, dtype=np.complex64), dev)

    # matrix coordinates must equal the matrix size
    with pytest.raises(V.VkFftError):
        build(real_conv_config(V, [32, 48], "F32", matrix=2).with_coordinate_features(3), 4)
    # formatted strides only for scalar K = 1
    with pytest.raises(V.VkFftError) as e:
        build(real_conv_config(V, [32, 48], "F32", coords=2, in_strides={0: 50}), 2)
    assert e.value.variant == "UnsupportedKernelPath" and "K1" in str(e.value)
    # zero padding with a symmetric matrix kernel
    with pytest.raises(V.VkFftError) as e:
        build(real_conv_config(V, [32, 48], "F32", coords=2, matrix=2, symmetric=True, pads={0: (0, 4)}), 3)
    assert e.value.variant == "UnsupportedKernelPath"
    # matrix kernel spectrum: K * planes copies
    with pytest.raises(V.VkFftError):
        build(real_conv_config(V, [32, 48], "F32", coords=2, matrix=2), 3)
    ir = build(real_conv_config(V, [32, 48], "F32", coords=2, matrix=2), 4)
    assert ir.input_elements == 2 * 32 * 48 and ir.output_elements == 2 * 32 * 48
