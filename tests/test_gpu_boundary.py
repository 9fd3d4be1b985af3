"""Zero padding and formatted buffer strides on the B200 (boundary gather / scatter passes
around the transform) against the oracle on the manually padded / packed tensors."""
import numpy as np
import pytest

import oracle
from boundary_layout import pack, pad_mask, resolve, unpack
from conftest import rel_l2

TOL = {"F32": 2e-6, "F64": 1e-13}
NP = {"F32": (np.complex64, np.float32), "F64": (np.complex128, np.float64)}

CASES = [
    dict(mode="c2c", dims=[4096], batch=64, prec="F32", pad={0: [2048, 4096]}),
    dict(mode="c2c_inv", dims=[4096], batch=16, prec="F64", pad={0: [100, 300]}),
    dict(mode="c2c", dims=[64, 64, 64], batch=1, prec="F32", pad={0: [32, 64], 1: [32, 64], 2: [32, 64]}),
    dict(mode="c2c", dims=[256, 128], batch=2, prec="F32", pad={1: [64, 128]}, domain="frequency"),
    dict(mode="c2c_inv", dims=[256, 128], batch=2, prec="F64", pad={0: [10, 20]}, domain="frequency"),
    dict(mode="r2c", dims=[4096], batch=32, prec="F32", pad={0: [1000, 3000]}),
    dict(mode="c2r", dims=[2048], batch=8, prec="F64", pad={0: [7, 1300]}),
    dict(mode="r2c", dims=[64, 128], batch=2, prec="F32", pad={0: [16, 48], 1: [0, 32]}),
    dict(mode="c2c", dims=[128, 100], batch=3, prec="F32", in_strides={0: 130}, in_batch_stride=20000,
         out_strides={0: 101}, out_batch_stride=13000),
    dict(mode="r2c", dims=[64, 256], batch=2, prec="F64", in_strides={0: 300}, out_strides={0: 140},
         out_batch_stride=9000, pad={0: [10, 20]}),
    dict(mode="c2r", dims=[32, 512], batch=2, prec="F32", in_strides={0: 260}, in_batch_stride=8400,
         out_strides={0: 520}),
    dict(mode="c2c", dims=[4099], batch=4, prec="F64", pad={0: [2000, 4099]}),
]


def run_case(V, ctx, case):
    dims, batch, mode, prec = case["dims"], case["batch"], case["mode"], case["prec"]
    cdt, rdt = NP[prec]
    pads = case.get("pad", {})
    freq = case.get("domain") == "frequency"
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    for axis, (lo, hi) in pads.items():
        cfg = cfg.with_zero_padding(axis, lo, hi)
    if freq:
        cfg = cfg.with_zero_padding_domain(V.ZeroPaddingDomain.FREQUENCY)
    for axis, st in (case.get("in_strides") or {}).items():
        cfg = cfg.with_input_buffer_axis_stride(axis, st)
    for axis, st in (case.get("out_strides") or {}).items():
        cfg = cfg.with_output_buffer_axis_stride(axis, st)
    if case.get("in_batch_stride"):
        cfg = cfg.with_input_buffer_batch_stride(case["in_batch_stride"])
    if case.get("out_batch_stride"):
        cfg = cfg.with_output_buffer_batch_stride(case["out_batch_stride"])
    nd = len(dims)
    shape = (batch,) + tuple(dims)
    half = list(dims[:-1]) + [dims[-1] // 2 + 1]
    mask = pad_mask(dims, pads) if pads else np.zeros(dims, dtype=bool)
    rng = np.random.default_rng(sum(dims) + batch)
    direction = V.Direction.FORWARD
    if mode in ("c2c", "c2c_inv"):
        inv = mode == "c2c_inv"
        direction = V.Direction.INVERSE if inv else V.Direction.FORWARD
        x = (rng.uniform(-1, 1, shape) + 1j * rng.uniform(-1, 1, shape)).astype(cdt)
        pad_in = bool(pads) and (freq == inv)
        xi = np.where(mask, 0, x) if pad_in else x
        ref = oracle.fft_nd(xi.astype(np.complex128), nd, inverse=inv)
        if pads and not pad_in:
            ref = np.where(mask, 0, ref)
        in_dims, out_dims, out_dt = dims, dims, cdt
    elif mode == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
        x = rng.uniform(-1, 1, shape).astype(rdt)
        ref = oracle.r2c_nd(np.where(mask, 0, x).astype(np.float64), nd)
        in_dims, out_dims, out_dt = dims, half, cdt
    else:
        cfg = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        direction = V.Direction.INVERSE
        x = oracle.r2c_nd(rng.uniform(-1, 1, shape), nd).astype(cdt)
        ref = np.where(mask, 0, oracle.c2r_nd(x.astype(np.complex128), dims[-1], nd, normalize=True))
        in_dims, out_dims, out_dt = half, dims, rdt
    ir = V.TransformIr.build(cfg, direction, ctx.device_profile())
    # host API: logical (dense) arrays in and out, as the reference's executors take them
    host = ctx.execute_transform(ir, x.reshape(-1))
    err_host = rel_l2(host, ref)
    # device buffers: the formatted (physical) layouts
    import torch
    phys = pack(x, in_dims, case.get("in_strides"), case.get("in_batch_stride"))
    st, bs = resolve(out_dims, case.get("out_strides"), case.get("out_batch_stride"))
    assert ir.input_buffer_elements == phys.size and ir.output_buffer_elements == bs * batch
    real_view = np.float64 if prec == "F64" else np.float32
    xd = torch.from_numpy(np.ascontiguousarray(phys).view(real_view)).cuda()
    n_out = bs * batch * (1 if out_dt == rdt else 2)
    yd = torch.full((n_out,), 3.0, dtype=xd.dtype, device="cuda")
    ctx.execute_resident(ir, xd.data_ptr(), yd.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    out = yd.cpu().numpy().view(out_dt)
    got = unpack(out, out_dims, case.get("out_strides"), case.get("out_batch_stride"), batch)
    if case.get("out_strides") or case.get("out_batch_stride"):
        # elements of the formatted output buffer outside the tensor are not written
        touched = pack(np.ones((batch,) + tuple(out_dims), dtype=bool), out_dims, case.get("out_strides"),
                       case.get("out_batch_stride"), False)
        fill = 3.0 if out_dt == rdt else 3.0 + 3.0j  # the float buffer of 3.0 viewed as complex
        assert np.all(out[~touched] == fill)
    return err_host, rel_l2(got, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[f"{c['mode']}-{c['dims']}-{c['prec']}" for c in CASES])
def test_zero_padding_and_formatted_strides(V, ctx, case):
    err_host, err_dev = run_case(V, ctx, case)
    assert err_host <= TOL[case["prec"]] and err_dev <= TOL[case["prec"]], (err_host, err_dev)
