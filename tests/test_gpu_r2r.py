"""DCT / DST on the B200 (R2rIr and NdR2rIr, r2r_ir.rs:621-2017) through the C ABI.

Checked against the oracle's direct sums of the FFTW REDFT/RODFT definitions
(r2r_ir.rs:2351-2433), against the reference's FFTW 3.3.9 DCT-II goldens
(tests/fixtures/fftw_precision_v1.txt dct2-n37, fftw_precision_medium_v1.txt
dct2-nd-17x34), and at full size through inverse-pair round trips
(inverse_partner / inverse_pair_scale, r2r_ir.rs:2317-2349) plus a sampled subset of lines.
Tolerances: relL2 <= 2e-6 (f32 compute), <= 1e-13 (f64 compute)."""
import os

import numpy as np
import pytest

import oracle
from conftest import rel_l2

TOL = {"F32": 2e-6, "F64": 1e-13}
RDT = {"F32": np.float32, "F64": np.float64}
KINDS = ("DCT1", "DCT2", "DCT3", "DCT4", "DST1", "DST2", "DST3", "DST4")
GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fftw_golden.npz")


def r2r_config(V, dims, kind, prec, batch=1, normalize=False):
    return (V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
            .with_transform(V.TransformKind[kind]).with_inverse_normalization(normalize))


def run(V, ctx, dims, kind, prec, batch=1, inverse=False, normalize=False, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (batch,) + tuple(dims)).astype(RDT[prec])
    d = V.Direction.INVERSE if inverse else V.Direction.FORWARD
    ir = V.TransformIr.build(r2r_config(V, dims, kind, prec, batch, normalize), d, ctx.device_profile())
    y = ctx.execute_transform(ir, x).reshape(x.shape)
    ref = oracle.r2r_nd(x.astype(np.float64), kind, len(dims), inverse=inverse, normalize=normalize)
    return rel_l2(y, ref), ir


LENGTHS_1D = [2, 3, 16, 31, 64, 100, 257, 1024, 4096, 4097]


@pytest.mark.gpu
@pytest.mark.parametrize("prec", ["F32", "F64"])
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("n", LENGTHS_1D)
def test_r2r_1d_matches_definition(V, ctx, kind, n, prec):
    batch = max(1, min(64, 65536 // n))
    err, ir = run(V, ctx, [n], kind, prec, batch=batch, seed=n)
    assert ir.family == V.Family.REAL_TO_REAL
    assert err <= TOL[prec], (kind, n, prec, err)


ND_CASES = [
    dict(dims=[17, 34], kind="DCT2", prec="F32"),
    dict(dims=[64, 64], kind="DCT2", prec="F64", batch=3),
    dict(dims=[30, 45], kind="DST2", prec="F32", batch=2),
    dict(dims=[16, 24, 20], kind="DCT3", prec="F64"),
    dict(dims=[32, 32, 32], kind="DCT4", prec="F32"),
    dict(dims=[9, 33], kind="DST4", prec="F64"),
    dict(dims=[65, 40], kind="DCT1", prec="F64"),
    dict(dims=[20, 31], kind="DST1", prec="F32", batch=2),
    dict(dims=[256, 256], kind="DCT2", prec="F32"),
    dict(dims=[48, 50], kind="DST3", prec="F64", inverse=True, normalize=True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", ND_CASES, ids=[str(c) for c in ND_CASES])
def test_r2r_nd_matches_definition(V, ctx, case):
    err, ir = run(V, ctx, case["dims"], case["kind"], case["prec"], batch=case.get("batch", 1),
                  inverse=case.get("inverse", False), normalize=case.get("normalize", False))
    assert ir.family == V.Family.REAL_TO_REAL_ND
    assert err <= TOL[case["prec"]], (case, err)


@pytest.mark.gpu
@pytest.mark.parametrize("kind", KINDS)
def test_r2r_inverse_direction_matches_partner(V, ctx, kind):
    """Inverse = the partner kind scaled by inverse_pair_scale when normalising."""
    for normalize in (False, True):
        err, _ = run(V, ctx, [48], kind, "F64", batch=5, inverse=True, normalize=normalize, seed=7)
        assert err <= TOL["F64"], (kind, normalize, err)


@pytest.mark.gpu
def test_r2r_matches_fftw_goldens(V, ctx):
    """The reference's FFTW 3.3.9 DCT-II fixtures, run on the device (f64 compute)."""
    z = np.load(GOLDEN)
    dev = ctx.device_profile()
    x = z["compact/dct2-n37/input"]
    ir = V.TransformIr.build(r2r_config(V, [37], "DCT2", "F64"), V.Direction.FORWARD, dev)
    assert np.abs(ctx.execute_transform(ir, x) - z["compact/dct2-n37/output"]).max() <= 2e-10 * 37
    shape = tuple(int(v) for v in z["medium/dct2-nd-17x34/shape"])
    n = int(np.prod(shape))
    t = np.arange(n, dtype=np.float64)
    real_v1 = np.sin(0.173 * t) + 0.003 * t - 0.27 * np.cos(0.071 * t)  # the fixture's real-v1 formula
    ir = V.TransformIr.build(r2r_config(V, list(shape), "DCT2", "F64"), V.Direction.FORWARD, dev)
    got = ctx.execute_transform(ir, real_v1)
    assert np.abs(got - z["medium/dct2-nd-17x34/output"]).max() <= 2e-10 * n


FULL = [
    dict(dims=[4096], batch=16384, kind="DCT2", prec="F32"),
    dict(dims=[4096], batch=4096, kind="DCT4", prec="F64"),
    dict(dims=[1025], batch=16384, kind="DCT1", prec="F32"),
    dict(dims=[4095], batch=8192, kind="DST4", prec="F32"),
    dict(dims=[512, 512], batch=16, kind="DCT2", prec="F32"),
    dict(dims=[128, 128, 128], batch=2, kind="DST2", prec="F64"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", FULL, ids=[str(c) for c in FULL])
def test_r2r_full_size_round_trip_and_sampled_lines(V, ctx, case):
    """Large batches: forward -> normalised inverse restores the input, and a sample of
    the forward lines matches the oracle's direct sums."""
    dims, B, kind, prec = case["dims"], case["batch"], case["kind"], case["prec"]
    rng = np.random.default_rng(11)
    x = rng.uniform(-1, 1, (B,) + tuple(dims)).astype(RDT[prec])
    dev = ctx.device_profile()
    fwd = V.TransformIr.build(r2r_config(V, dims, kind, prec, B), V.Direction.FORWARD, dev)
    inv = V.TransformIr.build(r2r_config(V, dims, kind, prec, B, normalize=True), V.Direction.INVERSE, dev)
    y = ctx.execute_transform(fwd, x).reshape(x.shape)
    back = ctx.execute_transform(inv, y).reshape(x.shape)
    assert rel_l2(back, x) <= 2 * TOL[prec] + (4e-7 if prec == "F32" else 0), "round trip"
    pick = rng.choice(B, size=min(B, 4), replace=False)
    ref = oracle.r2r_nd(x[pick].astype(np.float64), kind, len(dims))
    assert rel_l2(y[pick], ref) <= TOL[prec], "sampled lines"


@pytest.mark.gpu
def test_r2r_zero_padding_and_omitted_axis(V, ctx):
    """Spatial zero padding masks the forward input / inverse output (r2r_ir.rs:1241-1277);
    an omitted axis is left untransformed."""
    rng = np.random.default_rng(5)
    dims = [40, 24]
    x = rng.uniform(-1, 1, (2,) + tuple(dims))
    dev = ctx.device_profile()
    cfg = r2r_config(V, dims, "DCT2", "F64", 2).with_zero_padding(0, 10, 25)
    keep = np.ones(dims)
    keep[10:25, :] = 0.0
    y = ctx.execute_transform(V.TransformIr.build(cfg, V.Direction.FORWARD, dev), x)
    assert rel_l2(y, oracle.r2r_nd(x * keep, "DCT2", 2)) <= TOL["F64"]
    y = ctx.execute_transform(V.TransformIr.build(cfg.with_inverse_normalization(True), V.Direction.INVERSE, dev), x)
    assert rel_l2(y, oracle.r2r_nd(x, "DCT2", 2, inverse=True, normalize=True) * keep) <= TOL["F64"]
    cfg = r2r_config(V, dims, "DST4", "F64", 2).with_omit_dimension(1, True)
    y = ctx.execute_transform(V.TransformIr.build(cfg, V.Direction.FORWARD, dev), x)
    assert rel_l2(y, oracle.r2r_nd(x, "DST4", 2, omitted=(1,))) <= TOL["F64"]


@pytest.mark.gpu
def test_r2r_resident_matches_host(V, ctx):
    import torch
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, (64, 1000)).astype(np.float32)
    ir = V.TransformIr.build(r2r_config(V, [1000], "DST2", "F32", 64), V.Direction.FORWARD, ctx.device_profile())
    host = ctx.execute_transform(ir, x)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(ir.output_elements, dtype=torch.float32, device="cuda")
    ws = torch.empty(max(ir.workspace_bytes, 1), dtype=torch.uint8, device="cuda")
    ctx.execute_resident(ir, xd.data_ptr(), yd.data_ptr(), ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(yd.cpu().numpy(), host)


@pytest.mark.gpu
def test_r2r_f16_storage(V, ctx):
    """F16 storage / F32 compute: the quantised input's transform, quantised to f16."""
    rng = np.random.default_rng(4)
    x = rng.uniform(-1, 1, (8, 256)).astype(np.float16)
    cfg = (V.FftConfig([256]).with_batch_count(8).with_precision(V.Precision.F16_STORAGE_F32_COMPUTE)
           .with_transform(V.TransformKind.DCT2))
    ir = V.TransformIr.build(cfg, V.Direction.FORWARD, ctx.device_profile())
    y = ctx.execute_transform(ir, x.astype(np.float32))
    ref = oracle.r2r_nd(x.astype(np.float64), "DCT2", 1)
    assert rel_l2(y, ref.astype(np.float16).astype(np.float64)) <= 2e-3
