"""Double-double precision on the B200 (DoubleDouble / DoubleDoubleF64Storage,
double_double.rs; DD IR families double_double_ir.rs) through the C ABI.

Checked against the crate's binary128 golden vectors
(tests/fixtures/quad_precision_medium_double_double_v1.txt and
quad_precision_medium_dd_f64_storage_v1.txt, extracted into
tests/golden/quad_dd_golden.npz) at the crate's GPU gates
(tests/quad_medium_double_double_golden.rs:269: max abs <= 2e-30 * n;
tests/quad_medium_dd_f64_storage_golden.rs:210-216: <= 64 ulp or max abs <= 3e-12 * n),
and against the direct binary128 oracle (oracle/dd_oracle.c) on seeded inputs."""
import os

import numpy as np
import pytest

import oracle

DD_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quad_dd_golden.npz")
KIND = {0: "C2C", 1: "R2C", 2: "DCT2"}


def dd_words(rng, shape, complex_):
    w = 4 if complex_ else 2
    x = np.zeros(tuple(shape) + (w,))
    for k in range(0, w, 2):
        hi = rng.uniform(-1, 1, shape)
        x[..., k] = hi
        x[..., k + 1] = hi * np.ldexp(rng.uniform(-1, 1, shape), -55)
    return x


def golden_config(V, name, kind, shape, precision):
    cfg = V.FftConfig(list(shape)).with_precision(precision).with_transform(V.TransformKind[KIND[kind]])
    if name == "c2c-bluestein-n103":  # the fixture's tuning (quad_medium_double_double_golden.rs:170-174)
        cfg = cfg.with_tuning(V.PlannerTuning(max_rader_fft_prime=100))
    return cfg


def names(prefix):
    return sorted({k.split("/")[1] for k in np.load(DD_GOLDEN).files if k.startswith(prefix + "/")})


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("dd"))
def test_dd_matches_quad_goldens(V, ctx, name):
    z = np.load(DD_GOLDEN)
    shape = tuple(int(v) for v in z[f"dd/{name}/shape"])
    kind = int(z[f"dd/{name}/kind"])
    cfg = golden_config(V, name, kind, shape, V.Precision.DOUBLE_DOUBLE)
    ir = V.TransformIr.build(cfg, V.Direction.FORWARD, ctx.device_profile())
    got = ctx.execute_transform_double_double(ir, z[f"dd/{name}/input"].ravel())
    n = int(np.prod(shape))
    err = oracle.dd_max_abs_diff(got, z[f"dd/{name}/output"])
    assert err <= 2e-30 * n, (name, err)


@pytest.mark.gpu
@pytest.mark.parametrize("name", names("dd_f64"))
def test_dd_f64_storage_matches_quad_goldens(V, ctx, name):
    z = np.load(DD_GOLDEN)
    shape = tuple(int(v) for v in z[f"dd_f64/{name}/shape"])
    kind = int(z[f"dd_f64/{name}/kind"])
    cfg = golden_config(V, name, kind, shape, V.Precision.DOUBLE_DOUBLE_F64_STORAGE)
    ir = V.TransformIr.build(cfg, V.Direction.FORWARD, ctx.device_profile())
    inp = z[f"dd_f64/{name}/input"]
    x = inp[:, 0] + 1j * inp[:, 1] if inp.ndim == 2 else inp
    got = np.asarray(ctx.execute_transform_double_double_f64_storage(ir, x))
    want = z[f"dd_f64/{name}/output"]
    got_f = got.view(np.float64).ravel() if np.iscomplexobj(got) else got.ravel()
    want_f = want.ravel()
    n = int(np.prod(shape))
    ulps = np.abs(got_f.view(np.int64) - want_f.view(np.int64))
    assert ulps.max() <= 64 or np.abs(got_f - want_f).max() <= 3e-12 * n, name


CASES = [
    dict(mode="c2c", dims=[16], batch=64),
    dict(mode="c2c", dims=[360], batch=8, inverse=True, normalize=True),
    dict(mode="c2c", dims=[1000], batch=4),
    dict(mode="c2c", dims=[2048], batch=2),
    dict(mode="c2c", dims=[4096], batch=2, inverse=True),
    dict(mode="c2c", dims=[4099], batch=1),
    dict(mode="c2c", dims=[17, 34], batch=3),
    dict(mode="c2c", dims=[12, 10, 20], batch=1, inverse=True, normalize=True),
    dict(mode="r2c", dims=[64, 64], batch=1),
    dict(mode="r2c", dims=[1000], batch=3),
    dict(mode="r2r", dims=[64], batch=8, r2r="DCT2"),
    dict(mode="r2r", dims=[17, 34], batch=1, r2r="DST3"),
    dict(mode="r2r", dims=[100], batch=4, r2r="DCT4", inverse=True, normalize=True),
    dict(mode="r2r", dims=[33], batch=4, r2r="DCT1"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_dd_matches_quad_oracle(V, ctx, case):
    dims, B = case["dims"], case["batch"]
    rng = np.random.default_rng(sum(dims) + B)
    inverse, normalize = case.get("inverse", False), case.get("normalize", False)
    cfg = (V.FftConfig(dims).with_batch_count(B).with_precision(V.Precision.DOUBLE_DOUBLE)
           .with_inverse_normalization(normalize))
    d = V.Direction.INVERSE if inverse else V.Direction.FORWARD
    nd, N = len(dims), int(np.prod(dims))
    shape = (B,) + tuple(dims)
    dev = ctx.device_profile()
    if case["mode"] == "c2c":
        x = dd_words(rng, shape, True)
        ir = V.TransformIr.build(cfg, d, dev)
        ref = oracle.dd_fft_nd(x, nd, inverse=inverse, normalize=normalize)
    elif case["mode"] == "r2c":
        x = dd_words(rng, shape, False)
        ir = V.TransformIr.build(cfg.with_transform(V.TransformKind.R2C), V.Direction.FORWARD, dev)
        ref = oracle.dd_r2c_nd(x, nd)
    else:
        x = dd_words(rng, shape, False)
        ir = V.TransformIr.build(cfg.with_transform(V.TransformKind[case["r2r"]]), d, dev)
        ref = oracle.dd_r2r_nd(x, case["r2r"], nd, inverse=inverse, normalize=normalize)
    got = ctx.execute_transform_double_double(ir, x.ravel())
    err = oracle.dd_max_abs_diff(got, ref)
    assert err <= 2e-30 * N, (case, err)


@pytest.mark.gpu
@pytest.mark.parametrize("dims,batch", [([4096], 512), ([1024, 1024], 1), ([65537], 8)])
def test_dd_round_trip_at_size(V, ctx, dims, batch):
    """Forward then normalised inverse restores the input to double-double accuracy (the
    oracle's O(n^2) sums are too slow at these sizes); includes a four-step 4096 line,
    2D and a Bluestein axis."""
    rng = np.random.default_rng(7)
    shape = (batch,) + tuple(dims)
    x = dd_words(rng, shape, True)
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision.DOUBLE_DOUBLE)
    dev = ctx.device_profile()
    fwd = V.TransformIr.build(cfg, V.Direction.FORWARD, dev)
    inv = V.TransformIr.build(cfg.with_inverse_normalization(True), V.Direction.INVERSE, dev)
    y = ctx.execute_transform_double_double(fwd, x.ravel())
    back = ctx.execute_transform_double_double(inv, y)
    assert oracle.dd_max_abs_diff(back, x) <= 1e-28


@pytest.mark.gpu
def test_dd_c2r_inverts_r2c(V, ctx):
    rng = np.random.default_rng(3)
    dims, B = [48, 90], 2
    x = dd_words(rng, (B,) + tuple(dims), False)
    cfg = V.FftConfig(dims).with_batch_count(B).with_precision(V.Precision.DOUBLE_DOUBLE)
    dev = ctx.device_profile()
    r2c = V.TransformIr.build(cfg.with_transform(V.TransformKind.R2C), V.Direction.FORWARD, dev)
    c2r = V.TransformIr.build(cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True),
                              V.Direction.INVERSE, dev)
    spec = ctx.execute_transform_double_double(r2c, x.ravel())
    assert oracle.dd_max_abs_diff(spec, oracle.dd_r2c_nd(x, 2)) <= 2e-30 * 48 * 90
    back = ctx.execute_transform_double_double(c2r, spec)
    assert oracle.dd_max_abs_diff(back, x) <= 1e-29
