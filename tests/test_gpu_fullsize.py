"""Parity at the BASELINE sizes: every config runs at its stated shape on the B200, through
the C ABI on device buffers, and is checked against the CPU oracle (the restatement of
vkfft-rs src/reference.rs) on sampled lines, planes and pencils, plus a full
forward -> normalised-inverse round trip on the device.

The reference itself reports an error beside its one published large case
(docs/PORTING_PLAN.md:281, N=524288 x 8); these tests do the same for the BASELINE shapes:
  config 2  C2C 4096 x 65536 (the persistent kernel's loop runs ~150 line groups per CTA),
            R2C / C2R 4096 x 65536
  config 3  C2C 512^3, R2C 1024^3
  config 4  [1024, 17, 65537] f32 / f64, 4099 x 16384 (Bluestein and recursive-Rader
            tunings) f32 / f64, 65537 x 2048 f32 / f64
  config 5  64 images 2048^2 convolved with the sigma = 8 Gaussian
Sampled batch lines are compared with the oracle's transform of the same input lines.  For
an ND transform, a plane n0 of the transform over the faster axes (Z, the same dims without
the outermost one, batched over it) is compared with the oracle's transform of the input
plane, and pencils Y[:, k1, k2] of the full transform with the oracle's axis-0 transform of
the pencils Z[:, k1, k2] -- together they pin every axis of the full-size tensor.
Tolerances: relative L2 <= 2e-6 (f32) / 1e-13 (f64) for each transform, twice that for a
forward + inverse round trip (two transforms' rounding) -- or, where the reference's own
algorithm loses more than that, 1.25 times the oracle's round-trip error on sampled lines:
the reference evaluates the Bluestein chirp angle pi*i*i/N in f64 without reducing i*i
mod 2N (reference.rs:121-125), a phase error of ~1e-11 relative at N = 65537 that the
GPU reproduces in both directions, so an f64 round trip through it cannot reach 2e-13."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

TOL = {"F32": 2e-6, "F64": 1e-13}
TDT = {"F32": torch.float32, "F64": torch.float64}
REC_TUNING = dict(min_rader_direct_prime=17, max_rader_direct_prime=89, min_rader_fft_prime=17,
                  max_rader_fft_prime=16384, allow_recursive_fft_rader=True)


@pytest.fixture(autouse=True)
def _release_device_memory():
    yield
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def dev_uniform(scalars, prec, seed, lo=-1.0, hi=1.0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    t = torch.rand(scalars, generator=g, device="cuda", dtype=TDT[prec])
    return t.mul_(hi - lo).add_(lo)


def dev_normal(scalars, prec, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return torch.randn(scalars, generator=g, device="cuda", dtype=TDT[prec])


def execute(ctx, ir, x, out_scalars):
    """b200fft_execute on device buffers (caller-provided workspace), errors checked."""
    y = torch.empty(out_scalars, dtype=x.dtype, device="cuda")
    ws = torch.empty(max(ir.workspace_bytes, 1), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    ctx.execute_resident(ir, x.data_ptr(), y.data_ptr(), ws.data_ptr(), s)
    ctx.synchronize(s)
    del ws
    return y


def sample_lines(batch, k=16, seed=0):
    """First, second, middle and last line plus random ones (covers every CTA iteration of
    the persistent kernels: the last line is in the last line group)."""
    rng = np.random.default_rng(seed)
    fixed = {0, 1, batch // 2, batch - 1}
    rest = rng.choice(batch, size=min(batch, k) - len(fixed), replace=False)
    return np.array(sorted(fixed | set(int(v) for v in rest)))[:k]


def to_c128(t):
    a = t.double().cpu().numpy()
    return a[..., 0::2] + 1j * a[..., 1::2]


def to_f64(t):
    return t.double().cpu().numpy()


def dev_rel_l2(a, b, chunk=1 << 27):
    """relative L2 of a against b over the whole device tensors, accumulated in f64."""
    num = torch.zeros((), dtype=torch.float64, device="cuda")
    den = torch.zeros((), dtype=torch.float64, device="cuda")
    for u, v in zip(a.reshape(-1).split(chunk), b.reshape(-1).split(chunk)):
        d = u.double() - v.double()
        num += (d * d).sum()
        vv = v.double()
        den += (vv * vv).sum()
    return float((num / den).sqrt())


def build(V, ctx, dims, batch, prec, direction, kind=None, tuning=None):
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    cfg = cfg.with_inverse_normalization(True)
    if kind is not None:
        cfg = cfg.with_transform(kind)
    if tuning is not None:
        cfg = cfg.with_tuning(V.PlannerTuning(**tuning))
    return V.TransformIr.build(cfg, direction, ctx.device_profile())


def round_trip_tol(lines_in, prec):
    """2 x the per-transform tolerance, or 1.25 x the oracle's own forward + normalised
    inverse error on these lines when the reference's algorithm loses more."""
    fwd = oracle.fft_nd(lines_in, 1)
    back = oracle.fft_nd(fwd, 1, inverse=True, normalize=True)
    return max(2 * TOL[prec], 1.25 * rel_l2(back, lines_in))


def exact_err_bound(lines_in, prec, inverse=False):
    """Relative L2 of the oracle itself against an exact DFT on these lines: the reference's
    CPU path computes 4099 by Bluestein with an unreduced f64 chirp (8e-13 relative), which
    an exact planned algorithm (Rader) does not reproduce."""
    ref = oracle.fft_nd(lines_in, 1, inverse=inverse, normalize=inverse)
    exact = np.fft.ifft(lines_in, axis=-1) if inverse else np.fft.fft(lines_in, axis=-1)
    return ref, exact, rel_l2(ref, exact)


# ---- batched 1D C2C: configs 2 and 4 ------------------------------------------------

C2C_1D = [
    pytest.param(4096, 65536, "F32", None, 1, id="config2-c2c-4096x65536"),
    pytest.param(4099, 16384, "F32", None, 3, id="config4-4099x16384-bluestein-f32"),
    pytest.param(4099, 16384, "F64", None, 3, id="config4-4099x16384-bluestein-f64"),
    pytest.param(4099, 16384, "F32", REC_TUNING, 3, id="config4-4099x16384-rader-f32"),
    pytest.param(4099, 16384, "F64", REC_TUNING, 3, id="config4-4099x16384-rader-f64"),
    pytest.param(65537, 2048, "F32", None, 3, id="config4-65537x2048-f32"),
    pytest.param(65537, 2048, "F64", None, 3, id="config4-65537x2048-f64"),
]


@pytest.mark.parametrize("n,batch,prec,tuning,seed", C2C_1D)
def test_batched_c2c_at_baseline_size(V, ctx, n, batch, prec, tuning, seed):
    fwd = build(V, ctx, [n], batch, prec, V.Direction.FORWARD, tuning=tuning)
    inv = build(V, ctx, [n], batch, prec, V.Direction.INVERSE, tuning=tuning)
    x = dev_uniform(batch * n * 2, prec, seed)
    y = execute(ctx, fwd, x, x.numel())
    idx = sample_lines(batch, seed=seed)
    idx_t = torch.from_numpy(idx).cuda()
    xs = to_c128(x.view(batch, 2 * n)[idx_t])
    ys = to_c128(y.view(batch, 2 * n)[idx_t])
    ref, exact, oracle_err = exact_err_bound(xs, prec)
    if fwd.axis_child(0).kind == V.AlgorithmKind.RADER:
        assert rel_l2(ys, exact) <= TOL[prec]
        assert rel_l2(ys, ref) <= TOL[prec] + 1.05 * oracle_err
    else:
        assert rel_l2(ys, ref) <= TOL[prec], (fwd.axis_child(0), rel_l2(ys, ref))
    z = execute(ctx, inv, y, y.numel())
    zs = to_c128(z.view(batch, 2 * n)[idx_t])
    iref, iexact, ierr = exact_err_bound(ys, prec, inverse=True)
    if inv.axis_child(0).kind == V.AlgorithmKind.RADER:
        assert rel_l2(zs, iexact) <= TOL[prec]
    else:
        assert rel_l2(zs, iref) <= TOL[prec]
    assert dev_rel_l2(z, x) <= round_trip_tol(xs, prec)


def test_config2_r2c_c2r_at_baseline_size(V, ctx):
    n, batch, prec = 4096, 65536, "F32"
    fwd = build(V, ctx, [n], batch, prec, V.Direction.FORWARD, kind=V.TransformKind.R2C)
    inv = build(V, ctx, [n], batch, prec, V.Direction.INVERSE, kind=V.TransformKind.C2R)
    h = n // 2 + 1
    x = dev_uniform(batch * n, prec, 1)
    y = execute(ctx, fwd, x, batch * h * 2)
    idx_t = torch.from_numpy(sample_lines(batch, seed=1)).cuda()
    xs = to_f64(x.view(batch, n)[idx_t])
    ys = to_c128(y.view(batch, 2 * h)[idx_t])
    assert rel_l2(ys, oracle.r2c(xs)) <= TOL[prec]
    z = execute(ctx, inv, y, batch * n)
    zs = to_f64(z.view(batch, n)[idx_t])
    assert rel_l2(zs, oracle.c2r(ys, n, normalize=True)) <= TOL[prec]
    assert dev_rel_l2(z, x) <= 2 * TOL[prec]


# ---- ND: configs 3 and 4 ------------------------------------------------------------

def _pencil_points(d1, d2, seed):
    rng = np.random.default_rng(seed)
    pts = {(0, 0), (d1 - 1, d2 - 1), (d1 // 2, 1)}
    while len(pts) < 8:
        pts.add((int(rng.integers(d1)), int(rng.integers(d2))))
    return sorted(pts)


def nd_parity(V, ctx, dims, prec, seed, real=False, normal=False):
    """Full ND transform Y of dims = [d0, d1, d2] against the oracle through planes of Z (the
    transform of the faster axes, batched over d0) and pencils of Y along axis 0."""
    d0, d1, d2 = dims
    w = d2 // 2 + 1 if real else d2
    kind = V.TransformKind.R2C if real else None
    fwd = build(V, ctx, dims, 1, prec, V.Direction.FORWARD, kind=kind)
    sub = build(V, ctx, [d1, d2], d0, prec, V.Direction.FORWARD, kind=kind)
    in_scalars = d0 * d1 * d2 * (1 if real else 2)
    out_scalars = d0 * d1 * w * 2
    x = dev_normal(in_scalars, prec, seed) if normal else dev_uniform(in_scalars, prec, seed)
    pts = _pencil_points(d1, w, seed)
    y = execute(ctx, fwd, x, out_scalars)
    yv = y.view(d0, d1, w, 2)
    y_pencils = np.stack([yv[:, a, b, 0].double().cpu().numpy() + 1j * yv[:, a, b, 1].double().cpu().numpy()
                          for a, b in pts])
    del y, yv
    torch.cuda.empty_cache()
    z = execute(ctx, sub, x, out_scalars)
    zv = z.view(d0, d1, w, 2)
    z_pencils = np.stack([zv[:, a, b, 0].double().cpu().numpy() + 1j * zv[:, a, b, 1].double().cpu().numpy()
                          for a, b in pts])
    planes = sorted({0, d0 // 3, d0 - 1})
    for p in planes:
        zp = to_c128(z.view(d0, d1 * w * 2)[p]).reshape(d1, w)
        if real:
            xp = to_f64(x.view(d0, d1, d2)[p])
            ref = oracle.r2c_nd(xp, 2)
        else:
            xp = to_c128(x.view(d0, d1, 2 * d2)[p])
            ref = oracle.fft_nd(xp, 2)
        assert rel_l2(zp, ref) <= TOL[prec], ("plane", p, rel_l2(zp, ref))
    del z, zv
    torch.cuda.empty_cache()
    ref = oracle.fft_nd(z_pencils, 1)
    assert rel_l2(y_pencils, ref) <= TOL[prec], ("pencils", rel_l2(y_pencils, ref))
    return fwd, x


def nd_round_trip(V, ctx, dims, prec, x, real=False):
    """relative L2 of inverse(forward(x)) against x over the whole tensor, and its bound
    (round_trip_tol on lines of the fastest axis, which carries the slowest-converging
    algorithm of the BASELINE ND shapes)."""
    d0, d1, d2 = dims
    w = d2 // 2 + 1 if real else d2
    fwd = build(V, ctx, dims, 1, prec, V.Direction.FORWARD, kind=V.TransformKind.R2C if real else None)
    inv = build(V, ctx, dims, 1, prec, V.Direction.INVERSE, kind=V.TransformKind.C2R if real else None)
    y = execute(ctx, fwd, x, d0 * d1 * w * 2)
    z = execute(ctx, inv, y, x.numel())
    del y
    idx_t = torch.from_numpy(sample_lines(d0 * d1, k=8, seed=d2)).cuda()
    if real:
        lines = to_f64(x.view(d0 * d1, d2)[idx_t]).astype(np.complex128)
    else:
        lines = to_c128(x.view(d0 * d1, 2 * d2)[idx_t])
    return dev_rel_l2(z, x), round_trip_tol(lines, prec)


def test_config3_c2c_512cubed(V, ctx):
    dims = [512, 512, 512]
    _, x = nd_parity(V, ctx, dims, "F32", 2, normal=True)
    err, tol = nd_round_trip(V, ctx, dims, "F32", x)
    assert err <= tol


def test_config3_r2c_1024cubed(V, ctx):
    dims = [1024, 1024, 1024]
    _, x = nd_parity(V, ctx, dims, "F32", 2, real=True, normal=True)
    err, tol = nd_round_trip(V, ctx, dims, "F32", x, real=True)
    assert err <= tol


@pytest.mark.parametrize("prec", ["F32", "F64"])
def test_config4_1024x17x65537(V, ctx, prec):
    dims = [1024, 17, 65537]
    fwd, x = nd_parity(V, ctx, dims, prec, 3)
    assert [fwd.axis_child(k).kind.name for k in range(3)] == ["STOCKHAM", "RADER", "BLUESTEIN"]
    err, tol = nd_round_trip(V, ctx, dims, prec, x)
    assert err <= tol, (err, tol)


# ---- config 5: ND real convolution ---------------------------------------------------

def gaussian_spectrum(dims, sigma=8.0):
    """Compact R2C spectrum of a centred Gaussian normalised to sum 1, shifted to the origin
    (exp(-r^2 / 2 sigma^2) over the circular distance to pixel (0, 0))."""
    h, w = dims
    yy = np.minimum(np.arange(h), h - np.arange(h))[:, None].astype(np.float64)
    xx = np.minimum(np.arange(w), w - np.arange(w))[None, :].astype(np.float64)
    g = np.exp(-(yy * yy + xx * xx) / (2 * sigma * sigma))
    g /= g.sum()
    return np.fft.rfft2(g)


def test_config5_convolution_64x2048sq(V, ctx):
    dims, C = [2048, 2048], 64
    n = dims[0] * dims[1]
    spec = gaussian_spectrum(dims)
    cfg = (V.FftConfig(dims).with_transform(V.TransformKind.R2C).with_convolution(True)
           .with_coordinate_features(C))
    conv = V.NdRealConvolutionIr.build_from_spectrum(cfg, spec.astype(np.complex64), ctx.device_profile())
    x = dev_uniform(C * n, "F32", 4, lo=0.0, hi=1.0)
    y = torch.empty_like(x)
    ws = torch.empty(max(conv.workspace_bytes, 1), dtype=torch.uint8, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    ctx.execute_nd_real_convolution_resident(conv, x.data_ptr(), y.data_ptr(), ws.data_ptr(), s)
    ctx.synchronize(s)
    for img in (0, 37, C - 1):
        xi = to_f64(x.view(C, n)[img]).reshape(dims)
        yi = to_f64(y.view(C, n)[img]).reshape(dims)
        # the device holds the f32-rounded spectrum: the oracle convolves with the same values
        ref = oracle.convolve_nd(xi, spec.astype(np.complex64), dims, 1)
        assert rel_l2(yi, ref) <= TOL["F32"], (img, rel_l2(yi, ref))
