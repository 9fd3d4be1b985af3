"""The CPU oracle (oracle/reference_oracle.c, a restatement of vkfft-rs src/reference.rs)
checked against the FFTW 3.3.9 golden vectors the reference commits, at the reference's
CPU tolerance (tests/fftw_medium_golden.rs:161-171: max abs diff <= 2e-10 * n), and
against its own self-tests (reference.rs:156-201)."""
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fftw_golden.npz")


def golden():
    return np.load(GOLDEN)


def complex_v1(n):
    x = np.arange(n, dtype=np.float64)
    return np.sin(0.137 * x) + 0.0013 * x + 1j * (np.cos(0.071 * x) - 0.0009 * x)


def real_v1(n):
    x = np.arange(n, dtype=np.float64)
    return np.sin(0.173 * x) + 0.003 * x - 0.27 * np.cos(0.071 * x)


def complex_f32_v1(n):
    x = np.arange(n, dtype=np.float32)
    re = np.sin(np.float32(0.137) * x) + np.float32(0.0013) * x
    im = np.cos(np.float32(0.071) * x) - np.float32(0.0009) * x
    return re.astype(np.float32).astype(np.float64) + 1j * im.astype(np.float32).astype(np.float64)


def real_f32_v1(n):
    x = np.arange(n, dtype=np.float32)
    v = np.sin(np.float32(0.173) * x) + np.float32(0.003) * x - np.float32(0.27) * np.cos(np.float32(0.071) * x)
    return v.astype(np.float32).astype(np.float64)


def case_names(prefix):
    z = golden()
    return sorted({k.rsplit("/", 1)[0].split("/", 1)[1] for k in z.files if k.startswith(prefix + "/")})


@pytest.mark.parametrize("name", case_names("medium"))
def test_oracle_matches_fftw_medium(name):
    z = golden()
    shape = tuple(int(v) for v in z[f"medium/{name}/shape"])
    kind = int(z[f"medium/{name}/kind"])
    expected = z[f"medium/{name}/output"]
    n = int(np.prod(shape))
    if kind == 0:
        got = oracle.fft(complex_v1(n)).ravel()
    elif kind == 1:
        got = oracle.r2c_nd(real_v1(n).reshape(shape), len(shape)).ravel()
    else:  # ND DCT-II (FFTW REDFT10 on every axis)
        got = oracle.r2r_nd(real_v1(n).reshape(shape), "DCT2", len(shape)).ravel()
    assert np.abs(got - expected).max() <= 2e-10 * n


@pytest.mark.parametrize("name", case_names("medium_f32"))
def test_oracle_matches_fftw_medium_f32_inputs(name):
    # float-evaluated inputs (tests/fftw_medium_f32_golden.rs:111-130), f64 transform
    z = golden()
    shape = tuple(int(v) for v in z[f"medium_f32/{name}/shape"])
    kind = int(z[f"medium_f32/{name}/kind"])
    expected = z[f"medium_f32/{name}/output"]
    n = int(np.prod(shape))
    if kind == 0:
        got = oracle.fft(complex_f32_v1(n)).ravel()
    elif kind == 1:
        got = oracle.r2c_nd(real_f32_v1(n).reshape(shape), len(shape)).ravel()
    else:
        got = oracle.r2r_nd(real_f32_v1(n).reshape(shape), "DCT2", len(shape)).ravel()
    # libm sinf/cosf and numpy float32 sin/cos may differ by an ulp of the input
    assert np.abs(got - expected).max() <= 1e-4 * n


def test_oracle_matches_fftw_compact_inline_inputs():
    z = golden()
    x = z["compact/c2c-n47/input"]
    assert np.abs(oracle.fft(x) - z["compact/c2c-n47/output"]).max() <= 2e-10 * 47
    r = z["compact/r2c-n45/input"]
    assert np.abs(oracle.r2c(r) - z["compact/r2c-n45/output"]).max() <= 2e-10 * 45
    d = z["compact/dct2-n37/input"]
    assert np.abs(oracle.r2r_nd(d, "DCT2", 1) - z["compact/dct2-n37/output"]).max() <= 2e-10 * 37


@pytest.mark.parametrize("kind", ["DCT1", "DCT2", "DCT3", "DCT4", "DST1", "DST2", "DST3", "DST4"])
def test_oracle_r2r_inverse_pairs(kind):
    """Normalised inverse of every kind restores the input (inverse_partner and
    inverse_pair_scale, r2r_ir.rs:2317-2349), over two axes and a batch axis."""
    x = sample(3 * 9 * 10).reshape(3, 9, 10).real
    y = oracle.r2r_nd(oracle.r2r_nd(x, kind, 2), kind, 2, inverse=True, normalize=True)
    assert np.abs(y - x).max() <= 1e-13


def sample(n):
    x = np.arange(n, dtype=np.float64)
    return (np.sin(0.37 * x) + x * 0.01) + 1j * (np.cos(0.19 * x) - x * 0.02)


@pytest.mark.parametrize("n", [2, 3, 4, 6, 7, 11, 13, 17, 19, 31, 47, 77])
def test_oracle_fft_matches_dft(n):
    # reference.rs:177-190
    x = sample(n)
    assert np.abs(oracle.fft(x) - oracle.dft(x)).max() <= 5e-10 * n


@pytest.mark.parametrize("n", [8, 17, 47, 64])
def test_oracle_normalized_round_trip(n):
    # reference.rs:192-200
    x = sample(n)
    back = oracle.fft(oracle.fft(x), inverse=True, normalize=True)
    assert np.abs(back - x).max() < 5e-10 * n


def test_oracle_bluestein_chirp_is_unreduced():
    """The reference's f64 Bluestein chirp angle is not reduced mod 2n: at N=65537 its
    error against an exact DFT is ~1e-11 (the parity target for the GPU f64 path is the
    reference itself, which carries this error)."""
    rng = np.random.default_rng(3)
    x = rng.uniform(-1, 1, 65537) + 1j * rng.uniform(-1, 1, 65537)
    got = oracle.fft(x)
    exact = np.fft.fft(x)
    err = np.linalg.norm(got - exact) / np.linalg.norm(exact)
    assert 1e-12 < err < 1e-10


def test_oracle_next_smooth_and_c2r_round_trip():
    assert oracle.next_smooth_at_least(2 * 65537 - 1) == 131220
    assert oracle.next_smooth_at_least(2 * 4099 - 1) == 8232
    assert oracle.next_smooth_at_least(2061) == 2100
    rng = np.random.default_rng(0)
    r = rng.standard_normal((3, 30))
    back = oracle.c2r(oracle.r2c(r), 30, normalize=True)
    assert np.abs(back - r).max() < 1e-12


DD_GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "quad_dd_golden.npz")


def dd_case(z, set_name, name):
    pre = f"{set_name}/{name}/"
    return (tuple(int(v) for v in z[pre + "shape"]), int(z[pre + "kind"]), z[pre + "input"], z[pre + "output"])


def dd_oracle_for(kind, shape, words):
    """The double-double oracle applied as the fixture's kind prescribes (forward)."""
    nd = len(shape)
    if kind == 0:
        return oracle.dd_fft_nd(words.reshape(shape + (4,)), nd)
    if kind == 1:
        return oracle.dd_r2c_nd(words.reshape(shape + (2,)), nd)
    return oracle.dd_r2r_nd(words.reshape(shape + (2,)), "DCT2", nd)


@pytest.mark.parametrize("name", sorted({k.split("/")[1] for k in np.load(DD_GOLDEN).files if k.startswith("dd/")}))
def test_dd_oracle_matches_quad_goldens(name):
    """The double-double oracle (dd_oracle.c) against the crate's binary128 fixtures at the
    crate's CPU gate (tests/quad_medium_double_double_golden.rs:269: max abs <= 2e-31 * n)."""
    z = np.load(DD_GOLDEN)
    shape, kind, inp, out = dd_case(z, "dd", name)
    got = dd_oracle_for(kind, shape, inp)
    n = int(np.prod(shape))
    assert oracle.dd_max_abs_diff(got, out) <= 2e-31 * n


@pytest.mark.parametrize("name", sorted({k.split("/")[1] for k in np.load(DD_GOLDEN).files if k.startswith("dd_f64/")}))
def test_dd_oracle_matches_f64_storage_goldens(name):
    """DoubleDoubleF64Storage fixtures: binary64 inputs, outputs rounded to binary64."""
    z = np.load(DD_GOLDEN)
    shape, kind, inp, out = dd_case(z, "dd_f64", name)
    if kind == 0:
        words = np.zeros(inp.shape[:-1] + (4,))
        words[..., 0], words[..., 2] = inp[..., 0], inp[..., 1]
    else:
        words = np.zeros(inp.shape + (2,))
        words[..., 0] = inp
    got = dd_oracle_for(kind, shape, words)
    rounded = got.reshape(-1, 2).sum(axis=1)  # hi + lo rounded to binary64
    # the crate's CPU gate (tests/quad_medium_dd_f64_storage_golden.rs:210-216); only the
    # mathematically zero bins (quad residues near 1e-30) differ at all
    n = int(np.prod(shape))
    assert np.abs(rounded - out.reshape(-1)).max() <= 8e-13 * n
