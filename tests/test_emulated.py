"""CPU emulation of the B200 launch programs (tests/emulator): the product's lowering and
the kernel's op functions executed thread by thread on the host, under AddressSanitizer,
against the oracle.  Catches lowering and index errors without a GPU; the GPU parity
suite (test_gpu_parity.py) is the parity claim itself."""
import pytest

import emulator

pytestmark = pytest.mark.skipif(not emulator.available(), reason="AddressSanitizer runtime not installed")

TOL = {"F32": 2e-6, "F64": 1e-13, "DD": 1.0}  # DD: error / (2e-30 N) or relL2 / 1e-15 (f64 storage)
REC = dict(min_rader_direct_prime=17, max_rader_direct_prime=89, min_rader_fft_prime=17, max_rader_fft_prime=16384,
           allow_recursive_fft_rader=True)

CASES = [
    dict(kind="c2c", dims=[1024], batch=3, prec="F32"),
    dict(kind="c2c", dims=[4096], batch=1, prec="F64", inverse=True, normalize=True),
    dict(kind="c2c", dims=[360], batch=3, prec="F64"),
    dict(kind="c2c", dims=[11 * 13 * 2], batch=2, prec="F32"),
    dict(kind="c2c", dims=[17], batch=40, prec="F64"),
    dict(kind="c2c", dims=[47], batch=9, prec="F64"),
    dict(kind="c2c", dims=[89], batch=9, prec="F32"),
    dict(kind="c2c", dims=[17 * 17], batch=2, prec="F64"),
    dict(kind="c2c", dims=[83 * 4], batch=2, prec="F64", inverse=True, normalize=True),
    dict(kind="c2c", dims=[4099], batch=1, prec="F32"),
    dict(kind="c2c", dims=[4099], batch=1, prec="F64"),
    dict(kind="c2c", dims=[65536 * 2], batch=1, prec="F32"),
    dict(kind="c2c", dims=[8, 16], batch=2, prec="F64"),
    dict(kind="c2c", dims=[6, 17, 10], batch=1, prec="F64", inverse=True, normalize=True),
    dict(kind="c2c", dims=[3, 1, 47], batch=2, prec="F64"),
    dict(kind="r2c", dims=[4096], batch=2, prec="F32"),
    dict(kind="r2c", dims=[30], batch=3, prec="F64"),
    dict(kind="r2c", dims=[45], batch=3, prec="F64"),
    dict(kind="r2c", dims=[94], batch=3, prec="F64"),
    dict(kind="r2c", dims=[206], batch=2, prec="F64"),
    dict(kind="r2c", dims=[17, 34], batch=1, prec="F64"),
    dict(kind="c2r", dims=[4096], batch=2, prec="F32", normalize=True),
    dict(kind="c2r", dims=[206], batch=2, prec="F64", normalize=True),
    dict(kind="c2r", dims=[45], batch=2, prec="F64", normalize=True),
    dict(kind="c2r", dims=[12, 30], batch=1, prec="F64", normalize=True),
    # nested and pass-level Rader (recursive tuning), Rader four-step, f64 CT x Bluestein
    dict(kind="c2c", dims=[107], batch=3, prec="F64", tuning=REC),
    dict(kind="c2c", dims=[683], batch=2, prec="F32", tuning=REC),
    dict(kind="c2c", dims=[4099], batch=2, prec="F32", tuning=REC),
    dict(kind="r2c", dims=[8704], batch=1, prec="F64"),
    dict(kind="c2r", dims=[8704], batch=1, prec="F64", normalize=True),
    dict(kind="r2c", dims=[4106], batch=1, prec="F64"),
    dict(kind="c2r", dims=[4106], batch=1, prec="F64", normalize=True),
    dict(kind="c2c", dims=[4106], batch=1, prec="F64", inverse=True, normalize=True),
    dict(kind="c2c", dims=[17 * 4096], batch=1, prec="F32"),
    dict(kind="c2r", dims=[3, 206], batch=1, prec="F64", normalize=True),
    # FFT convolution: fused outermost axis (K = 1), K > 1 fan-out, conjugation + cross power,
    # broadcast kernel, Rader / Bluestein / four-step outer axes
    dict(kind="conv", dims=[32, 48], batch=1, prec="F32", coords=3),
    dict(kind="conv", dims=[16, 12, 20], batch=1, prec="F64", coords=2, copies=1),
    dict(kind="conv", dims=[32, 48], batch=1, prec="F64", coords=2, kernels=3),
    dict(kind="conv", dims=[30, 34], batch=1, prec="F64", coords=2, conj=True, cross=True),
    dict(kind="conv", dims=[97, 40], batch=1, prec="F64", coords=1),
    dict(kind="conv", dims=[4099, 6], batch=1, prec="F32", coords=1),
    dict(kind="conv", dims=[8192, 6], batch=1, prec="F32", coords=1, kernels=2),
    # slab decomposition: every rank's programs, the exchange pass scattering into the
    # ranks' exchange buffers (all ranks emulated in one process)
    dict(kind="slab", mode="c2c", dims=[8, 12, 10], batch=1, prec="F64", nranks=2),
    dict(kind="slab", mode="c2c_inv", dims=[8, 12, 10], batch=1, prec="F64", nranks=4, normalize=True),
    dict(kind="slab", mode="r2c", dims=[8, 16, 12], batch=1, prec="F64", nranks=4),
    dict(kind="slab", mode="c2r", dims=[8, 16, 12], batch=1, prec="F64", nranks=2, normalize=True),
    dict(kind="slab", mode="c2c", dims=[16, 24], batch=1, prec="F32", nranks=8),
    dict(kind="slab", mode="c2c_inv", dims=[16, 24], batch=1, prec="F32", nranks=2),
    dict(kind="slab", mode="c2c", dims=[34, 18, 17], batch=1, prec="F64", nranks=2),
    dict(kind="slab", mode="c2c", dims=[4, 4, 6, 10], batch=1, prec="F64", nranks=2),
    dict(kind="slab", mode="c2r", dims=[4, 4, 6, 10], batch=1, prec="F64", nranks=2, normalize=True),
    dict(kind="slab", mode="c2c", dims=[8, 8, 8], batch=1, prec="F64", nranks=1),
    dict(kind="slab", mode="c2c", dims=[4099 * 2, 4, 3], batch=1, prec="F32", nranks=2),
    dict(kind="slab", mode="c2c_inv", dims=[4099 * 2, 4, 3], batch=1, prec="F32", nranks=2, normalize=True),
    # zero padding (spatial / frequency, every boundary) and formatted buffer strides
    dict(kind="bnd", mode="c2c", dims=[64], batch=3, prec="F64", pad={"0": [40, 64]}),
    dict(kind="bnd", mode="c2c_inv", dims=[64], batch=3, prec="F64", pad={"0": [10, 20]}, normalize=True),
    dict(kind="bnd", mode="c2c", dims=[16, 12, 10], batch=2, prec="F64", pad={"0": [8, 16], "1": [6, 12], "2": [5, 10]}),
    dict(kind="bnd", mode="c2c", dims=[16, 12], batch=2, prec="F64", pad={"1": [6, 12]}, domain="frequency"),
    dict(kind="bnd", mode="c2c_inv", dims=[16, 12], batch=2, prec="F64", pad={"0": [3, 5]}, domain="frequency"),
    dict(kind="bnd", mode="r2c", dims=[34], batch=2, prec="F64", pad={"0": [7, 13]}),
    dict(kind="bnd", mode="c2r", dims=[34], batch=2, prec="F64", pad={"0": [7, 13]}),
    dict(kind="bnd", mode="r2c", dims=[6, 8], batch=2, prec="F64", pad={"0": [1, 2], "1": [2, 4]}),
    dict(kind="bnd", mode="c2c", dims=[8, 10], batch=3, prec="F64", in_strides={"0": 13}, in_batch_stride=120,
         out_strides={"0": 11}, out_batch_stride=100),
    dict(kind="bnd", mode="r2c", dims=[6, 8], batch=2, prec="F32", in_strides={"0": 9}, out_strides={"0": 7},
         out_batch_stride=50, pad={"0": [1, 2]}),
    dict(kind="bnd", mode="c2r", dims=[6, 8], batch=2, prec="F64", in_strides={"0": 6}, in_batch_stride=40,
         out_strides={"0": 10}),
    dict(kind="bnd", mode="c2c", dims=[4099], batch=2, prec="F32", pad={"0": [2000, 4099]}),
    # C2C convolution (ConvolutionIr / NdConvolutionIr) and kernelConvolution preparation
    dict(kind="cconv", dims=[64], batch=3, prec="F64"),
    dict(kind="cconv", dims=[64], batch=1, prec="F64", kernels=3),
    dict(kind="cconv", dims=[60], batch=1, prec="F64", matrix=2),
    dict(kind="cconv", dims=[60], batch=1, prec="F64", matrix=2, symmetric=True),
    dict(kind="cconv", dims=[48], batch=1, prec="F64", matrix=3, kernels=2),
    dict(kind="cconv", dims=[64], batch=2, prec="F32", conj=True, cross=True),
    dict(kind="cconv", dims=[16, 12], batch=2, prec="F64"),
    dict(kind="cconv", dims=[16, 12], batch=1, prec="F64", kernels=3),
    dict(kind="cconv", dims=[8, 6, 10], batch=1, prec="F64", matrix=3),
    dict(kind="cconv", dims=[16, 12], batch=1, prec="F64", matrix=2, symmetric=True, conj=True),
    dict(kind="cconv", dims=[4099], batch=1, prec="F32"),
    dict(kind="kprep", dims=[64], batch=2, prec="F64", coords=3),
    dict(kind="kprep", dims=[60], batch=1, prec="F32", coords=2, real=True),
    dict(kind="kprep", dims=[16, 10], batch=2, prec="F64", coords=2, real=True),
    # three-pass Bluestein on a contiguous axis (row-ordered spectrum / twiddle tables) and
    # on a strided one
    dict(kind="c2c", dims=[4099], batch=2, prec="F64"),
    dict(kind="c2c", dims=[4099], batch=1, prec="F64", inverse=True, normalize=True),
    dict(kind="c2c", dims=[65537], batch=1, prec="F32"),
    dict(kind="c2c", dims=[3, 4099], batch=1, prec="F64"),
    dict(kind="c2c", dims=[4099, 3], batch=1, prec="F64"),
    # DCT / DST (r2r_ir.rs): every kind, odd/even lengths, ND, inverse pairs, padding
    *[dict(kind="r2r", r2r=k, dims=[n], batch=3, prec=p) for k in
      ("DCT1", "DCT2", "DCT3", "DCT4", "DST1", "DST2", "DST3", "DST4") for n in (2, 17, 64) for p in ("F32", "F64")],
    *[dict(kind="r2r", r2r=k, dims=[n], batch=2, prec="F64") for k in ("DCT1", "DST4", "DCT4") for n in (3, 257, 4097)],
    dict(kind="r2r", r2r="DCT1", dims=[1025], batch=2, prec="F32"),
    dict(kind="r2r", r2r="DCT2", dims=[12, 10, 9], batch=2, prec="F64"),
    dict(kind="r2r", r2r="DST3", dims=[16, 33], batch=1, prec="F32"),
    dict(kind="r2r", r2r="DCT4", dims=[8, 12], batch=2, prec="F64", omit=[0]),
    dict(kind="r2r", r2r="DCT2", dims=[40], batch=2, prec="F64", inverse=True, normalize=True),
    dict(kind="r2r", r2r="DST1", dims=[6, 20], batch=2, prec="F64", inverse=True, normalize=True),
    dict(kind="r2r", r2r="DCT3", dims=[32, 6], batch=1, prec="F32", pad={0: (20, 32)}),
    dict(kind="r2r", r2r="DST2", dims=[32], batch=2, prec="F64", inverse=True, pad={0: (5, 9)}),
    # double-double (double_double.rs; reference tolerance: the crate's GPU gate)
    dict(kind="dd", dims=[16], batch=3, prec="DD"),
    dict(kind="dd", dims=[60], batch=2, prec="DD", inverse=True, normalize=True),
    dict(kind="dd", dims=[103], batch=1, prec="DD", tuning=dict(max_rader_fft_prime=100)),
    dict(kind="dd", dims=[257], batch=2, prec="DD"),
    dict(kind="dd", dims=[1536], batch=1, prec="DD"),
    dict(kind="dd", dims=[4096], batch=1, prec="DD", inverse=True),
    dict(kind="dd", dims=[8, 12, 10], batch=1, prec="DD"),
    dict(kind="dd", dims=[17, 34], batch=1, prec="DD", mode="r2c"),
    dict(kind="dd", dims=[64, 64], batch=1, prec="DD", mode="c2r"),
    dict(kind="dd", dims=[90], batch=2, prec="DD", mode="c2r"),
    dict(kind="dd", dims=[17, 34], batch=1, prec="DD", mode="r2r", r2r="DCT2"),
    dict(kind="dd", dims=[33], batch=2, prec="DD", mode="r2r", r2r="DST4", inverse=True, normalize=True),
    dict(kind="dd", dims=[64], batch=2, prec="DD", mode="r2r", r2r="DCT3"),
    dict(kind="dd", dims=[60], batch=2, prec="DD", precision="DOUBLE_DOUBLE_F64_STORAGE"),
    dict(kind="dd", dims=[16, 20], batch=1, prec="DD", precision="DOUBLE_DOUBLE_F64_STORAGE", mode="r2c"),
    # mixed storage / compute precision (config.rs:107-161)
    dict(kind="mixed", dims=[64], batch=3, prec="F32", precision="F16_STORAGE_F32_COMPUTE"),
    dict(kind="mixed", dims=[60], batch=2, prec="F32", precision="F16_STORAGE_F32_COMPUTE", real=True),
    dict(kind="mixed", dims=[64], batch=3, prec="F64", precision="F64_COMPUTE_F32_STORAGE"),
    dict(kind="mixed", dims=[16, 10], batch=2, prec="F64", precision="F64_COMPUTE_F32_STORAGE", real=True),
    dict(kind="mixed", dims=[4099], batch=1, prec="F64", precision="F64_COMPUTE_F32_STORAGE"),
]


@pytest.fixture(scope="module")
def results():
    emulator.build()
    return emulator.run_cases(CASES)


@pytest.mark.parametrize("i", range(len(CASES)), ids=[f"{c['kind']}{'-' + c['mode'] if 'mode' in c else ''}{'-' + c['r2r'] if 'r2r' in c else ''}"
                              f"{'-inv' if c.get('inverse') else ''}-{c['dims']}-{c['prec']}"
                              + (f"-P{c['nranks']}" if "nranks" in c else "") + (f"-pad{c['pad']}" if "pad" in c else "")
                              + ("-strided" if "in_strides" in c or "out_strides" in c else "")
                              + (f"-{c['precision']}" if "precision" in c else "") for c in CASES])
def test_emulated_program_matches_oracle(results, i):
    r = results[i]
    assert "error" not in r, r
    assert r["err"] <= TOL[CASES[i]["prec"]], (CASES[i], r)
