"""The ahead-of-time specialised pass kernels (no GPU needed): every generic pass of the
BASELINE configurations 3-5 and of the reference's published lengths runs a precompiled
sm_100a kernel specialised for its structure -- the build's catalogue covers them -- and no
run-time compiler is part of the library."""
import os
import subprocess

import pytest

REC = dict(min_rader_direct_prime=17, max_rader_direct_prime=89, min_rader_fft_prime=17, max_rader_fft_prime=16384,
           allow_recursive_fft_rader=True)

CASES = [
    # BASELINE config 4 (both precisions, both tunings of 4099) and 5
    ("c2c", [1024, 17, 65537], 1, "F32", None), ("c2c", [1024, 17, 65537], 1, "F64", None),
    ("c2c", [4099], 16384, "F32", None), ("c2c", [4099], 16384, "F64", None),
    ("c2c", [4099], 16384, "F32", REC), ("c2c", [4099], 16384, "F64", REC),
    ("c2c", [65537], 2048, "F32", None), ("c2c", [65537], 2048, "F64", None),
    # any larger batch of a catalogued shape has the same pass structure
    ("c2c", [4099], 100000, "F32", None), ("c2c", [65537], 4096, "F64", None),
    # the reference's published pair lengths and family representatives
    ("c2c", [103], 64, "F32", None), ("c2c", [257], 64, "F64", None), ("c2c", [5760], 64, "F32", None),
    ("c2c", [4089], 64, "F32", REC), ("c2c", [131072], 256, "F32", None), ("r2c", [8704], 256, "F64", None),
    ("c2r", [206], 256, "F32", None), ("c2c", [360], 512, "DOUBLE_DOUBLE", None),
]


def profile(V):
    return V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA).replace(
        shared_memory_bytes=49152, shared_memory_pow2_bytes=32768, max_threads_per_block=1024,
        max_workgroup_size=[1024, 1024, 64])


@pytest.mark.parametrize("kind,dims,batch,prec,tuning", CASES,
                         ids=[f"{c[0]}-{c[1]}x{c[2]}-{c[3]}{'-rec' if c[4] else ''}" for c in CASES])
def test_catalogue_covers_every_generic_pass(V, kind, dims, batch, prec, tuning):
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    if kind == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
    elif kind == "c2r":
        cfg = cfg.with_transform(V.TransformKind.C2R)
    if tuning:
        cfg = cfg.with_tuning(V.PlannerTuning(**tuning))
    for direction, norm in ((V.Direction.FORWARD, False), (V.Direction.INVERSE, True)):
        if kind == "r2c" and direction == V.Direction.INVERSE:
            continue
        if kind == "c2r" and direction == V.Direction.FORWARD:
            continue
        ir = V.TransformIr.build(cfg.with_inverse_normalization(norm), direction, profile(V))
        covered, total = ir.specialised_passes
        # every generic pass is specialised (the BASELINE 65537 / 17 axes have none left:
        # they run the register kernels)
        assert covered == total, (dims, direction, covered, total)


def test_config5_convolution_is_covered(V):
    import numpy as np
    dims = [2048, 2048]
    cfg = (V.FftConfig(dims).with_transform(V.TransformKind.R2C).with_convolution(True)
           .with_coordinate_features(64))
    spec = np.zeros(2048 * 1025, dtype=np.complex64)
    conv = V.NdRealConvolutionIr.build_from_spectrum(cfg, spec, profile(V))
    assert conv.specialised_passes[0] == conv.specialised_passes[1]


def test_uncatalogued_shape_runs_the_interpreter(V):
    # a Bluestein length outside the catalogue: its passes run the precompiled interpreter
    ir = V.TransformIr.build(V.FftConfig([4001 * 3]).with_batch_count(7), V.Direction.FORWARD, profile(V))
    covered, total = ir.specialised_passes
    assert total >= 1 and covered < total


def test_library_links_no_runtime_compiler(V):
    lib = os.path.join(os.path.dirname(V.__file__), os.pardir, "libb200fft.so")
    out = subprocess.run(["ldd", os.path.abspath(lib)], capture_output=True, text=True).stdout
    assert "nvrtc" not in out and "libnvJitLink" not in out, out



@pytest.mark.parametrize("dims,prec,labels", [
    ([4096], "F32", ["register stockham (bulk prefetch)"]),
    ([4096], "F64", ["register stockham"]),
    ([512, 512, 512], "F32", ["register stockham (bulk prefetch)", "register stockham", "register stockham"]),
])
def test_pass_labels_name_each_launch(V, cuda_profile, dims, prec, labels):
    """b200fft_transform_describe_passes lists the kernel kind of every launch: dense
    contiguous f32 lines take the bulk-copy prefetch kernel, strided and f64 lines the
    ordinary register kernel."""
    ir = V.TransformIr.build(V.FftConfig(dims).with_batch_count(64 if len(dims) == 1 else 1)
                             .with_precision(V.Precision[prec]), V.Direction.FORWARD, cuda_profile)
    assert ir.pass_labels == labels
    assert len(ir.pass_labels) == ir.launch_count
