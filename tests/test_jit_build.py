"""The run-time specialised pass kernels compile (NVRTC for sm_100a, no GPU needed) for
every kind of generic pass the lowering emits: mixed-radix Stockham, direct / FFT /
nested / pass-level Rader, fused and three-pass Bluestein, four-step, even-half real
pre/post processing, Hermitian expansion, f32, f64 and double-double."""
import pytest

REC = dict(min_rader_direct_prime=17, max_rader_direct_prime=89, min_rader_fft_prime=17, max_rader_fft_prime=16384,
           allow_recursive_fft_rader=True)

CASES = [
    ("c2c", [360], 3, "F64", None), ("c2c", [47], 9, "F32", None), ("c2c", [17, 34], 2, "F64", None),
    ("c2c", [4099], 2, "F32", None), ("c2c", [65537], 1, "F32", None), ("c2c", [4106], 1, "F64", None),
    ("c2c", [107], 3, "F64", REC), ("c2c", [4099], 2, "F32", REC), ("r2c", [30], 3, "F64", None),
    ("c2r", [206], 2, "F64", None), ("c2r", [45], 2, "F64", None), ("c2c", [17 * 4096], 1, "F32", None),
    ("c2c", [360], 2, "DOUBLE_DOUBLE", None), ("c2c", [103], 1, "DOUBLE_DOUBLE", None),
    ("c2c", [257], 1, "DOUBLE_DOUBLE", None), ("r2c", [34], 2, "DOUBLE_DOUBLE", None),
    ("c2c", [4096], 1, "DOUBLE_DOUBLE_F64_STORAGE", None),
]


@pytest.mark.parametrize("kind,dims,batch,prec,tuning", CASES, ids=[f"{c[0]}-{c[1]}-{c[3]}" for c in CASES])
def test_specialised_pass_kernels_compile(V, kind, dims, batch, prec, tuning):
    dev = V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA).replace(
        shared_memory_bytes=49152, shared_memory_pow2_bytes=32768, max_threads_per_block=1024,
        max_workgroup_size=[1024, 1024, 64])
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    direction = V.Direction.FORWARD
    if kind == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
    elif kind == "c2r":
        cfg = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        direction = V.Direction.INVERSE
    if tuning:
        cfg = cfg.with_tuning(V.PlannerTuning(**tuning))
    ir = V.TransformIr.build(cfg, direction, dev)
    assert ir.compile_check() >= 1
