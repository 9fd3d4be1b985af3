"""b200fft_execute_static_workspace: the entry point that allocates no device memory.

Collected last (file name) so that it also runs after every other GPU test has used the
context's own scratch and tables.  Each case compares two calls in a row of the static
entry point with the ordinary resident entry point (b200fft_execute) on the same input.
The two calls agree bit for bit; against b200fft_execute they agree to the parity
tolerance, because b200fft_execute runs catalogued generic passes on their ahead-of-time
specialised kernels while the static entry point runs every generic pass on the
precompiled interpreter kernel (the same arithmetic, compiled differently)."""
import numpy as np
import pytest

NP = {"F32": (np.complex64, np.float32), "F64": (np.complex128, np.float64)}
TOL = {"F32": 2e-6, "F64": 1e-13}


def close(a, b, prec):
    import torch
    return float(torch.linalg.norm((a - b).double()) / torch.linalg.norm(b.double())) <= TOL[prec]

# transforms whose programs use scratch buffers (four-step, Bluestein, multi-axis real)
CASES = [
    dict(dims=[4099], batch=8, prec="F32", kind="c2c"),
    dict(dims=[65536 * 2], batch=2, prec="F32", kind="c2c"),
    dict(dims=[6, 17, 10], batch=1, prec="F64", kind="c2c"),
    dict(dims=[8704], batch=2, prec="F64", kind="r2c"),
    dict(dims=[12, 30], batch=3, prec="F64", kind="c2r"),
    dict(dims=[1024], batch=8, prec="F32", kind="c2c"),
]


def build(V, ctx, case):
    cfg = V.FftConfig(case["dims"]).with_batch_count(case["batch"]).with_precision(V.Precision[case["prec"]])
    direction = V.Direction.FORWARD
    if case["kind"] == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
    elif case["kind"] == "c2r":
        cfg = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        direction = V.Direction.INVERSE
    return V.TransformIr.build(cfg, direction, ctx.device_profile())


def device_buffers(ir, case, seed=0):
    import torch
    cdt, rdt = NP[case["prec"]]
    tdt = {np.float32: torch.float32, np.float64: torch.float64}[rdt]
    rng = np.random.default_rng(seed)
    n_in = ir.input_elements * (1 if case["kind"] == "r2c" else 2)
    n_out = ir.output_elements * (1 if case["kind"] == "c2r" else 2)
    x = torch.from_numpy(rng.uniform(-1, 1, n_in).astype(rdt)).cuda()
    outs = [torch.full((n_out,), float("nan"), dtype=tdt, device="cuda") for _ in range(3)]
    return x, outs


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES, ids=[f"{c['kind']}-{c['dims']}x{c['batch']}-{c['prec']}" for c in CASES])
def test_static_workspace_matches_resident_twice(V, ctx, case):
    import torch
    ir = build(V, ctx, case)
    assert ir.workspace_bytes < V.STATIC_WORKSPACE_BYTES
    x, (ref, a, b) = device_buffers(ir, case)
    s = torch.cuda.current_stream().cuda_stream
    ctx.execute_resident(ir, x.data_ptr(), ref.data_ptr(), stream=s)
    ctx.execute_static_workspace(ir, x.data_ptr(), a.data_ptr(), stream=s)
    ctx.execute_static_workspace(ir, x.data_ptr(), b.data_ptr(), stream=s)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert close(a, ref, case["prec"])


@pytest.mark.gpu
def test_static_workspace_switches_between_transforms(V, ctx):
    """A, B, A: each switch re-uploads the tables of the transform being run."""
    import torch
    s = torch.cuda.current_stream().cuda_stream
    runs = []
    for case in (CASES[0], CASES[2]):
        ir = build(V, ctx, case)
        x, (ref, a, b) = device_buffers(ir, case, seed=7)
        ctx.execute_resident(ir, x.data_ptr(), ref.data_ptr(), stream=s)
        runs.append((ir, x, ref, a, b))
    for ir, x, ref, a, b in runs:
        ctx.execute_static_workspace(ir, x.data_ptr(), a.data_ptr(), stream=s)
    ir, x, ref, a, b = runs[0]
    ctx.execute_static_workspace(ir, x.data_ptr(), b.data_ptr(), stream=s)
    torch.cuda.synchronize()
    for (ir, x, ref, a, b), case in zip(runs, (CASES[0], CASES[2])):
        assert close(a, ref, case["prec"])
    assert torch.equal(runs[0][4], runs[0][3])


@pytest.mark.gpu
def test_static_workspace_calls_allocate_no_device_memory(V, ctx):
    """After the first call on the device (symbol lookup, kernel modules loaded), further
    calls -- new transforms included, whose tables are copied in -- leave the device's
    free memory unchanged."""
    import torch
    s = torch.cuda.current_stream().cuda_stream
    warm = [build(V, ctx, c) for c in CASES]
    bufs = [device_buffers(ir, c) for ir, c in zip(warm, CASES)]
    for ir, (x, outs) in zip(warm, bufs):
        ctx.execute_static_workspace(ir, x.data_ptr(), outs[0].data_ptr(), stream=s)
    torch.cuda.synchronize()
    fresh = [build(V, ctx, c) for c in CASES]  # new transforms: never uploaded anywhere
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(2):
        for ir, (x, outs) in zip(fresh, bufs):
            ctx.execute_static_workspace(ir, x.data_ptr(), outs[1].data_ptr(), stream=s)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    for (x, outs) in bufs:
        assert torch.equal(outs[0], outs[1])


@pytest.mark.gpu
def test_static_workspace_rejects_transforms_beyond_its_size(V, ctx):
    import torch
    ir = build(V, ctx, dict(dims=[65536 * 2], batch=32, prec="F32", kind="c2c"))  # four-step: 32 MiB scratch
    assert ir.workspace_bytes > V.STATIC_WORKSPACE_BYTES
    x = torch.empty(8, dtype=torch.float32, device="cuda")  # never touched: rejected before any launch
    with pytest.raises(V.VkFftError) as e:
        ctx.execute_static_workspace(ir, x.data_ptr(), x.data_ptr())
    assert e.value.variant == "ResourceLimitExceeded"
    assert "static workspace holds" in str(e.value)
