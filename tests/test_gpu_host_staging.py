"""Host execution with pageable and page-locked arrays.

execute_transform takes the caller's arrays as they are, as the reference's
execute_transform_f32 / _f64 take slices (native_runtime.rs:339-359).  Pinned arrays are
copied by the copy engine directly; large pageable ones go through the context's pinned
staging (chunks copied by a host thread pool, each chunk's DMA queued as it lands), small
pageable ones through the driver's pageable copy.  Every combination must give exactly
what one resident execution of the same transform gives: odd byte counts (a short last
chunk), arrays of several staging windows, the sub-batch pipeline of large batches,
asynchronous tickets, back-to-back calls of different sizes."""
import numpy as np
import pytest

from conftest import rel_l2

NP = {"F32": (np.complex64, np.float32), "F64": (np.complex128, np.float64)}
TOL = {"F32": 2e-6, "F64": 1e-13}

# (dims, batch, precision, kind); bytes per direction in the comment
CASES = [
    ([4096], 64, "F32", "c2c"),         # 2 MiB: the driver's pageable copy
    ([4099], 3, "F64", "c2c"),          # 196 752 B
    ([1000, 37], 5, "F32", "r2c"),      # real input 740 000 B, complex output 760 000 B
    ([24, 1000], 7, "F64", "c2r"),      # complex input, real output
    ([4099], 257, "F32", "c2c"),        # 8 427 544 B: staged, a short last chunk
    ([1000, 1000], 3, "F64", "r2c"),    # 24 MB real in, 12 MB complex out: staged, odd sizes
    ([65536], 80, "F32", "c2c"),        # 40 MiB: staged in several windows
    ([4096], 4096 + 37, "F32", "c2c"),  # 128 MiB: sub-batches of 32 MiB and a remainder
]


def build(V, ctx, dims, batch, prec, kind):
    cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
    direction = V.Direction.FORWARD
    if kind == "r2c":
        cfg = cfg.with_transform(V.TransformKind.R2C)
    elif kind == "c2r":
        cfg = cfg.with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
        direction = V.Direction.INVERSE
    return V.TransformIr.build(cfg, direction, ctx.device_profile())


def host_array(torch, n, dtype, pinned):
    """A flat numpy array of n elements of `dtype`, page-locked when `pinned`."""
    if not pinned:
        return np.empty(n, dtype=dtype)
    words = n * np.dtype(dtype).itemsize // 4
    return torch.empty(words, dtype=torch.float32).pin_memory().numpy().view(dtype)


def resident(torch, ctx, ir, x):
    xd = torch.from_numpy(np.ascontiguousarray(x).view(np.uint8).copy()).cuda()
    yd = torch.empty(ir.output_items * np.dtype(ir.output_dtype()).itemsize, dtype=torch.uint8, device="cuda")
    ctx.execute_resident(ir, xd.data_ptr(), yd.data_ptr(), stream=torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return yd.cpu().numpy().view(ir.output_dtype())


@pytest.mark.gpu
@pytest.mark.parametrize("dims,batch,prec,kind", CASES)
def test_host_execution_pageable_and_pinned_match_resident(V, ctx, dims, batch, prec, kind):
    torch = pytest.importorskip("torch")
    ir = build(V, ctx, dims, batch, prec, kind)
    rng = np.random.default_rng(batch + len(dims))
    words = ir.input_items * (2 if np.dtype(ir.input_dtype()).kind == "c" else 1)
    src = rng.uniform(-1, 1, words).astype(NP[prec][1]).view(ir.input_dtype())
    ref = resident(torch, ctx, ir, src)
    pipelined = ir.input_items * np.dtype(ir.input_dtype()).itemsize >= (96 << 20)
    for pin_in in (False, True):
        for pin_out in (False, True):
            x = host_array(torch, ir.input_items, ir.input_dtype(), pin_in)
            x[:] = src
            out = host_array(torch, ir.output_items, ir.output_dtype(), pin_out)
            for call in range(2):  # the staging rings are reused by the second call
                out[:] = 0
                got = ctx.execute_transform(ir, x, out=out)
                assert got is out
                if pipelined:  # sub-batch programs run the same kernels per line
                    assert rel_l2(got, ref) <= TOL[prec], (pin_in, pin_out, call)
                else:
                    assert np.array_equal(got, ref), (pin_in, pin_out, call)
            assert np.array_equal(x, src)  # copy semantics: the input is left as it was


@pytest.mark.gpu
def test_async_tickets_with_pageable_arrays(V, ctx):
    torch = pytest.importorskip("torch")
    ir = build(V, ctx, [8192], 160, "F32", "c2c")  # 10 MiB: staged
    rng = np.random.default_rng(3)
    xs = [(rng.uniform(-1, 1, ir.input_items) + 1j * rng.uniform(-1, 1, ir.input_items)).astype(np.complex64)
          for _ in range(3)]
    tickets = [ctx.submit_transform(ir, x) for x in xs]
    for x, t in zip(xs, tickets):
        got = t.wait()
        assert np.array_equal(got, resident(torch, ctx, ir, x))
