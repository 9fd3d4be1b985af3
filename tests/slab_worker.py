"""One rank of the multi-GPU slab test (launched by tests/test_gpu_slab.py under
torch.distributed.run, one process per GPU).  Host coordination over gloo; the data
path is the library's own exchange (peer stores + device barrier).

Checks, per case: forward slab transform of a seeded global tensor against the
oracle's pencil of the global transform, and the inverse back to the input.  Then the
barrier timeout: rank 1 connects but does not execute; rank 0's exchange barrier must
give up after its short limit and report through b200fft_context_synchronize."""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "vkfft-rs_b200"))
import oracle  # noqa: E402
import vkfft_rs as V  # noqa: E402

TOL = {"F32": 2e-6, "F64": 1e-13}


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.complex128).ravel()
    b = np.asarray(b, dtype=np.complex128).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def to_dev(a):
    t = torch.from_numpy(np.ascontiguousarray(a).view(np.float64 if a.dtype in (np.complex128, np.float64)
                                                       else np.float32).ravel().copy())
    return t.cuda()


def run_case(ctx, rank, world, dims, prec, real):
    cdt, rdt = (np.complex64, np.float32) if prec == "F32" else (np.complex128, np.float64)
    D0, D1 = dims[0], dims[1]
    L0, C1 = D0 // world, D1 // world
    rng = np.random.default_rng(5)
    x = rng.uniform(-1, 1, dims) if real else rng.uniform(-1, 1, dims) + 1j * rng.uniform(-1, 1, dims)
    cfg = V.FftConfig(dims).with_precision(V.Precision[prec]).with_inverse_normalization(True)
    fwd_cfg = cfg.with_transform(V.TransformKind.R2C) if real else cfg
    inv_cfg = cfg.with_transform(V.TransformKind.C2R) if real else cfg
    dev = ctx.device_profile()
    fwd = V.SlabTransform.build(fwd_cfg, V.Direction.FORWARD, world, rank, dev)
    inv = V.SlabTransform.build(inv_cfg, V.Direction.INVERSE, world, rank, dev)
    fwd.setup(ctx)
    inv.setup(ctx)
    mine = x[rank * L0:(rank + 1) * L0].astype(rdt if real else cdt)
    xin = to_dev(mine)
    spec = torch.empty(fwd.output_elements * 2, dtype=xin.dtype, device="cuda")
    back = torch.empty_like(xin)
    s = torch.cuda.current_stream().cuda_stream
    full = oracle.r2c_nd(x, len(dims)) if real else oracle.fft_nd(x, len(dims))
    ref = full[:, rank * C1:(rank + 1) * C1]
    errs = []
    for _ in range(2):  # two calls: both exchange buffers (call parity) are used
        ctx.execute_slab(fwd, xin.data_ptr(), spec.data_ptr(), stream=s)
        ctx.execute_slab(inv, spec.data_ptr(), back.data_ptr(), stream=s)
        ctx.synchronize(s)
        got = spec.cpu().numpy().view(cdt)
        errs.append(rel_l2(got, ref))
        got_back = back.cpu().numpy().view(rdt if real else cdt)
        errs.append(rel_l2(got_back, mine))
    fwd.destroy()
    inv.destroy()
    return max(errs)


def main():
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    ctx = V.CudaExecutionContext(local)
    failures = []
    cases = [([64, 32, 48], "F32", False), ([32, 64, 64], "F32", True), ([16, 24, 20], "F64", False),
             ([34, 18, 17], "F64", False), ([8198, 4, 6], "F32", False), ([128, 256], "F32", False),
             # the exchange passes of these run the strided 512- and 1024-point register
             # kernels (axis 1 forward, axis 0 inverse)
             ([512, 512, 8], "F32", False), ([1024, 1024, 2], "F32", False), ([512, 512, 4], "F64", False)]
    for dims, prec, real in cases:
        if dims[0] % world or dims[1] % world:
            continue
        err = run_case(ctx, rank, world, dims, prec, real)
        if not err <= TOL[prec]:
            failures.append((dims, prec, real, err))
    # barrier timeout: rank 1 is alive and connected but never executes
    dev = ctx.device_profile()
    slab = V.SlabTransform.build(V.FftConfig([16, 16, 16]), V.Direction.FORWARD, world, rank, dev)
    slab.setup(ctx)
    if rank == 0:
        slab.set_timeout(0.5)
        xin = torch.zeros(slab.input_elements * 2, dtype=torch.float32, device="cuda")
        out = torch.empty(slab.output_elements * 2, dtype=torch.float32, device="cuda")
        ctx.execute_slab(slab, xin.data_ptr(), out.data_ptr())
        try:
            ctx.synchronize()
            failures.append("barrier did not report the missing peer")
        except V.VkFftError as e:
            if "barrier timed out" not in str(e):
                failures.append(f"unexpected error: {e}")
        ctx.synchronize()  # the error was cleared; the context stays usable
    dist.barrier()
    slab.destroy()
    ctx.close()
    dist.destroy_process_group()
    if failures:
        print(f"rank {rank} FAILURES: {failures}", flush=True)
        return 1
    print(f"rank {rank} ok", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
