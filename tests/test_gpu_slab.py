"""Slab-decomposed transforms on the B200: one rank on one GPU (the exchange pass stores
into the rank's own exchange buffer, the barrier waits on its own flag) against the
oracle, and -- where the box has two or more GPUs -- two ranks as two processes
(tests/slab_worker.py)."""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle
from conftest import rel_l2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TOL = {"F32": 2e-6, "F64": 1e-13}


def _dev(a):
    import torch
    flat = np.ascontiguousarray(a)
    view = flat.view(np.float64 if flat.dtype in (np.complex128, np.float64) else np.float32).ravel()
    return torch.from_numpy(view.copy()).cuda()


@pytest.mark.gpu
@pytest.mark.parametrize("dims,prec,real", [([64, 32, 48], "F32", False), ([32, 64, 64], "F32", True),
                                            ([16, 24, 20], "F64", False), ([34, 18, 17], "F64", False),
                                            ([128, 256], "F32", False), ([64, 64, 64], "F64", True)])
def test_single_rank_slab_roundtrip(V, ctx, dims, prec, real):
    import torch
    cdt, rdt = (np.complex64, np.float32) if prec == "F32" else (np.complex128, np.float64)
    rng = np.random.default_rng(2)
    x = rng.uniform(-1, 1, dims) if real else rng.uniform(-1, 1, dims) + 1j * rng.uniform(-1, 1, dims)
    cfg = V.FftConfig(dims).with_precision(V.Precision[prec]).with_inverse_normalization(True)
    dev = ctx.device_profile()
    fwd = V.SlabTransform.build(cfg.with_transform(V.TransformKind.R2C) if real else cfg, V.Direction.FORWARD, 1, 0,
                                dev)
    inv = V.SlabTransform.build(cfg.with_transform(V.TransformKind.C2R) if real else cfg, V.Direction.INVERSE, 1, 0,
                                dev)
    fwd.connect(ctx, [fwd.attach(ctx)])
    inv.connect(ctx, [inv.attach(ctx)])
    xin = _dev(x.astype(rdt if real else cdt))
    spec = torch.empty(fwd.output_elements * 2, dtype=xin.dtype, device="cuda")
    back = torch.empty_like(xin)
    s = torch.cuda.current_stream().cuda_stream
    ref = oracle.r2c_nd(x, len(dims)) if real else oracle.fft_nd(x, len(dims))
    for _ in range(3):
        ctx.execute_slab(fwd, xin.data_ptr(), spec.data_ptr(), stream=s)
        ctx.execute_slab(inv, spec.data_ptr(), back.data_ptr(), stream=s)
        ctx.synchronize(s)
        assert rel_l2(spec.cpu().numpy().view(cdt), ref) <= TOL[prec]
        assert rel_l2(back.cpu().numpy().view(rdt if real else cdt), x) <= TOL[prec]
    fwd.destroy()
    inv.destroy()


@pytest.mark.gpu
def test_two_rank_slab_over_nvlink():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29600 + os.getpid() % 1000),
           os.path.join(ROOT, "tests", "slab_worker.py")]
    proc = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, cwd=ROOT)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    assert proc.stdout.count(" ok") == 2, proc.stdout
