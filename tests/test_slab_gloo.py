"""Slab decomposition across processes on the CPU (gloo, world size 2).

Each rank builds its slab plan with the product's planner (host only), checks the
per-rank sizes it reports against the documented layouts -- slabs [D0/P, D1, ...] in,
pencils [D0, D1/P, ...] out -- and runs the decomposition itself numerically: local FFTs
of the higher axes, the all-to-all exchange over gloo, the FFT of axis 0.  The result
must equal the rank's pencil of the global transform, i.e. the layout contract the GPU
kernels implement (and that the CPU emulator checks pass by pass) is the one a
distributed caller observes."""
import os
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _worker(rank, world, port, dims, real, q):
    try:
        sys.path.insert(0, os.path.join(ROOT, "vkfft-rs_b200"))
        import torch
        import vkfft_rs as V
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        dev = V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA).replace(
            shared_memory_bytes=49152, shared_memory_pow2_bytes=32768, max_threads_per_block=1024,
            max_workgroup_size=[1024, 1024, 64])
        cfg = V.FftConfig(dims)
        if real:
            cfg = cfg.with_transform(V.TransformKind.R2C)
        slab = V.SlabTransform.build(cfg, V.Direction.FORWARD, world, rank, dev)
        D0, D1 = dims[0], dims[1]
        L0, C1 = D0 // world, D1 // world
        rest = list(dims[2:])
        if real:
            rest[-1] = rest[-1] // 2 + 1
        H = int(np.prod(rest))
        assert slab.planes_per_rank == L0 and slab.columns_per_rank == C1
        assert slab.input_elements == L0 * int(np.prod(dims[1:]))
        assert slab.output_elements == D0 * C1 * H
        rng = np.random.default_rng(11)
        x = rng.uniform(-1, 1, dims) if real else rng.uniform(-1, 1, dims) + 1j * rng.uniform(-1, 1, dims)
        mine = x[rank * L0:(rank + 1) * L0]
        # local FFTs of the higher axes
        y = np.fft.rfftn(mine, axes=list(range(1, len(dims)))) if real else np.fft.fftn(mine, axes=list(range(1, len(dims))))
        # exchange: block r = axis-1 indices of rank r, as [L0, C1, H] complex128 pairs
        send = [torch.from_numpy(np.ascontiguousarray(y[:, r * C1:(r + 1) * C1]).view(np.float64).copy())
                for r in range(world)]
        recv = [torch.empty_like(send[0]) for _ in range(world)]
        recv[rank] = send[rank]
        reqs = []
        for r in range(world):  # gloo has no all_to_all: pairwise sends and receives
            if r != rank:
                reqs.append(dist.isend(send[r], r))
                reqs.append(dist.irecv(recv[r], r))
        for req in reqs:
            req.wait()
        pencil = np.concatenate([t.numpy().view(np.complex128).reshape(L0, C1, *rest) for t in recv], axis=0)
        out = np.fft.fft(pencil, axis=0)
        assert out.size == slab.output_elements
        full = np.fft.rfftn(x) if real else np.fft.fftn(x)
        ref = full[:, rank * C1:(rank + 1) * C1]
        err = np.linalg.norm(out - ref) / np.linalg.norm(ref)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, float(err), None))
    except Exception as e:  # reported to the parent
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("dims,real", [([8, 12, 10], False), ([8, 16, 12], True), ([6, 4, 5, 8], False)])
def test_slab_layout_contract_world2(dims, real):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, dims, real, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err, exc in results:
        assert exc is None, f"rank {rank}: {exc}"
        assert err < 1e-12, (rank, err)


@pytest.mark.parametrize("dims,prec", [([512, 512, 8], "F32"), ([1024, 1024, 2], "F32"), ([512, 512, 4], "F64"),
                                       ([512, 512, 512], "F32"), ([64, 1024, 16], "F32")])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_slab_exchange_pass_tables_match_its_kernel(V, cuda_profile, dims, prec, world):
    """The exchange pass runs the peer-scatter twin of the register kernel the lowering
    picked, which may split the line into other radices (512 and 1024 f32 strided lines
    do).  Building the plan fails unless every register pass reads the stage twiddles of
    its own radix split; both directions, every rank."""
    cfg = V.FftConfig(dims).with_precision(V.Precision[prec]).with_inverse_normalization(True)
    for rank in range(world):
        for direction in (V.Direction.FORWARD, V.Direction.INVERSE):
            slab = V.SlabTransform.build(cfg, direction, world, rank, cuda_profile)
            assert slab.planes_per_rank == dims[0] // world
            slab.destroy()
