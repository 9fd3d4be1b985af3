"""Device buffers that are not 16-byte aligned.

The bulk-copy prefetch kernels (contiguous register lines) read their input with
cp.async.bulk, which needs 16-byte aligned addresses; a pass whose input pointer is only
8-byte aligned (a view one complex f32 point into an allocation) runs the ordinary twin
of its kernel instead.  The result must be the same transform, checked against the
oracle."""
import numpy as np
import pytest

import oracle
from conftest import rel_l2, uniform_complex


@pytest.mark.gpu
@pytest.mark.parametrize("dims,batch", [([4096], 16), ([512, 512], 1), ([1024, 6, 10], 1), ([2048], 40)])
def test_misaligned_device_buffers_fall_back(V, ctx, dims, batch):
    torch = pytest.importorskip("torch")
    ir = V.TransformIr.build(V.FftConfig(dims).with_batch_count(batch), V.Direction.FORWARD, ctx.device_profile())
    rng = np.random.default_rng(11)
    x = uniform_complex(rng, (batch,) + tuple(dims), np.complex64)
    n = x.size
    raw_in = torch.zeros(2 * n + 4, dtype=torch.float32, device="cuda")
    raw_out = torch.zeros(2 * n + 4, dtype=torch.float32, device="cuda")
    xin = raw_in[2:2 + 2 * n]  # one complex point past the allocation's start
    xout = raw_out[2:2 + 2 * n]
    assert xin.data_ptr() % 16 == 8 and xout.data_ptr() % 16 == 8
    xin.copy_(torch.from_numpy(x.view(np.float32).ravel()).cuda())
    wsb = torch.empty(max(ir.workspace_bytes, 1), dtype=torch.uint8, device="cuda")
    ctx.execute_resident(ir, xin.data_ptr(), xout.data_ptr(), wsb.data_ptr(),
                         torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    y = xout.cpu().numpy().view(np.complex64).reshape(x.shape)
    ref = oracle.fft_nd(x.astype(np.complex128), len(dims))
    assert rel_l2(y, ref) <= 2e-6
