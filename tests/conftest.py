import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "vkfft-rs_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libb200fft.so")


@pytest.fixture(scope="session")
def V():
    import vkfft_rs
    return vkfft_rs


@pytest.fixture(scope="session")
def cuda_profile(V):
    """DeviceProfile the reference reports for a B200 (cuda/runtime.rs:1204-1225):
    49152 B shared per block, 32768 pow2, 1024 threads, block dims [1024,1024,64]."""
    return V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA).replace(
        shared_memory_bytes=49152, shared_memory_pow2_bytes=32768, max_threads_per_block=1024,
        max_workgroup_size=[1024, 1024, 64])


@pytest.fixture(scope="session")
def ctx(V):
    c = V.CudaExecutionContext(0)
    yield c
    c.close()


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.complex128).ravel()
    b = np.asarray(b, dtype=np.complex128).ravel()
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def uniform_complex(rng, shape, dtype):
    re = rng.uniform(-1.0, 1.0, size=shape)
    im = rng.uniform(-1.0, 1.0, size=shape)
    return (re + 1j * im).astype(dtype)
