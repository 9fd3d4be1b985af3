"""The host copy pool behind the pinned staging of pageable host arrays, on the CPU.

tests/native/copy_pool_test.cpp drives CopyPool (vkfft-rs_b200/csrc/host_staging.cpp)
with 0, 1, 3 and 7 workers, with and without idle polling: thousands of back-to-back jobs
whose every item must run exactly once, jobs whose items the caller consumes as they
finish (start / finish), and an item that throws."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = "/usr/local/cuda"


def test_copy_pool_runs_every_item_once(tmp_path):
    if shutil.which("g++") is None or not os.path.exists(os.path.join(CUDA, "include", "cuda_runtime.h")):
        pytest.skip("needs g++ and the CUDA headers")
    exe = tmp_path / "copy_pool_test"
    csrc = os.path.join(ROOT, "vkfft-rs_b200", "csrc")
    cmd = ["g++", "-O2", "-std=c++17", "-pthread", f"-I{csrc}", f"-I{CUDA}/include",
           os.path.join(ROOT, "tests", "native", "copy_pool_test.cpp"), os.path.join(csrc, "host_staging.cpp"),
           f"-L{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{CUDA}/lib64", "-o", str(exe)]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == "ok"
