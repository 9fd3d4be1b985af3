"""ctypes front end of the CPU kernel emulator (libb200fft_emu.so) -- TEST INFRASTRUCTURE ONLY.

The emulator runs the product's lowering and the kernel's op functions on the host
(see emulate.cpp).  It is built with AddressSanitizer, so it is loaded in a child
process that preloads the ASan runtime (`run_cases`)."""
import ctypes
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libb200fft_emu.so")
ASAN = "/usr/lib/x86_64-linux-gnu/libasan.so.8"
LIBSTDCXX = "/usr/lib/x86_64-linux-gnu/libstdc++.so.6"


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def available():
    return os.path.exists(ASAN)


def _load():
    root = os.path.dirname(os.path.dirname(HERE))
    sys.path.insert(0, os.path.join(root, "vkfft-rs_b200"))
    import vkfft_rs as V
    lib = ctypes.CDLL(LIB)
    lib.b200fft_emu_run.argtypes = [ctypes.POINTER(V._Config), ctypes.c_int, ctypes.POINTER(V._Device),
                                    ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_size_t,
                                    ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int)]
    lib.b200fft_emu_run.restype = ctypes.c_int
    return V, lib


def emulate(V, lib, cfg, direction, device, x, out_elems, out_dtype):
    x = np.ascontiguousarray(x)
    out = np.empty(out_elems, dtype=out_dtype)
    err = ctypes.create_string_buffer(512)
    launches = ctypes.c_int(0)
    st = lib.b200fft_emu_run(ctypes.byref(cfg._s), int(direction), ctypes.byref(device._c()), x.ctypes.data,
                             x.nbytes, out.ctypes.data, out.nbytes, err, 512, ctypes.byref(launches))
    if st != 0:
        raise V.VkFftError(st, err.value.decode())
    return out, launches.value


def run_cases(cases, timeout=900):
    """Run a list of case dicts in a child process with ASan preloaded; returns results."""
    env = dict(os.environ)
    # libstdc++ after the ASan runtime: its __cxa_throw interceptor needs the real symbol
    # to be resolvable when the host process (python) does not link libstdc++ itself
    env["LD_PRELOAD"] = ASAN + " " + LIBSTDCXX
    env["ASAN_OPTIONS"] = "detect_leaks=0:verify_asan_link_order=0:abort_on_error=1"
    proc = subprocess.run([sys.executable, os.path.join(HERE, "runner.py")], input=json.dumps(cases),
                          capture_output=True, text=True, env=env, timeout=timeout)
    if proc.returncode != 0:
        raise RuntimeError(f"emulator child failed (rc={proc.returncode}):\n{proc.stderr[-4000:]}")
    return json.loads(proc.stdout.strip().splitlines()[-1])
