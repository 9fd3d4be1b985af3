"""Benchmark of the B200 FFT engine on BASELINE config 2 (C2C f32, N=4096 x batch 65536,
forward then normalised inverse).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one forward + one inverse C2C pass over the whole batch.  `value` is the
aggregate GFLOP/s (5 N log2 N per complex transform, two transforms per element per
step) with the data resident in HBM; `e2e` is the same metric through the host API
(execute_transform with pinned host arrays: each step uploads its input and downloads
its result).  Under torchrun every rank processes its own 65536-transform shard (weak
scaling, no collective on the data path); times are CUDA-event durations on the
launching stream, max over ranks.  `--impl reference` times the CPU oracle (the
reference's CPU path restated in C, oracle/) on this host's cores instead.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "vkfft-rs_b200"))

N = 4096
BATCH = 65536
FLOP_PER_TRANSFORM = 5.0 * N * math.log2(N)
METRIC = "batched C2C FFT GFLOP/s (5N*log2N), N=4096 f32, forward+inverse"


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return d.get("c2c_4096_f32_bytes_per_launch")
    return None


class ClockSampler:
    """Clocks and throttle reasons of this rank's GPU during the timed region.

    Two readers: NVML, polled every millisecond between `mark_start` and `mark_end` (a
    timed region of a few tens of milliseconds still gets tens of samples, all taken with
    the GPU under this benchmark's load), and the pool's nvidia-smi clocks line, started
    before the warm-up, whose rows inside the window widened by one period are the
    fallback when NVML is unavailable.  The GPU is matched by PCI bus id, which holds
    under CUDA_VISIBLE_DEVICES and torchrun.  Only reads; no setting is changed."""

    QUERY = ("pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_MS = 50
    # NVML clocks-event reason bits (nvml.h: HwSlowdown, HwThermalSlowdown,
    # SwThermalSlowdown, SwPowerCap)
    REASON_BITS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
                   "sw_power_cap": 0x4}

    def __init__(self, device_ordinal):
        self.bus_id = None
        try:
            import torch
            pr = torch.cuda.get_device_properties(device_ordinal)  # domain / bus / device numbers
            self.bus_id = f"{pr.pci_domain_id:08X}:{pr.pci_bus_id:02X}:{pr.pci_device_id:02X}.0"
        except Exception:
            pass
        self.rows = []  # nvidia-smi: (wall time, fields)
        self.nv = []    # NVML: (sm MHz, reasons bitmask)
        self.nv_max = None
        self.proc = None
        self.t_start = self.t_end = None
        self.active = False
        self.stop = False
        self.handle = None
        self.nvml_error = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            # match this rank's GPU among NVML's devices by PCI bus id (domain width differs)
            for k in range(pynvml.nvmlDeviceGetCount()):
                h = pynvml.nvmlDeviceGetHandleByIndex(k)
                bid = pynvml.nvmlDeviceGetPciInfo(h).busId
                bid = bid.decode() if isinstance(bid, bytes) else bid
                if self.bus_id and self._same_bus(bid, self.bus_id):
                    self.handle = h
                    break
            if self.handle is None:
                raise RuntimeError(f"no NVML device with PCI bus id {self.bus_id}")
            self.nv_max = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
            pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception as e:  # the nvidia-smi rows remain
            self.handle = None
            self.nvml_error = f"{type(e).__name__}: {e}"

    @staticmethod
    def _same_bus(a, b):
        # nvidia-smi prints an 8-digit domain (00000000:1B:00.0), torch a 4-digit one
        return a.split(":", 1)[-1].upper() == b.split(":", 1)[-1].upper()

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", str(self.PERIOD_MS)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        if self.handle is not None:
            self.poller = threading.Thread(target=self._poll, daemon=True)
            self.poller.start()
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9 and (self.bus_id is None or self._same_bus(parts[0], self.bus_id)):
                self.rows.append((time.time(), parts))

    def _poll(self):
        nv = self.nvml
        while not self.stop:
            if self.active:
                try:
                    sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                    self.nv.append((sm, rs))
                except Exception:
                    pass
                time.sleep(0.001)
            else:
                time.sleep(0.002)

    def mark_start(self):
        self.t_start = time.time()
        self.active = True

    def mark_end(self):
        self.active = False
        self.t_end = time.time()
        # at least one nvidia-smi row after the window closes
        n = len(self.rows)
        t0 = time.time()
        while len(self.rows) == n and time.time() - t0 < 1.0 and self.proc and self.proc.poll() is None:
            time.sleep(0.005)

    def __exit__(self, *exc):
        self.stop = True
        self.active = False
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.nv:
            sm = [v for v, _ in self.nv]
            reasons = sorted({k for _, r in self.nv for k, bit in self.REASON_BITS.items() if r & bit})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": self.nv_max, "reasons": reasons,
                    "samples": len(sm), "sm_mhz_min": min(sm),
                    "window": "NVML polled every 1 ms inside the timed region (GPU matched by PCI bus id)"}
        rows = [r for _, r in self.rows]
        if self.t_start is not None and self.t_end is not None:
            pad = 1.5 * self.PERIOD_MS * 1e-3
            rows = [r for t, r in self.rows if self.t_start - pad <= t <= self.t_end + pad]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0,
                    "nvml_error": self.nvml_error}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows),
                "window": "nvidia-smi rows in the timed region +- one sampling period (50 ms)",
                "nvml_error": self.nvml_error}


def cpu_baseline(steps_hint=1, budget_s=12.0):
    """The CPU oracle on a bounded sample of the same workload (all host cores)."""
    import oracle
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    sample = max(threads * 2, 16)
    x = (rng.uniform(-1, 1, (sample, N)) + 1j * rng.uniform(-1, 1, (sample, N))).astype(np.complex64)
    xd = x.astype(np.complex128)
    done = 0
    t0 = time.perf_counter()
    while True:
        y = np.empty_like(xd)
        oracle.lib().oracle_fft_batch(oracle._dp(xd), oracle._dp(y), N, sample, 0, 0, threads)
        oracle.lib().oracle_fft_batch(oracle._dp(y), oracle._dp(xd), N, sample, 1, 1, threads)
        done += sample
        if time.perf_counter() - t0 >= budget_s / max(steps_hint, 1):
            break
    dt = time.perf_counter() - t0
    gflops = 2 * FLOP_PER_TRANSFORM * done / dt / 1e9
    return {"value": gflops, "unit": "GFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{done} forward+inverse pairs of N=4096 (f64 oracle) in {dt:.1f}s"}


def live_copy_gbs(stream):
    """Copy bandwidth of this GPU right now (read + write bytes of a 2 GiB device copy,
    best of 5): context for the roofline fraction, whose peak is the pool's measured one."""
    import torch
    a = torch.empty(1 << 29, dtype=torch.float32, device="cuda")
    b = torch.empty_like(a)
    best = None
    for _ in range(5):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        b.copy_(a)
        e1.record(stream)
        e1.synchronize()
        t = e0.elapsed_time(e1)
        best = t if best is None else min(best, t)
    del a, b
    return 2 * (1 << 31) / (best * 1e-3) / 1e9


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def headline_config(ws):
    """`config` of the headline line, shared by both arms."""
    return {"workload": "BASELINE config 2: C2C N=4096 x batch 65536 per rank, forward + normalised inverse",
            "global_batch": BATCH * ws, "seq_len": N, "parallelism": f"batch-sharded x{ws}",
            "l2": "inputs (2 GiB per rank) larger than L2; no flush"}


def run_reference(args):
    """The reference's CPU algorithm (the C port of src/reference.rs in oracle/) on all host
    cores, on the headline's metric and config.  A step is one forward + normalised inverse
    pass over a fixed sample of the 65536 lines, sized in the warm-up so that a step takes
    about a second; `ms_per_step` is the time of that step as run, and the time the whole
    batch would take at the same rate is reported beside it."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)

    def pair(xd, y):
        lines = xd.shape[0]
        oracle.lib().oracle_fft_batch(oracle._dp(xd), oracle._dp(y), N, lines, 0, 0, threads)
        oracle.lib().oracle_fft_batch(oracle._dp(y), oracle._dp(xd), N, lines, 1, 1, threads)

    probe = max(2 * threads, 16)
    xd = (rng.uniform(-1, 1, (probe, N)) + 1j * rng.uniform(-1, 1, (probe, N))).astype(np.complex64).astype(np.complex128)
    y = np.empty_like(xd)
    t0 = time.perf_counter()
    pair(xd, y)
    dt = time.perf_counter() - t0
    lines = int(min(BATCH, max(threads, round(probe * 1.0 / max(dt, 1e-6)))))
    lines = max(threads, lines - lines % threads) if lines >= threads else lines
    xd = (rng.uniform(-1, 1, (lines, N)) + 1j * rng.uniform(-1, 1, (lines, N))).astype(np.complex64).astype(np.complex128)
    y = np.empty_like(xd)
    for _ in range(args.warmup):
        pair(xd, y)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        pair(xd, y)
        times.append(time.perf_counter() - t0)
    step_s = statistics.mean(times)
    value = 2 * FLOP_PER_TRANSFORM * lines / step_s / 1e9
    cfg = headline_config(ws)
    cfg["sampled_fraction"] = lines / (BATCH * ws)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "ms_per_step_full_batch": step_s * 1e3 * BATCH * ws / lines,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": cfg,
        "cpu_baseline": {"value": value, "unit": "GFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"{lines} of the {BATCH * ws} lines per step (forward + normalised inverse, "
                                   f"f64 oracle), {args.steps} steps of {step_s:.2f} s"},
        "e2e": {"value": value, "unit": "GFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def headline_parity(ctx, fwd, a, b, sp, rank, dist, lines=16):
    """After the timed region: one more forward transform of the current data, and 16
    sampled lines of it (first, last and random ones, spread over every line group of the
    persistent kernel) against the CPU oracle; the max relative L2 over the ranks."""
    import torch
    import oracle
    ctx.execute_resident(fwd, a.data_ptr(), b.data_ptr(), stream=sp)
    ctx.synchronize(sp)
    rng = np.random.default_rng(100 + rank)
    idx = sorted({0, BATCH - 1} | set(int(v) for v in rng.choice(BATCH, lines - 2, replace=False)))[:lines]
    it = torch.tensor(idx, device="cuda")
    xa = a.view(BATCH, 2 * N)[it].double().cpu().numpy()
    ya = b.view(BATCH, 2 * N)[it].double().cpu().numpy()
    xs = xa[:, 0::2] + 1j * xa[:, 1::2]
    ys = ya[:, 0::2] + 1j * ya[:, 1::2]
    ref = oracle.fft_nd(xs, 1)
    err = float(np.linalg.norm(ys - ref) / np.linalg.norm(ref))
    if dist:
        t = torch.tensor([err], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        err = float(t[0])
    return {"relL2": err, "lines": len(idx), "tol": 2e-6, "ok": err <= 2e-6,
            "check": "forward transform of the data after the timed steps; sampled lines against the CPU "
                     "oracle (f64 restatement of reference.rs), max over ranks"}


def timed_steps(steps, warmup, stream, calls, dist):
    """Warm-up, then `steps` steps of `calls` bracketed by barriers and synchronisation;
    returns the device milliseconds of one step (CUDA events on `stream`), max over ranks."""
    import torch
    for _ in range(max(warmup, 3)):
        for f in calls:
            f()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        for f in calls:
            f()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    if dist:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
    return ms


def slab_section(args, ctx, dev, stream, ws, rank, dist):
    """BASELINE config 3 (C2C 512^3 f32, N(0,1) input) as the strong-scaling companion of the
    headline: on one GPU the local 3D transform, on N GPUs the slab decomposition (rank g
    owns planes g*512/N.., the all-to-all is fused into the axis-1 pass's stores over
    NVLink).  A step is one forward + one normalised inverse transform; GFLOP/s counts
    5 n log2 n per transform (n = 512^3) for the whole job.  Phase times are of one more
    forward call (max over ranks); nvlink_gbs = bytes one GPU stores into the others /
    the exchange pass's time.  Parity (N > 1): the gathered slab output against the
    single-GPU transform of the gathered input on rank 0 -- the path the full-size test
    pins to the CPU oracle at this size."""
    import torch
    import vkfft_rs as V
    D = 512
    n = D ** 3
    flop = 2 * 5.0 * n * math.log2(n)
    sp = stream.cuda_stream
    cfg = V.FftConfig([D, D, D]).with_inverse_normalization(True)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2 + rank)
    out = {"workload": "BASELINE config 3: C2C 512^3 f32, forward + normalised inverse",
           "scaling": "strong (one tensor over all GPUs)"}
    if ws == 1:
        fwd = V.TransformIr.build(cfg, V.Direction.FORWARD, dev)
        inv = V.TransformIr.build(cfg, V.Direction.INVERSE, dev)
        x = torch.randn((n * 2,), device="cuda", generator=gen)
        y = torch.empty_like(x)
        wsb = torch.empty((max(fwd.workspace_bytes, inv.workspace_bytes, 1),), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        ms = timed_steps(args.steps, args.warmup, stream,
                         [lambda: ctx.execute_resident(fwd, x.data_ptr(), y.data_ptr(), wsb.data_ptr(), sp),
                          lambda: ctx.execute_resident(inv, y.data_ptr(), x.data_ptr(), wsb.data_ptr(), sp)], None)
        ctx.synchronize(sp)
        out.update({"ms_per_step": ms, "gflops": flop / (ms * 1e-3) / 1e9, "parallelism": "1 GPU (local 3D transform)",
                    "gpu_launches_per_step": fwd.launch_count + inv.launch_count})
        return out
    fwd = V.SlabTransform.build(cfg, V.Direction.FORWARD, ws, rank, dev)
    inv = V.SlabTransform.build(cfg, V.Direction.INVERSE, ws, rank, dev)
    fwd.setup(ctx)
    inv.setup(ctx)
    fwd.set_phase_timing(True)
    x = torch.randn((fwd.input_elements * 2,), device="cuda", generator=gen)
    x0 = x.clone()
    y = torch.empty((fwd.output_elements * 2,), device="cuda")
    torch.cuda.synchronize()
    ms = timed_steps(args.steps, args.warmup, stream,
                     [lambda: ctx.execute_slab(fwd, x.data_ptr(), y.data_ptr(), stream=sp),
                      lambda: ctx.execute_slab(inv, y.data_ptr(), x.data_ptr(), stream=sp)], dist)
    ctx.synchronize(sp)
    # phases of the forward transform (from the original input), median of 3 calls
    phases = []
    for _ in range(3):
        dist.barrier()
        ctx.execute_slab(fwd, x0.data_ptr(), y.data_ptr(), stream=sp)
        phases.append(fwd.phase_times())
    ctx.synchronize(sp)
    ph = [statistics.median(p[k] for p in phases) for k in range(4)]
    t = torch.tensor(ph, device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ph = [float(v) for v in t]
    remote = fwd.output_elements * 8 * (ws - 1) / ws
    # parity: y holds the forward transform of x0
    xin = torch.empty((ws * x0.numel(),), device="cuda")
    dist.all_gather_into_tensor(xin, x0)
    yall = torch.empty((ws * y.numel(),), device="cuda")
    dist.all_gather_into_tensor(yall, y)
    err = None
    if rank == 0:
        full = V.TransformIr.build(cfg, V.Direction.FORWARD, dev)
        yref = torch.empty_like(xin)
        ctx.execute_resident(full, xin.data_ptr(), yref.data_ptr(), stream=sp)
        ctx.synchronize(sp)
        # [P, D0, D1/P, D2, 2] -> [D0, P, D1/P, D2, 2]
        yslab = yall.view(ws, D, D // ws, D, 2).permute(1, 0, 2, 3, 4).reshape(-1)
        err = float(torch.linalg.vector_norm((yslab - yref).double()) / torch.linalg.vector_norm(yref.double()))
        del yref, yslab
    del xin, yall
    fwd.destroy()
    inv.destroy()
    out.update({
        "ms_per_step": ms, "gflops": flop / (ms * 1e-3) / 1e9, "parallelism": f"slab x{ws}",
        "forward_phases_ms": {"local_passes": ph[0], "exchange_pass": ph[1], "barrier": ph[2], "after_exchange": ph[3]},
        "nvlink": {"bytes_per_gpu_per_direction": remote, "exchange_pass_gbs": remote / (ph[1] * 1e-3) / 1e9,
                   "whole_forward_gbs": remote / (sum(ph) * 1e-3) / 1e9, "peak_gbs": 770.0,
                   "peak_source": "measured peer copy of this pool (nominal 900)"},
        "parity": None if err is None else {"relL2_vs_single_gpu": err, "tol": 2e-6, "ok": err <= 2e-6},
    })
    return out


def conv_section(args, ctx, dev, stream, ws, rank, dist):
    """BASELINE config 5 (64 images 2048^2 f32, U[0,1], convolved with one sigma = 8
    Gaussian) sharded by image: 64/N images per rank, no collective on the data path.  A
    step is one convolution (R2C -> spectrum multiply -> normalised C2R) of the rank's
    images; GFLOP/s counts 2 x 2.5 n log2 n per image (n = 2048^2) for the whole job.
    Parity: one image of rank 0 against the CPU oracle."""
    import torch
    import vkfft_rs as V
    dims, total = [2048, 2048], 64
    n = dims[0] * dims[1]
    per = total // ws
    sp = stream.cuda_stream
    cfg = (V.FftConfig(dims).with_transform(V.TransformKind.R2C).with_convolution(True)
           .with_coordinate_features(per))
    spec = gaussian_spectrum(dims)
    conv = V.NdRealConvolutionIr.build_from_spectrum(cfg, spec, dev)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4 + rank)
    x = torch.rand((per * n,), device="cuda", generator=gen)
    y = torch.empty_like(x)
    wsb = torch.empty((max(conv.workspace_bytes, 1),), dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ms = timed_steps(args.steps, args.warmup, stream,
                     [lambda: ctx.execute_nd_real_convolution_resident(conv, x.data_ptr(), y.data_ptr(),
                                                                       wsb.data_ptr(), sp)], dist)
    ctx.synchronize(sp)
    err = None
    if rank == 0:
        import oracle
        xi = x[:n].double().cpu().numpy().reshape(dims)
        ref = oracle.convolve_nd(xi, spec, dims, 1)
        yi = y[:n].double().cpu().numpy().reshape(dims)
        err = float(np.linalg.norm(yi - ref) / np.linalg.norm(ref))
    flop = total * 2 * 2.5 * n * math.log2(n)
    return {"workload": "BASELINE config 5: 64 images 2048^2 f32 convolved with a sigma=8 Gaussian",
            "images_per_rank": per, "parallelism": f"images sharded x{ws}", "scaling": "strong (64 images in total)",
            "ms_per_step": ms, "gflops": flop / (ms * 1e-3) / 1e9,
            "parity": None if err is None else {"relL2_image0": err, "tol": 2e-6, "ok": err <= 2e-6}}


# The reference's published pair-latency matrix (docs/PORTING_PLAN.md:281, RTX 4090, CUDA,
# examples/native_benchmark.rs defaults: batch 64, 20 timed pairs after 3 warm-up pairs,
# host-inclusive: each pair uploads the input, runs the forward and the normalised
# inverse transform and downloads the result).  The N4089 rows plan with the portable
# tuning on a device profile whose shared memory is cut to 32 / 16 KiB (the p29-FFT
# witnesses, native_benchmark.rs:733-757).
PUBLISHED_PAIRS = [
    dict(n=4096, batch=64, ms=0.339), dict(n=103, batch=64, ms=0.657), dict(n=257, batch=64, ms=0.306),
    dict(n=5760, batch=64, ms=0.507), dict(n=8192, batch=64, ms=0.572),
    dict(n=4089, batch=64, ms=0.454, shared=32 * 1024), dict(n=4089, batch=64, ms=0.548, shared=16 * 1024),
    dict(n=524288, batch=8, ms=99.107),
]


def run_published_pairs(args):
    """bench.py --workload published-pairs: the reference's published cases, timed the way
    its benchmark times them (host-inclusive forward + normalised inverse pairs through the
    host API, wall clock) and device-resident (CUDA events), with the round-trip error."""
    import torch
    import vkfft_rs as V
    ws, rank, local = dist_env()
    if rank != 0:
        return 0
    torch.cuda.set_device(local)
    ctx = V.CudaExecutionContext(local)
    dev = ctx.device_profile()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    iters = args.steps
    rows = []
    for case in PUBLISHED_PAIRS:
        n, batch = case["n"], case["batch"]
        d = dev
        cfg = V.FftConfig([n]).with_batch_count(batch)
        if case.get("shared"):
            d = dev.replace(shared_memory_bytes=case["shared"], shared_memory_pow2_bytes=case["shared"])
            cfg = cfg.with_tuning(V.PlannerTuning.portable())
        fwd = V.TransformIr.build(cfg, V.Direction.FORWARD, d)
        inv = V.TransformIr.build(cfg.with_inverse_normalization(True), V.Direction.INVERSE, d)
        idx = np.arange(n * batch, dtype=np.float32)
        x = (np.sin(np.float32(0.0031) * idx) + idx * np.float32(1e-7)
             + 1j * np.cos(np.float32(0.0023) * idx)).astype(np.complex64)
        mid = np.empty_like(x)
        back = np.empty_like(x)
        for _ in range(max(args.warmup, 3)):
            ctx.execute_transform(fwd, x, out=mid)
            ctx.execute_transform(inv, mid, out=back)
        t0 = time.perf_counter()
        for _ in range(iters):
            ctx.execute_transform(fwd, x, out=mid)
            ctx.execute_transform(inv, mid, out=back)
        host_ms = (time.perf_counter() - t0) / iters * 1e3
        err = float(np.linalg.norm(back.astype(np.complex128) - x) / np.linalg.norm(x.astype(np.complex128)))
        xd = torch.from_numpy(x.view(np.float32)).cuda()
        yd = torch.empty_like(xd)
        zd = torch.empty_like(xd)
        wsb = torch.empty((max(fwd.workspace_bytes, inv.workspace_bytes, 1),), dtype=torch.uint8, device="cuda")
        torch.cuda.synchronize()
        res_ms = timed_steps(iters, args.warmup, stream,
                             [lambda: ctx.execute_resident(fwd, xd.data_ptr(), yd.data_ptr(), wsb.data_ptr(), sp),
                              lambda: ctx.execute_resident(inv, yd.data_ptr(), zd.data_ptr(), wsb.data_ptr(), sp)],
                             None)
        ctx.synchronize(sp)
        kinds = [fwd.axis_child(0).kind.name]
        rows.append({"n": n, "batch": batch, "shared_bytes": case.get("shared"), "algorithm": kinds[0],
                     "host_pair_ms": host_ms, "resident_pair_ms": res_ms, "reference_rtx4090_host_pair_ms": case["ms"],
                     "host_speedup_vs_published": case["ms"] / host_ms, "round_trip_rel_l2": err,
                     "launches_per_pair": fwd.launch_count + inv.launch_count})
    line = {"metric": "forward + normalised inverse pair latency, the reference's published matrix",
            "value": statistics.mean(r["host_speedup_vs_published"] for r in rows), "unit": "x (geomean-free mean speed-up)",
            "n_gpus": 1, "steps": iters, "warmup": args.warmup, "higher_is_better": True,
            "vs_baseline": None, "dtype": "f32", "data": "the reference benchmark's deterministic input",
            "config": {"workload": "published-pairs (docs/PORTING_PLAN.md:281; examples/native_benchmark.rs)",
                       "timing": "host-inclusive: wall clock over the timed pairs through execute_transform "
                                 "(pageable host arrays); resident: CUDA events",
                       "reference_hardware": "RTX 4090 (CUDA), the reference's own figures"},
            "cases": rows}
    print(json.dumps(line))
    ctx.close()
    return 0


def run_ours(args):
    import torch
    import vkfft_rs as V
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = V.CudaExecutionContext(local)
    dev = ctx.device_profile()
    cfg = V.FftConfig([N]).with_batch_count(BATCH).with_inverse_normalization(True)
    fwd = V.TransformIr.build(cfg, V.Direction.FORWARD, dev)
    inv = V.TransformIr.build(cfg, V.Direction.INVERSE, dev)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1 + rank)
    a = (torch.rand((BATCH, N, 2), device="cuda", generator=gen) * 2 - 1).contiguous()
    b = torch.empty_like(a)
    torch.cuda.synchronize()  # the inputs were generated on the default stream
    # a dedicated (non-default) stream: the kernels and the timing events share it
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream

    def step():
        ctx.execute_resident(fwd, a.data_ptr(), b.data_ptr(), stream=sp)
        ctx.execute_resident(inv, b.data_ptr(), a.data_ptr(), stream=sp)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # per-launch timing of the dominant kernel (forward pass) on the same stream
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        clk.mark_start()
        ev0.record(stream)
        for k in range(args.steps):
            evs[k][0].record(stream)
            ctx.execute_resident(fwd, a.data_ptr(), b.data_ptr(), stream=sp)
            evs[k][1].record(stream)
            ctx.execute_resident(inv, b.data_ptr(), a.data_ptr(), stream=sp)
        ev1.record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    ctx.synchronize(sp)  # raises if a kernel recorded an error
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    elapsed_ms = ev0.elapsed_time(ev1)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    rank_ms = [elapsed_ms / args.steps]
    if dist:
        t = torch.tensor([elapsed_ms, fwd_ms], device="cuda", dtype=torch.float64)
        every = [torch.zeros_like(t) for _ in range(ws)]
        dist.all_gather(every, t)
        rank_ms = [float(v[0]) / args.steps for v in every]
        elapsed_ms = max(float(v[0]) for v in every)
        fwd_ms = max(float(v[1]) for v in every)
    ms_per_step = elapsed_ms / args.steps
    total_transforms = 2 * BATCH * ws
    value = total_transforms * FLOP_PER_TRANSFORM / (ms_per_step * 1e-3) / 1e9
    parity = headline_parity(ctx, fwd, a, b, sp, rank, dist)

    if args.skip_e2e:
        e2e_value = None
    # e2e through the host API with pinned host arrays
    def pinned():
        t = torch.empty((BATCH * N * 2,), dtype=torch.float32, pin_memory=True)
        return t, t.numpy().view(np.complex64)

    if not args.skip_e2e:
        host_in_t, x_host = pinned()
        host_spec_t, spec = pinned()
        host_back_t, back = pinned()
        host_in_t.copy_(a.reshape(-1).cpu())
        e2e_steps = max(1, min(args.steps, 10))  # host-side timing: enough steps to average PCIe noise
        ctx.execute_transform(fwd, x_host, out=spec)  # warm the staging buffers
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            ctx.execute_transform(fwd, x_host, out=spec)
            ctx.execute_transform(inv, spec, out=back)
        e2e_s = (time.perf_counter() - t0) / e2e_steps
        if dist:
            t = torch.tensor([e2e_s], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t[0])
        e2e_value = total_transforms * FLOP_PER_TRANSFORM / e2e_s / 1e9
    bytes_one = BATCH * N * 8
    if not args.skip_e2e:
        del host_in_t, host_spec_t, host_back_t, x_host, spec, back
    del a, b
    torch.cuda.empty_cache()
    sections = {}
    if not args.headline_only:
        sections["slab_512^3"] = slab_section(args, ctx, dev, stream, ws, rank, dist)
        torch.cuda.empty_cache()
        sections["conv_2048_sharded"] = conv_section(args, ctx, dev, stream, ws, rank, dist)
        torch.cuda.empty_cache()

    peak, peak_kind = load_peaks()
    box_copy = live_copy_gbs(stream)
    alg_bytes = 2 * N * BATCH * 8  # one read + one write of the tensor per launch
    achieved = alg_bytes / (fwd_ms * 1e-3) / 1e9
    traffic = load_traffic()
    line = {
        "metric": METRIC, "value": value, "unit": "GFLOP/s", "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (uniform [-1,1], torch generator seed 1+rank)",
        "config": headline_config(ws),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_source": peak_kind, "this_gpu_copy_gbs": box_copy,
                     "kernel": "reg_fft_persistent<float,4096> (register-resident Stockham with bulk-copy prefetch, one launch per transform direction)"},
        "e2e": None if e2e_value is None else {"value": e2e_value, "unit": "GFLOP/s", "h2d_bytes_per_step": 2 * bytes_one,
                "d2h_bytes_per_step": 2 * bytes_one, "path": "execute_transform (host arrays, pinned)"},
        "gpu_launches": args.steps * (fwd.launch_count + inv.launch_count),
        "clocks": clk.summary(),
        "rank_ms_per_step": rank_ms,
        "parity": parity,
    }
    line.update(sections)
    if rank == 0:
        line["cpu_baseline"] = cpu_baseline(1, budget_s=12.0) if (ws == 1 and not args.skip_cpu) else None
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return 0


# The other BASELINE configs (config 1, config 2 real, 3, 4, 5) as single-GPU measurement
# lines: `python bench.py --workload <name>`.  A step is one forward + one normalised
# inverse transform over the whole workload (one convolution for "conv-2048").  GFLOP/s
# counts 5 N log2 N per complex transform and 2.5 N log2 N per real one (N = product of
# the dims); the roofline fraction is the logical bytes (one read + one write of the
# tensors per direction) over the measured time of the whole transform, so extra passes
# and scratch round trips show up as a lower fraction.
REC_TUNING = dict(min_rader_direct_prime=17, max_rader_direct_prime=89, min_rader_fft_prime=17,
                  max_rader_fft_prime=16384, allow_recursive_fft_rader=True)
WORKLOADS = {
    "c2c-1024x8": dict(kind="c2c", dims=[1024], batch=8, prec="F32", config=1),
    "r2c-4096": dict(kind="r2c", dims=[4096], batch=65536, prec="F32", config=2),
    "c2c-512^3": dict(kind="c2c", dims=[512, 512, 512], batch=1, prec="F32", config=3, slab=True),
    "r2c-1024^3": dict(kind="r2c", dims=[1024, 1024, 1024], batch=1, prec="F32", config=3, slab=True),
    "c2c-1024x17x65537-f32": dict(kind="c2c", dims=[1024, 17, 65537], batch=1, prec="F32", config=4),
    "c2c-1024x17x65537-f64": dict(kind="c2c", dims=[1024, 17, 65537], batch=1, prec="F64", config=4),
    "c2c-4099-f32": dict(kind="c2c", dims=[4099], batch=16384, prec="F32", config=4),
    "c2c-4099-f64": dict(kind="c2c", dims=[4099], batch=16384, prec="F64", config=4),
    "c2c-4099-rader-f32": dict(kind="c2c", dims=[4099], batch=16384, prec="F32", config=4, tuning=REC_TUNING),
    "c2c-4099-rader-f64": dict(kind="c2c", dims=[4099], batch=16384, prec="F64", config=4, tuning=REC_TUNING),
    "c2c-65537-f32": dict(kind="c2c", dims=[65537], batch=2048, prec="F32", config=4),
    "c2c-65537-f64": dict(kind="c2c", dims=[65537], batch=2048, prec="F64", config=4),
    "conv-2048": dict(kind="conv", dims=[2048, 2048], batch=64, prec="F32", config=5),
    # config-4 shape family at 1/16 of the outer axis (570 MB, profiling the 17-point Rader
    # line kernel and the Bluestein passes of 65537 on a small case)
    "c2c-64x17x65537-f32": dict(kind="c2c", dims=[64, 17, 65537], batch=1, prec="F32", config=4),
    # small 2D case (512 MB): one contiguous and one strided 1024-point axis (profiling)
    "c2c-1024^2x64": dict(kind="c2c", dims=[1024, 1024], batch=64, prec="F32", config=3),
    # DCT / DST (not a headline config): forward DCT-II + normalised inverse (DCT-III)
    "dct2-4096-f32": dict(kind="r2r", r2r="DCT2", dims=[4096], batch=16384, prec="F32", config=0),
    "dct2-4096-f64": dict(kind="r2r", r2r="DCT2", dims=[4096], batch=8192, prec="F64", config=0),
    "dct4-4096-f32": dict(kind="r2r", r2r="DCT4", dims=[4096], batch=16384, prec="F32", config=0),
    "dct2-512^2-f32": dict(kind="r2r", r2r="DCT2", dims=[512, 512], batch=256, prec="F32", config=0),
    # double-double (not a headline config): C2C forward + normalised inverse
    "c2c-4096-dd": dict(kind="c2c", dims=[4096], batch=2048, prec="DOUBLE_DOUBLE", config=0),
    "c2c-1000-dd": dict(kind="c2c", dims=[1000], batch=8192, prec="DOUBLE_DOUBLE", config=0),
    # the reference's own published large case (N=524288 x batch 8 forward + inverse pair,
    # resident buffers: 7.319 ms on an RTX 4090); 32 MiB of data sits inside L2, so L2 is
    # flushed before every timed launch
    "c2c-524288x8": dict(kind="c2c", dims=[524288], batch=8, prec="F32", config=0, flush_l2=True,
                         label="reference-published pair", published_ms=7.319),
}


def gaussian_spectrum(dims, sigma=8.0):
    """R2C spectrum of a centred Gaussian (sum 1), circularly shifted to the origin (input
    preparation, untimed)."""
    h, w = dims
    yy = np.minimum(np.arange(h), h - np.arange(h))[:, None].astype(np.float64)
    xx = np.minimum(np.arange(w), w - np.arange(w))[None, :].astype(np.float64)
    g = np.exp(-(yy * yy + xx * xx) / (2 * sigma * sigma))
    g /= g.sum()
    return np.fft.rfft2(g).astype(np.complex64)


def run_slab_workload(args, wl, ctx, dev, dist, ws, rank, local):
    """3D config under torchrun: one slab-decomposed transform over all ranks (strong
    scaling).  The exchange runs inside the library (peer stores + device barrier)."""
    import torch
    import vkfft_rs as V
    kind, dims = wl["kind"], wl["dims"]
    n = int(np.prod(dims))
    cfg = V.FftConfig(dims).with_precision(V.Precision[wl["prec"]]).with_inverse_normalization(True)
    real = kind == "r2c"
    fwd = V.SlabTransform.build(cfg.with_transform(V.TransformKind.R2C) if real else cfg, V.Direction.FORWARD,
                                ws, rank, dev)
    inv = V.SlabTransform.build(cfg.with_transform(V.TransformKind.C2R) if real else cfg, V.Direction.INVERSE,
                                ws, rank, dev)
    fwd.setup(ctx)
    inv.setup(ctx)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(wl["config"] + rank)
    in_scalars = fwd.input_elements * (1 if real else 2)
    a = torch.rand((in_scalars,), device="cuda", generator=gen) * 2 - 1
    b = torch.empty((fwd.output_elements * 2,), device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    launches = [lambda: ctx.execute_slab(fwd, a.data_ptr(), b.data_ptr(), stream=sp),
                lambda: ctx.execute_slab(inv, b.data_ptr(), a.data_ptr(), stream=sp)]
    for _ in range(max(args.warmup, 3)):
        for f in launches:
            f()
    ctx.synchronize(sp)
    dist.barrier()
    torch.cuda.synchronize()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in launches]
           for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        clk.mark_start()
        for k in range(args.steps):
            for j, f in enumerate(launches):
                evs[k][j][0].record(stream)
                f()
                evs[k][j][1].record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    ctx.synchronize(sp)
    part_ms = [statistics.mean(evs[k][j][0].elapsed_time(evs[k][j][1]) for k in range(args.steps))
               for j in range(len(launches))]
    t = torch.tensor([sum(part_ms)] + part_ms, device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, part_ms = float(t[0]), [float(v) for v in t[1:]]
    flop = 2 * (2.5 if real else 5.0) * n * math.log2(n)
    value = flop / (ms * 1e-3) / 1e9
    peak, peak_kind = load_peaks()
    cplx_local = fwd.output_elements * 8
    in_local = fwd.input_elements * (4 if real else 8)
    achieved = (in_local + cplx_local) / (part_ms[0] * 1e-3) / 1e9
    nvlink_bytes = cplx_local * (ws - 1) / ws  # leaves this GPU per direction
    line = {
        "metric": f"{args.workload} GFLOP/s (5N*log2N complex, 2.5N*log2N real), slab over {ws} GPUs",
        "value": value, "unit": "GFLOP/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": wl["prec"].lower(), "data": "synthetic (torch generator)",
        "config": {"workload": f"BASELINE config {wl['config']}: {kind} {dims}, slab decomposition",
                   "parallelism": f"slab x{ws} (exchange fused into the last local FFT pass)"},
        "parts_ms": part_ms,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": peak_kind,
                     "basis": "per-rank logical bytes of the forward transform / its time"},
        "nvlink": {"bytes_per_direction_per_gpu": nvlink_bytes,
                   "achieved_gbs": nvlink_bytes / (part_ms[0] * 1e-3) / 1e9, "peak_gbs": 770.0},
        "gpu_launches": args.steps * (fwd.launch_count + inv.launch_count),
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line))
    fwd.destroy()
    inv.destroy()
    dist.barrier()
    dist.destroy_process_group()
    ctx.close()
    return 0


def run_workload(args):
    import torch
    import vkfft_rs as V
    wl = WORKLOADS[args.workload]
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dist = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    ctx = V.CudaExecutionContext(local)
    dev = ctx.device_profile()
    kind, dims, batch, prec = wl["kind"], wl["dims"], wl["batch"], wl["prec"]
    if ws > 1 and wl.get("slab"):
        return run_slab_workload(args, wl, ctx, dev, dist, ws, rank, local)
    dbl = prec in ("F64", "DOUBLE_DOUBLE")
    tdt = torch.float64 if dbl else torch.float32
    words = 2 if prec == "DOUBLE_DOUBLE" else 1  # float64 words per real value
    rsz = (8 if dbl else 4) * words
    n = int(np.prod(dims))
    half = int(np.prod(dims[:-1])) * (dims[-1] // 2 + 1)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(wl["config"] + rank)
    if kind == "conv":
        cfg = (V.FftConfig(dims).with_transform(V.TransformKind.R2C).with_convolution(True)
               .with_coordinate_features(batch))
        conv = V.NdRealConvolutionIr.build_from_spectrum(cfg, gaussian_spectrum(dims), dev)
        a = torch.rand((batch * n,), device="cuda", generator=gen, dtype=tdt)
        b = torch.empty_like(a)
        wsb = torch.empty((max(conv.workspace_bytes, 1),), dtype=torch.uint8, device="cuda")
        launches = [lambda sp: ctx.execute_nd_real_convolution_resident(conv, a.data_ptr(), b.data_ptr(),
                                                                        wsb.data_ptr(), sp)]
        flop = 2 * 2.5 * n * math.log2(n) * batch
        alg_bytes = [2 * batch * n * rsz + half * 2 * rsz]
        n_launch = None
    else:
        cfg = V.FftConfig(dims).with_batch_count(batch).with_precision(V.Precision[prec])
        cfg = cfg.with_inverse_normalization(True)
        if wl.get("tuning"):
            cfg = cfg.with_tuning(V.PlannerTuning(**wl["tuning"]))
        if kind == "c2c":
            fwd = V.TransformIr.build(cfg, V.Direction.FORWARD, dev)
            inv = V.TransformIr.build(cfg, V.Direction.INVERSE, dev)
            a = torch.rand((batch * n * 2 * words,), device="cuda", generator=gen, dtype=tdt) * 2 - 1
            if words == 2:  # double-double words: a small canonical low word under each high word
                a.view(-1, 2)[:, 1] *= 2.0 ** -60
            b = torch.empty_like(a)
            flop = 2 * 5.0 * n * math.log2(n) * batch
            alg_bytes = [2 * batch * n * 2 * rsz] * 2
        elif kind == "r2r":
            rc = cfg.with_transform(V.TransformKind[wl["r2r"]])
            fwd = V.TransformIr.build(rc, V.Direction.FORWARD, dev)
            inv = V.TransformIr.build(rc, V.Direction.INVERSE, dev)
            a = torch.rand((batch * n,), device="cuda", generator=gen, dtype=tdt) * 2 - 1
            b = torch.empty_like(a)
            flop = 2 * 2.5 * n * math.log2(n) * batch
            alg_bytes = [2 * batch * n * rsz] * 2
        else:
            fwd = V.TransformIr.build(cfg.with_transform(V.TransformKind.R2C), V.Direction.FORWARD, dev)
            inv = V.TransformIr.build(cfg.with_transform(V.TransformKind.C2R), V.Direction.INVERSE, dev)
            a = torch.rand((batch * n,), device="cuda", generator=gen, dtype=tdt) * 2 - 1
            b = torch.empty((batch * half * 2,), device="cuda", dtype=tdt)
            flop = 2 * 2.5 * n * math.log2(n) * batch
            alg_bytes = [batch * (n * rsz + half * 2 * rsz)] * 2
        wsb = torch.empty((max(fwd.workspace_bytes, inv.workspace_bytes, 1),), dtype=torch.uint8, device="cuda")
        launches = [lambda sp: ctx.execute_resident(fwd, a.data_ptr(), b.data_ptr(), wsb.data_ptr(), sp),
                    lambda sp: ctx.execute_resident(inv, b.data_ptr(), a.data_ptr(), wsb.data_ptr(), sp)]
        n_launch = fwd.launch_count + inv.launch_count
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sp = stream.cuda_stream
    # a 256 MiB write (twice the 126 MB L2) before each timed launch when the workload
    # itself would stay L2-resident
    flush = torch.empty((64 << 20,), device="cuda", dtype=torch.float32) if wl.get("flush_l2") else None
    for _ in range(max(args.warmup, 3)):
        for f in launches:
            f(sp)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in launches]
           for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        clk.mark_start()
        for k in range(args.steps):
            for j, f in enumerate(launches):
                if flush is not None:
                    flush.fill_(float(k + j))
                evs[k][j][0].record(stream)
                f(sp)
                evs[k][j][1].record(stream)
        torch.cuda.synchronize()
        clk.mark_end()
    part_ms = [statistics.mean(evs[k][j][0].elapsed_time(evs[k][j][1]) for k in range(args.steps))
               for j in range(len(launches))]
    ms = sum(part_ms)
    if dist:
        t = torch.tensor([ms] + part_ms, device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, part_ms = float(t[0]), [float(v) for v in t[1:]]
    peak, peak_kind = load_peaks()
    achieved = [alg_bytes[j] / (part_ms[j] * 1e-3) / 1e9 for j in range(len(launches))]
    value = flop * ws / (ms * 1e-3) / 1e9
    vs = None
    if wl.get("published_ms"):  # value / the reference's published figure for this workload
        vs = value / (flop / (wl["published_ms"] * 1e-3) / 1e9)
    line = {
        "metric": f"{args.workload} GFLOP/s (5N*log2N complex, 2.5N*log2N real and DCT/DST)", "value": value, "unit": "GFLOP/s",
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": vs, "dtype": "dd" if words == 2 else prec.lower(), "data": "synthetic (torch generator)",
        "config": {"workload": (f"BASELINE config {wl['config']}: " if wl["config"]
                                else f"{wl.get('label') or wl.get('r2r') or wl['prec'].lower()} ")
                               + f"{kind} {dims} x batch {batch}"
                               + (" recursive Rader tuning" if wl.get("tuning") else ""),
                   "global_batch": batch * ws, "parallelism": f"replicas x{ws}" if ws > 1 else "1 GPU",
                   "l2": ("flushed (256 MiB write) before each timed launch" if flush is not None
                          else "inputs larger than L2; no flush" if alg_bytes[0] / 2 > 126e6
                          else "L2-resident, no flush (launch-bound case)")},
        "parts_ms": part_ms,
        "roofline": {"bound": "hbm", "achieved": achieved[0], "peak": peak, "unit": "GB/s",
                     "frac": achieved[0] / peak, "frac_parts": [x / peak for x in achieved], "traffic": None,
                     "peak_source": peak_kind, "basis": "logical bytes of the whole transform / its time"},
        "gpu_launches": None if n_launch is None else args.steps * n_launch,
        "clocks": clk.summary(),
    }
    if rank == 0:
        print(json.dumps(line))
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    ctx.close()
    return 0


def main():
    global BATCH
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # default: ~0.45 s of timed work on config 2, long enough for several clock samples
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=BATCH, help="transforms per rank (profiling runs use fewer)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling runs: resident timing only")
    ap.add_argument("--skip-cpu", action="store_true", help="profiling runs: no CPU baseline")
    ap.add_argument("--headline-only", action="store_true",
                    help="profiling runs: no config-3 slab / config-5 sharded sections")
    ap.add_argument("--workload", default="c2c-4096", choices=["c2c-4096", "published-pairs"] + sorted(WORKLOADS),
                    help="c2c-4096 is the headline (config 2); the others measure the remaining configs")
    args = ap.parse_args()
    BATCH = args.batch
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "published-pairs":
        return run_published_pairs(args)
    if args.workload != "c2c-4096":
        return run_workload(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
