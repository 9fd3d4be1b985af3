"""Host-side checks of the C-ABI library: it loads, exports every entry point
include/b200fft.h declares, lowers the BASELINE configurations into launch programs,
and fails closed without a GPU.  No kernel is launched here."""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_library_exports_every_declared_symbol(V):
    lib = V.library()
    declared = V.exported_symbols()
    assert len(declared) >= 40
    missing = [name for name in declared if not hasattr(lib, name)]
    assert missing == []
    assert lib.b200fft_abi_version() == 1


def test_nm_lists_the_c_symbols():
    so = os.path.join(ROOT, "vkfft-rs_b200", "libb200fft.so")
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    for name in ("b200fft_execute", "b200fft_execute_host", "b200fft_transform_build", "b200fft_plan_build"):
        assert f" T {name}" in out


def test_baseline_programs_lower(V, cuda_profile):
    # (config, launches f32, launches f64): f64 Bluestein M=8232 exceeds one CTA's
    # shared memory and runs as three passes through scratch
    cases = [
        (V.FftConfig([1024]).with_batch_count(8), 1, 1),
        (V.FftConfig([4096]).with_batch_count(65536), 1, 1),
        (V.FftConfig([512, 512, 512]), 3, 3),
        (V.FftConfig([4099]).with_batch_count(16384), 1, 3),
        (V.FftConfig([65537]).with_batch_count(2048), 3, 3),
        (V.FftConfig([1024, 17, 65537]), 5, 5),
    ]
    for cfg, l32, l64 in cases:
        for prec, launches in ((V.Precision.F32, l32), (V.Precision.F64, l64)):
            ir = V.TransformIr.build(cfg.with_precision(prec), V.Direction.FORWARD, cuda_profile)
            assert ir.launch_count == launches
            assert (ir.workspace_bytes > 0) == (launches > 1 and cfg.dimensions[-1] != 512)
    r2c = V.FftConfig([4096]).with_batch_count(65536).with_transform(V.TransformKind.R2C)
    ir = V.TransformIr.build(r2c, V.Direction.FORWARD, cuda_profile)
    assert ir.input_is_real and not ir.output_is_real
    assert ir.input_elements == 4096 * 65536 and ir.output_elements == 2049 * 65536
    c2r = V.FftConfig([1024, 1024, 1024]).with_transform(V.TransformKind.C2R).with_inverse_normalization(True)
    ir = V.TransformIr.build(c2r, V.Direction.INVERSE, cuda_profile)
    assert ir.output_is_real and ir.launch_count == 3


def test_double_double_builds_and_convolution_fails_closed(V, cuda_profile):
    """Double-double transforms build for every family (C2C, R2C, C2R, R2R; 1D and ND);
    convolution stays rejected by FftConfig::validate as in the reference ("performConvolution
    currently requires ordinary or mixed F16/F32/F64 storage")."""
    for prec in (V.Precision.DOUBLE_DOUBLE, V.Precision.DOUBLE_DOUBLE_F64_STORAGE):
        for kind, d in ((V.TransformKind.C2C, V.Direction.FORWARD), (V.TransformKind.R2C, V.Direction.FORWARD),
                        (V.TransformKind.C2R, V.Direction.INVERSE), (V.TransformKind.DCT2, V.Direction.INVERSE)):
            for dims in ([64], [12, 34]):
                ir = V.TransformIr.build(V.FftConfig(dims).with_precision(prec).with_transform(kind), d, cuda_profile)
                assert ir.launch_count >= 1
    cfg = (V.FftConfig([32, 48]).with_transform(V.TransformKind.R2C).with_precision(V.Precision.DOUBLE_DOUBLE)
           .with_convolution(True))
    with pytest.raises(V.VkFftError) as e:
        V.NdRealConvolutionIr.build_from_spectrum(cfg, np.zeros(32 * 25, dtype=np.complex128), cuda_profile)
    assert e.value.variant == "UnsupportedKernelPath" and "F16/F32/F64 storage" in str(e.value)


def test_probe_without_gpu_reports_native_unavailable(V):
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(V.VkFftError) as e:
        V.probe()
    assert e.value.variant == "NativeUnavailable"
    with pytest.raises(V.VkFftError) as e:
        V.CudaExecutionContext(0)
    assert e.value.variant == "NativeUnavailable"


def test_codelets_match_naive_dft(tmp_path):
    """The generated butterflies (dft_codelets.cuh) are host-callable: compile them with
    g++ and compare each radix with a naive DFT."""
    src = tmp_path / "codelets.cpp"
    src.write_text(r'''
#include <cstdio>
#include <cmath>
#include <complex>
#include "dft_codelets.cuh"
template<int R> double check() {
  cplx<double> v[R]; std::complex<double> x[R];
  for (int i=0;i<R;i++){ x[i]={std::sin(1.3*i+0.2), std::cos(0.7*i*i+0.1)}; v[i]={x[i].real(), x[i].imag()}; }
  dft<R,double>(v);
  double err=0;
  for (int k=0;k<R;k++){ std::complex<double> s=0; for(int n=0;n<R;n++) s+=x[n]*std::polar(1.0,-2*M_PI*n*k/R);
    err=std::max(err, std::abs(s-std::complex<double>(v[k].x,v[k].y))); }
  return err;
}
int main(){
  double e[] = {check<2>(),check<3>(),check<4>(),check<5>(),check<6>(),check<7>(),check<8>(),check<9>(),
                check<10>(),check<11>(),check<12>(),check<13>(),check<14>(),check<15>(),check<16>(),check<32>()};
  double m = 0; for (double v : e) m = v > m ? v : m;
  printf("%.3e\n", m);
}
''')
    exe = tmp_path / "codelets"
    inc = os.path.join(ROOT, "vkfft-rs_b200", "csrc")
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", inc, str(src), "-o", str(exe)], check=True)
    err = float(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert err < 1e-12


def test_fault_injection_env_is_host_side(V):
    """B200FFT_FAULT only affects host-side allocation / launch calls; planning is untouched."""
    env = dict(os.environ, B200FFT_FAULT="alloc:1")
    code = ("import sys; sys.path.insert(0, %r); import vkfft_rs as V; "
            "d = V.DeviceProfile.generic(V.Backend.CUDA, V.GpuVendor.NVIDIA); "
            "V.TransformIr.build(V.FftConfig([64]), V.Direction.FORWARD, d); print('ok')"
            % os.path.join(ROOT, "vkfft-rs_b200"))
    out = subprocess.run(["python", "-c", code], env=env, capture_output=True, text=True, check=True).stdout
    assert out.strip() == "ok"
