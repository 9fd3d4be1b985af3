// B200 (sm_100a) FFT pass kernel.
//
// One CTA owns G lines of a pass.  It stages them in shared memory, runs the
// pass's op program on them and writes them back.  Global traffic is one read
// and one write per element per pass, issued as warp-coalesced accesses:
// element-fastest for contiguous lines, line-fastest for strided lines (the
// strided-axis case: G neighbouring lines are neighbouring addresses).  Radix
// stages are Stockham steps between two shared-memory buffers: a thread takes a
// butterfly, gathers its R inputs, applies the twiddles and the unrolled
// butterfly codelet and writes the R outputs to their autosorted positions in
// the other buffer.  Shared-memory indices are padded (one slot every 16
// elements, odd line strides) so the power-of-two strides of the stages do not
// collapse onto one bank.
//
// Inverse transforms run the forward network on conjugated data (the host
// program sets the conjugation flags), so every table holds forward roots only.
// Faults are never raised on the device: an unknown op or radix sets the pass's
// error word and is skipped uniformly by the whole CTA.
#ifndef B200FFT_EMULATE
#include <cuda_runtime.h>
#endif

#include "pass_device.cuh"

namespace b200fft {

#ifndef B200FFT_EMULATE
template <typename T, int MAXT>
__global__ void __launch_bounds__(MAXT) fft_pass_kernel(const __grid_constant__ PassParams p) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    cplx<T> *sm = reinterpret_cast<cplx<T> *>(smem_raw);
    const LineMeta lm = pass_prologue<T>(p, smem_raw);
    __syncthreads();
    for (int k = 0; k < p.nops; k++) {
        run_op<T>(p, p.ops[k], sm, lm);
        __syncthreads();
    }
}

// ---- host launch table ------------------------------------------------------

struct KernelVariant {
    int maxt;
    const void *fn;
};

// one variant per compute type (Program::scalar_kind): f32, f64, double-double
#define B200FFT_VARIANT(T, M) {M, (const void *)fft_pass_kernel<T, M>}
static const KernelVariant kVariants[] = {
    B200FFT_VARIANT(float, 1024),
    B200FFT_VARIANT(double, 512),
    B200FFT_VARIANT(dd, 256),
};
#undef B200FFT_VARIANT

int kernel_variant_for(int scalar_kind) { return scalar_kind; }
int kernel_variant_max_threads(int v) { return kVariants[v].maxt; }

// Opt every variant in to the full dynamic shared memory of an sm_100 CTA (227 KB).
// The attribute is per device, so it is set once for every device a context is made on.
void set_kernel_smem_limits() {
    static unsigned long long done_mask = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
    if (done_mask & (1ull << dev)) return;
    for (const KernelVariant &v : kVariants)
        cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    done_mask |= 1ull << dev;
}

cudaError_t launch_pass(int variant, const PassParams &p, int64_t grid, int threads, size_t smem,
                        cudaStream_t stream) {
    const void *fn = kVariants[variant].fn;
    void *args[] = {const_cast<PassParams *>(&p)};
    return cudaLaunchKernel(fn, dim3((unsigned)grid), dim3(threads), args, smem, stream);
}

#endif  // B200FFT_EMULATE

}  // namespace b200fft
