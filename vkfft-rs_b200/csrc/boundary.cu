// Convolution multiply kernel (one thread per output element) and boundary copy kernel,
// which gathers a caller's (formatted, zero-padded) input into a dense
// scratch tensor, or scatters a dense result into the caller's formatted output with the
// zero-padding interval applied.  One thread per logical element, grid-stride.
#include <cuda_runtime.h>

#include <algorithm>

#include "boundary_device.cuh"

namespace b200fft {

__global__ void __launch_bounds__(256) boundary_copy_kernel(const __grid_constant__ BoundaryCopy b) {
    for (int64_t L = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; L < b.total; L += (int64_t)gridDim.x * blockDim.x)
        boundary_copy_one(b, L);
}

template <typename T>
__global__ void __launch_bounds__(256) conv_multiply_kernel(const __grid_constant__ ConvMultiply m) {
    for (int64_t L = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; L < m.total; L += (int64_t)gridDim.x * blockDim.x)
        conv_multiply_one<T>(m, L);
}

// kind: Program::scalar_kind (0 f32, 1 f64, 2 double-double)
cudaError_t launch_conv_multiply(const ConvMultiply &m, int kind, cudaStream_t stream) {
    if (m.total <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((m.total + 255) / 256, 148 * 32);
    if (kind == 2)
        conv_multiply_kernel<dd><<<(unsigned)blocks, 256, 0, stream>>>(m);
    else if (kind == 1)
        conv_multiply_kernel<double><<<(unsigned)blocks, 256, 0, stream>>>(m);
    else
        conv_multiply_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(m);
    return cudaGetLastError();
}

template <typename T>
__global__ void __launch_bounds__(256) r2r_kernel(const __grid_constant__ R2rPass r) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < r.total; t += (int64_t)gridDim.x * blockDim.x)
        r2r_one<T>(r, t);
}

cudaError_t launch_r2r(const R2rPass &r, int kind, cudaStream_t stream) {
    if (r.total <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((r.total + 255) / 256, 148 * 32);
    if (kind == 2)
        r2r_kernel<dd><<<(unsigned)blocks, 256, 0, stream>>>(r);
    else if (kind == 1)
        r2r_kernel<double><<<(unsigned)blocks, 256, 0, stream>>>(r);
    else
        r2r_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(r);
    return cudaGetLastError();
}

cudaError_t launch_boundary_copy(const BoundaryCopy &b, cudaStream_t stream) {
    if (b.total <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((b.total + 255) / 256, 148 * 32);
    boundary_copy_kernel<<<(unsigned)blocks, 256, 0, stream>>>(b);
    return cudaGetLastError();
}

}  // namespace b200fft
