// Register-resident Stockham kernel for batched contiguous power-of-two C2C lines
// (the BASELINE config 1/2 hot path).
//
// A line of N points is owned by TT = N / E threads, each holding E points in
// registers.  With the load pattern "thread t holds positions t + m*TT", the
// first radix stage's butterflies are formed entirely from the thread's own
// registers and the last stage's outputs land on positions t + m*TT again, so
// global memory is read and written once, warp-coalesced (32 consecutive
// threads touch 32 consecutive complex values), with no shared-memory staging.
// Only the middle stages exchange through one padded shared-memory buffer.
// Twiddles come from per-stage transposed tables read through the read-only cache.
// Inverse transforms conjugate on load and store (the table stays forward).
#include <cuda_runtime.h>

#include <cstdint>

#include "dft_codelets.cuh"
#include "reg_kernels.hpp"

namespace b200fft {

namespace regk {

template <typename T> struct vec2;
template <> struct vec2<float> { using type = float2; };
template <> struct vec2<double> { using type = double2; };

__device__ __forceinline__ int pad(int e) { return e + (e >> 4); }

template <typename T> __device__ __forceinline__ cplx<T> mul(cplx<T> a, cplx<T> b) {
    return {a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x};
}
template <typename T> __device__ __forceinline__ cplx<T> tw_load(const cplx<T> *tw, int idx) {
    auto v = __ldg(reinterpret_cast<const typename vec2<T>::type *>(tw) + idx);
    return {v.x, v.y};
}

struct LineIO {
    int64_t in_off, out_off;
    bool valid;
};

// One radix-R stage with span P (product of the radices before it).  Its twiddles
// W_{P R}^{j q} are read from the stage's transposed table (row q-1 holds the P values
// of j, so a warp's loads are contiguous) at offset OFF; only the power-of-two rows
// are read and w_q = w_{q - lowbit(q)} * w_{lowbit(q)} forms the rest (at most three
// products deep).
template <typename T, int N, int E, int R, int P, int OFF, bool FIRST, bool LAST>
__device__ __forceinline__ void stage(cplx<T> (&v)[E], int t, cplx<T> *sline, const cplx<T> *tw, const RegParams &rp,
                                      const LineIO &io) {
    constexpr int TT = N / E;
    constexpr int NB = E / R;  // butterflies per thread
    if (!FIRST) {
        __syncthreads();  // previous stage's outputs are visible
#pragma unroll
        for (int k = 0; k < NB; k++)
#pragma unroll
            for (int q = 0; q < R; q++) v[k + q * NB] = sline[pad(t + k * TT + q * (N / R))];
        if (!LAST) __syncthreads();  // every thread has read before anyone overwrites
    }
#pragma unroll
    for (int k = 0; k < NB; k++) {
        cplx<T> x[R];
#pragma unroll
        for (int q = 0; q < R; q++) x[q] = v[k + q * NB];
        const int b = t + k * TT;
        const int j = b % P;
        if (P > 1) {
            cplx<T> w[R];
#pragma unroll
            for (int q = 1; q < R; q++) {
                if ((q & (q - 1)) == 0) {
                    w[q] = tw_load(tw, OFF + (q - 1) * P + j);
                } else {
                    const int lb = q & (-q);
                    w[q] = mul(w[q - lb], w[lb]);
                }
            }
#pragma unroll
            for (int q = 1; q < R; q++) x[q] = mul(x[q], w[q]);
        }
        dft<R, T>(x);
        if (LAST) {
            if (io.valid) {
#pragma unroll
                for (int q = 0; q < R; q++) {
                    cplx<T> y = x[q];
                    y.x *= T(rp.scale);
                    y.y *= rp.conj ? -T(rp.scale) : T(rp.scale);
                    typename vec2<T>::type w;
                    w.x = y.x;
                    w.y = y.y;
                    __stcs(reinterpret_cast<typename vec2<T>::type *>(rp.out) + io.out_off + b + q * (N / R), w);
                }
            }
        } else {
            const int e0 = (b - j) * R + j;
#pragma unroll
            for (int q = 0; q < R; q++) sline[pad(e0 + q * P)] = x[q];
        }
    }
}

template <typename T, int N, int E, int P, int OFF, bool FIRST, int R, int... Rest>
__device__ __forceinline__ void stages(cplx<T> (&v)[E], int t, cplx<T> *sline, const cplx<T> *tw, const RegParams &rp,
                                       const LineIO &io) {
    constexpr bool LAST = sizeof...(Rest) == 0;
    stage<T, N, E, R, P, OFF, FIRST, LAST>(v, t, sline, tw, rp, io);
    // the first stage (P = 1) has no twiddles and no table rows
    constexpr int NEXT_OFF = OFF + (P > 1 ? (R - 1) * P : 0);
    if constexpr (!LAST) stages<T, N, E, P * R, NEXT_OFF, false, Rest...>(v, t, sline, tw, rp, io);
}

template <typename T, int N, int E, int G, int... Rs>
__global__ void __launch_bounds__(G *(N / E)) reg_fft_kernel(const __grid_constant__ RegParams rp) {
    constexpr int TT = N / E;
    constexpr int LS = N + N / 16 + 1;  // padded line stride in shared memory
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int g = threadIdx.x / TT;
    const int t = threadIdx.x - g * TT;
    const int64_t line = (int64_t)blockIdx.x * G + g;
    LineIO io;
    io.valid = line < rp.nlines;
    io.in_off = line * rp.in_stride;
    io.out_off = line * rp.out_stride;
    cplx<T> *sline = reinterpret_cast<cplx<T> *>(smem_raw) + g * LS;
    const cplx<T> *tw = reinterpret_cast<const cplx<T> *>(rp.tw);
    cplx<T> v[E];
    if (io.valid) {
        const auto *src = reinterpret_cast<const typename vec2<T>::type *>(rp.in) + io.in_off + t;
#pragma unroll
        for (int m = 0; m < E; m++) {
            const auto w = __ldcs(src + m * TT);
            v[m] = {w.x, rp.conj ? -w.y : w.y};
        }
    } else {
#pragma unroll
        for (int m = 0; m < E; m++) v[m] = {T(0), T(0)};
    }
    stages<T, N, E, 1, 0, true, Rs...>(v, t, sline, tw, rp, io);
}

}  // namespace regk

// ---- variant table ----------------------------------------------------------------

struct RegVariant {
    int is_double, n, threads, g;
    size_t smem;
    const void *fn;
    int radices[8];
};

#define RV(T, N, E, G, ...)                                                                                 \
    {sizeof(T) == 8, N, G *(N / E), G, (size_t)G *(N + N / 16 + 1) * sizeof(T) * 2,                       \
     (const void *)regk::reg_fft_kernel<T, N, E, G, __VA_ARGS__>, {__VA_ARGS__}}

static const RegVariant kRegVariants[] = {
    RV(float, 16, 16, 64, 16),          RV(float, 32, 16, 64, 16, 2),     RV(float, 64, 16, 32, 16, 4),
    RV(float, 128, 16, 16, 16, 8),      RV(float, 256, 16, 16, 16, 16),   RV(float, 512, 16, 8, 16, 16, 2),
    RV(float, 1024, 16, 4, 16, 16, 4),  RV(float, 2048, 16, 2, 16, 16, 8), RV(float, 4096, 16, 1, 16, 16, 16),
    RV(float, 8192, 16, 1, 16, 16, 16, 2),
    RV(double, 16, 16, 64, 16),         RV(double, 32, 16, 64, 16, 2),    RV(double, 64, 16, 32, 16, 4),
    RV(double, 128, 16, 16, 16, 8),     RV(double, 256, 16, 16, 16, 16),  RV(double, 512, 16, 8, 16, 16, 2),
    RV(double, 1024, 16, 4, 16, 16, 4), RV(double, 2048, 16, 2, 16, 16, 8), RV(double, 4096, 16, 1, 16, 16, 16),
    RV(double, 8192, 16, 1, 16, 16, 16, 2),
};
#undef RV

int reg_variant_for(bool is_double, size_t n) {
    for (int i = 0; i < (int)(sizeof(kRegVariants) / sizeof(kRegVariants[0])); i++)
        if (kRegVariants[i].is_double == (int)is_double && (size_t)kRegVariants[i].n == n) return i;
    return -1;
}

// Radix sequence of a variant (0-terminated in the table); returns the stage count.
int reg_variant_radices(int v, int *out) {
    int n = 0;
    while (n < 8 && kRegVariants[v].radices[n]) {
        out[n] = kRegVariants[v].radices[n];
        n++;
    }
    return n;
}

void reg_variant_shape(int v, int *threads, int *lines_per_cta, size_t *smem) {
    *threads = kRegVariants[v].threads;
    *lines_per_cta = kRegVariants[v].g;
    *smem = kRegVariants[v].smem;
}

void set_reg_kernel_smem_limits() {
    static unsigned long long done_mask = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
    if (done_mask & (1ull << dev)) return;
    for (const RegVariant &v : kRegVariants)
        cudaFuncSetAttribute(v.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)v.smem);
    done_mask |= 1ull << dev;
}

cudaError_t launch_reg(int variant, const RegParams &rp, cudaStream_t stream) {
    const RegVariant &v = kRegVariants[variant];
    const int64_t grid = (rp.nlines + v.g - 1) / v.g;
    void *args[] = {const_cast<RegParams *>(&rp)};
    return cudaLaunchKernel(v.fn, dim3((unsigned)grid), dim3(v.threads), args, v.smem, stream);
}

}  // namespace b200fft
