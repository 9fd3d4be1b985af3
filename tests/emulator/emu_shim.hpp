// Host definitions of the CUDA keywords and intrinsics used by kernels.cu, so the
// kernel's op functions can be compiled as plain C++ and executed thread by thread
// on the CPU (test infrastructure only).
#pragma once
#include <vector_types.h>

#include <cstdint>

#undef __global__
#undef __device__
#undef __host__
#undef __forceinline__
#undef __launch_bounds__
#undef __grid_constant__
#undef __shared__
#undef __align__
#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __grid_constant__
#define __shared__
#define __align__(n) alignas(n)

struct EmuDim {
    unsigned x = 0, y = 0, z = 0;
};
extern EmuDim threadIdx, blockIdx, blockDim;

inline uint32_t __umulhi(uint32_t a, uint32_t b) { return (uint32_t)(((uint64_t)a * b) >> 32); }
template <class T> inline T __ldg(const T *p) { return *p; }
template <class T> inline T __ldcs(const T *p) { return *p; }
template <class T> inline void __stcs(T *p, T v) { *p = v; }
inline int atomicOr(int *p, int v) {
    int o = *p;
    *p |= v;
    return o;
}
inline void __syncthreads() {}
inline void __threadfence_system() {}
