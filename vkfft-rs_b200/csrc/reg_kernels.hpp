// Parameters of the register-resident Stockham kernels (reg_kernels.cu).
#pragma once
#include <cstdint>

#include "pass_desc.hpp"

namespace b200fft {

// Register-kernel data modes.
enum RegMode : int32_t {
    REG_C2C = 0,      // complex in, complex out
    REG_R2C_FULL = 1, // real in (promoted on load), first N/2+1 bins out (RealFftAlgorithm::FullComplex)
    REG_C2R_FULL = 2, // N/2+1 Hermitian bins in (mirrored on load), real part out
    REG_C2C_PEER = 3, // REG_C2C whose output is scattered into the ranks' exchange buffers (slab)
};

// Line l = o * ni + i; element p of the line is at o*os + i*is + p*es (units of the
// side's element: complex, or scalar for a real side).
struct RegSide {
    int64_t os, is, es;
};

struct RegParams {
    const void *in;
    void *out;
    const void *tw;      // per-stage transposed twiddle tables (reg_kernels.cu)
    int64_t nlines;      // transforms in this launch
    int64_t ni;          // inner line count (1 for contiguous lines)
    RegSide src, dst;
    double scale;        // applied on store
    int32_t conj;        // inverse: conjugate on load and on store
    int32_t n;
    PeerStore peer;      // REG_C2C_PEER: the ranks' exchange buffers
};

}  // namespace b200fft
