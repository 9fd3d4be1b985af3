// Parameters of the register-resident Stockham kernel (reg_kernels.cu).
#pragma once
#include <cstdint>

namespace b200fft {

struct RegParams {
    const void *in;
    void *out;
    const void *tw;      // forward W_N table of the pass precision
    int64_t nlines;      // transforms in this launch
    int64_t in_stride;   // complex elements between consecutive lines
    int64_t out_stride;
    double scale;        // applied on store
    int32_t conj;        // inverse: conjugate on load and on store
    int32_t n;
};

}  // namespace b200fft
