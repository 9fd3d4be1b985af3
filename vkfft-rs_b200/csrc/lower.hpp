// Lowering interface: axis jobs -> passes of a Program.
#pragma once

#include "program.hpp"

namespace b200fft {

// One complex axis transform over a dense tensor viewed as [no][N][S]: line (o, i)
// has element e at off + o*os + i + e*S.  (S = 1 for the contiguous axis.)
struct AxisJob {
    size_t N = 1;
    const AxisAlgorithm *alg = nullptr;
    int64_t no = 1, S = 1;
    bool inverse = false;
    double scale = 1.0;
    int in_buf = BUF_IN, out_buf = BUF_OUT;
    int64_t in_off = 0, out_off = 0;
    int64_t in_os = 0, out_os = 0;
    bool in_real = false;   // promote real input (FullComplex R2C)
    bool in_herm = false;   // input holds N/2+1 Hermitian bins (FullComplex C2R)
    bool out_real = false;  // keep the real part (FullComplex C2R)
    size_t out_count = 0;   // bins stored per line (0: N)
    PlannerTuning tuning;   // tuning of the plan (nested Rader convolutions are planned with it)
    bool in_nested_rader = false;  // inside a pass-level Rader convolution
    int64_t out_S = 0;      // element stride of the output side (0: S, the input's)
};

// Real transform of the contiguous axis: lines of N reals <-> N/2+1 complex bins.
struct RealAxisJob {
    size_t N = 2;
    int64_t lines = 1;
    bool normalize = false;
    bool full_complex = false;  // RealFftAlgorithm::FullComplex
    const AxisAlgorithm *alg = nullptr;  // algorithm of the executed complex child
    PlannerTuning tuning;
    int in_buf = BUF_IN, out_buf = BUF_OUT;
    int64_t in_off = 0, out_off = 0;
};

// DCT/DST of one axis of a real tensor [outer][n][inner] through its FFT reduction of
// length L (effective kind 0..3 DCT-I..IV, 4..7 DST-I..IV; fft_inverse: the reduction's
// FFT runs inverse).  Emits one register pass with the pre/post-processing fused into
// its load and store when L is a power of two with a register variant; false otherwise.
struct R2rAxisJob {
    size_t n = 1, L = 1;
    int kind = 0;
    bool fft_inverse = false;
    const AxisAlgorithm *alg = nullptr;  // algorithm of the internal FFT plan
    int64_t outer = 1, inner = 1;
    double scale = 1.0;
    int in_buf = BUF_IN, out_buf = BUF_OUT;
};
bool lower_r2r_axis_register(Program &prog, const R2rAxisJob &job);

std::vector<int> radix_schedule(size_t L);
int reg_variant_for(bool is_double, size_t n, int mode, bool strided);  // reg_kernels.cu (-1: none)
int reg_variant_radices(int v, int *out);
int reg_variant_peer_twin(int v);  // REG_C2C -> REG_C2C_PEER variant (-1: none)
int reg_variant_persistent_twin(int v);  // contiguous C2C / R2R / even-half -> bulk-prefetch variant (-1: none)
int reg_variant_lines_per_cta(int v);
int reg_variant_length(int v);
bool line_fits_on_chip(int complex_bytes, size_t L, const AxisAlgorithm *alg, bool strided);
void lower_c2c_axis(Program &prog, const AxisJob &job);
void lower_r2c_axis(Program &prog, const RealAxisJob &job);
void lower_c2r_axis(Program &prog, const RealAxisJob &job);

}  // namespace b200fft
