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
    REG_R2C_HALF = 4, // N = h: 2h reals read as h complex pairs, FFT_h, even-half post-processing
                      // (real_ir.rs:1002-1013) -> h+1 bins
    REG_C2R_HALF = 5, // N = h: h+1 bins, even-half pre-processing (real_ir.rs:1087-1100), inverse
                      // FFT_h -> 2h reals stored as h complex pairs
    REG_CONV = 6,     // strided lines: FFT, pointwise multiply by a spectrum table (tw2), inverse
                      // FFT (the fused outermost axis of the FFT convolution)
    REG_R2R = 7,      // DCT/DST of one axis: the FFT reduction's pre-processing on load (reads the
                      // real line), the FFT of length N = L, the post-processing on store (writes
                      // the real line); tw2 holds the reduction's twiddles by FFT position
    REG_R2R_HALF = 8, // DCT/DST-II/III of a contiguous line of n = 2N reals: the reduction's real
                      // length-n sequence through the even-half algebra, FFT of length N;
                      // tw2 = [W_n^k | W_4n^k], k = 0..N
    REG_RADER_LINE = 9,  // prime-length lines, one thread per line: Rader's algorithm in registers
                         // (N = P; tw = FFT_{P-1} of the Rader kernel / (P - 1))
    // The column passes of a four-step Bluestein convolution of a contiguous axis, M = M1 M2,
    // block position pos = n2 + M2 k1 of a line's M-point scratch block (lower.cpp; the rows
    // between them run the generic pass):
    REG_BLU_A = 10,   // strided columns n2 (length M1): x[n] * chirp[n] for n = n2 + M2 n1 < rp.n
                      // (else 0; conjugated first when inverse), FFT, * W_M^(n2 k1) = tw3[pos]
    REG_BLU_C = 12,   // strided columns: inverse FFT (conjugation trick), * chirp[n], scale, stored
                      // for n = n2 + M2 n1 < rp.n (conjugated last when inverse)
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
    const void *tw2;     // HALF modes: W_{2h}^k, k = 0..h; Bluestein modes: chirp / spectrum rows
    const void *tw3;     // Bluestein four-step modes: W_M^(n2 k1) by block position
    int64_t nlines;      // transforms in this launch
    int64_t ni;          // inner line count (1 for contiguous lines)
    RegSide src, dst;
    double scale;        // applied on store
    double scale2;       // REG_C2R_HALF: applied by the pre-processing (1/2 when normalised)
    int32_t conj;        // inverse: conjugate on load and on store
    int32_t n;
    int32_t real_ends;   // REG_C2R_HALF: use only the real parts of X[0] and X[h] (the
                         // FullComplex C2R result: its real output ignores those imaginary parts)
    int32_t conv_flags;  // REG_CONV: F_CONJ_IN / F_NORMALIZE / F_CONJ_OUT of the multiply
    int32_t r2r_kind;    // REG_R2R: effective kind 0..3 DCT-I..IV, 4..7 DST-I..IV
    int32_t r2r_n;       // REG_R2R: logical length of the real line
    int64_t conv_em;     // REG_CONV: spectrum index = i + p * conv_em + o * conv_om
    int64_t conv_om;
    int *err;            // persistent variants: error word (a bulk copy that never completed)
    PeerStore peer;      // REG_C2C_PEER: the ranks' exchange buffers
};

}  // namespace b200fft
