// Launch descriptor of one B200 FFT pass, shared by the host lowering and the
// device kernel.  A pass processes a batch of "lines" (independent 1D
// sub-transforms) with one CTA per G lines: the lines are loaded into shared
// memory, transformed by a short program of in-CTA operations (Stockham radix
// stages, pointwise multiplies, Rader gather/scatter, real-FFT pre/post
// processing) and stored back.  Plain POD so it can be a __grid_constant__
// kernel parameter.
#pragma once
#include <cstdint>

namespace b200fft {

constexpr int kMaxOps = 24;

enum OpType : int32_t {
    OP_LOAD = 1,           // global -> line region (with optional multiply / conjugation)
    OP_STORE = 2,          // line region -> global
    OP_STAGE = 3,          // one in-place Stockham radix stage over a region's sub-lines
    OP_MUL = 4,            // pointwise multiply of a region by a table
    OP_R2C_POST = 5,       // even-N R2C post-processing of a half-length spectrum
    OP_C2R_PRE = 6,        // even-N C2R pre-processing into a half-length spectrum
    OP_RADER_GATHER = 7,   // radix-p Rader step: twiddle, generator permutation into the W region
    OP_RADER_SCATTER = 8,  // radix-p Rader step: x0 + convolution -> Stockham output positions
    OP_HERM_EXPAND = 9,    // fill slots N/2+1..N-1 of a Hermitian half spectrum with conj(X[N-k])
    OP_PERMUTE_GATHER = 10,   // pass-level Rader: dst[m] = src[g^m] (m < p-1), dst[p-1] = src[0]
    OP_PERMUTE_SCATTER = 11,  // pass-level Rader: dst[g^-m] = x0 + c[m], dst[0] = x0 + A0
    OP_SAVE_DC = 12,          // line[slot] = line[0] (keeps the convolution's DC term)
};

enum MulKind : int32_t {
    MUL_NONE = 0,
    MUL_LUT_N = 1,       // value *= lut[n], n = c*cm + e*em (logical index of the element)
    MUL_TWIDDLE_CE = 2,  // value *= lut[c*e]  (four-step twiddle, c*e < table size)
};

enum OpFlags : int32_t {
    F_CONJ_IN = 1,    // conjugate the data before the multiply
    F_CONJ_LUT = 2,   // multiply by the conjugate of the table value
    F_CONJ_OUT = 4,   // conjugate the data after the multiply
    F_SAVE_DC = 8,    // OP_MUL: copy element 0 of every sub-line into the X0 region (slot 1) first
    F_DIRECT = 16,    // OP_RADER_SCATTER: direct O(p^2) convolution instead of the FFT result
    F_SCALE = 32,     // apply Op::scale
    F_OWN_INDEX = 64, // LOAD/STORE multiply: table index = c*op.cm + e*op.em (not the side's n)
    F_NORMALIZE = 128,  // OP_MUL: divide the product by its modulus (cross-power spectrum)
    F_LINE_FAST = 256,  // OP_MUL: threads walk the lines fastest (the table's fast index is the line)
};

// Fast unsigned division by a run-time constant (round-up multiply-shift, valid for n < 2^31).
struct FastDiv {
    uint32_t d, m, s, _pad;
};

// Global addressing of one side (input or output) of a pass.  A line index l is
// decomposed as l = (o * nc + c) * ni + i; element e of the line lives at
//   base + o*os + i*is + c*cs + e*es
// (units: complex elements, or scalars when real != 0).  The element's logical
// index within the full axis is n = c*cm + e*em; only n < count is read (others
// load as zero) or written.
struct Side {
    int64_t os, is, cs, es;
    int32_t real;
    int32_t count;
    int32_t cm, em;
    int32_t herm;  // input only: N when the side stores N/2+1 Hermitian bins; logical
                   // n > N/2 reads bin N-n conjugated (cm must be 0 or 1)
    int32_t _pad;
};

struct alignas(16) Op {
    int32_t type;
    int32_t flags;
    int32_t radix;      // STAGE radix; RADER prime p
    int32_t P;          // STAGE/RADER: product of the radices already applied (sub-transform span)
    int32_t len;        // length of the transform (sub-line length) this op works on
    int32_t nsub;       // number of sub-lines in the region
    int32_t src_base;   // shared-memory offset of the source region (complex elements)
    int32_t dst_base;   // shared-memory offset of the destination region
    int32_t sub_stride; // shared-memory distance between sub-lines (complex elements)
    int32_t mul;        // MulKind for LOAD/STORE/MUL
    int32_t cm, em;     // MUL: table index = c*cm + e*em (MUL_LUT_N)
    int32_t w_base;     // RADER: W region base (gather destination / scatter source)
    int32_t w_stride;   // RADER: W sub-line stride
    int32_t x0_base;    // RADER / MUL(F_SAVE_DC): X0 region base, two slots per butterfly
    int32_t nfull;      // R2C/C2R/HERM_EXPAND: full real length N; MUL: only n < nfull (0: all)
    int32_t pad_shift;  // shared-memory slot of element e: e + (e >> pad_shift) (31: unpadded);
                        // one value for every op of a pass
    FastDiv div_a;      // STAGE: len/radix; RADER: len/p; LOAD/STORE/MUL: len
    FastDiv div_b;      // STAGE/RADER: P
    FastDiv div_c;      // RADER: p
    const void *lut;    // twiddle / multiply table (complex of the pass precision)
    const void *lut2;   // RADER: generator powers (int32) ; R2C/C2R: W_N table
    const void *lut3;   // RADER: inverse generator powers (int32)
    double scale;
    int64_t om;         // MUL: table index += (line's outer index o) * om
    int64_t lut_off;    // MUL: table index += lut_off
    double scale_lo;    // double-double programs: low word of the scale (scale + scale_lo)
};

// Peer scatter of a pass's final store (the slab exchange fused into the last local FFT
// pass): the logical element index n of the axis selects the owner rank r = n / chunk and
// the element goes to ptr[r] at (local address) - r*sub + off.  n == 0 disables it.
constexpr int kMaxPeers = 8;
struct PeerStore {
    void *ptr[kMaxPeers];
    int64_t sub;    // chunk * (distance between consecutive logical elements)
    int64_t off;    // this rank's offset inside every destination block
    int32_t n;      // number of ranks (0: ordinary store)
    int32_t chunk;  // logical elements per destination rank
    FastDiv div;    // chunk
};

// Everything a pass launch describes except its op list (the op functions read this).
struct PassShape {
    int64_t nlines;   // total number of lines in this launch
    int64_t ni, nc;   // line decomposition
    int32_t G;        // lines per CTA
    int32_t nops;
    int32_t line_len;     // elements kept per line in shared memory
    int32_t line_stride;  // shared-memory distance between lines (odd, padded)
    int32_t meta_off;     // byte offset of the per-line address table in shared memory
    int32_t _pad;
    FastDiv div_g;        // G
    Side in, out;
    const void *src;
    void *dst;
    int *err;         // device error word (0 = ok), set instead of trapping
    PeerStore peer;   // STORE ops: optional scatter into the ranks' exchange buffers
};

struct PassParams : PassShape {
    Op ops[kMaxOps];
};

// Convolution multiply (convolution_ir.rs:36-151, :4252-4440): out system s, coordinate
// oc, element i of a T-element tensor:
//   matrix:   sum_ic prep(spec[(in_s C + ic) T + i]) ker[(kid planes + plane(oc, ic)) T + i]
//   scalar:   prep(spec[(in_s C + oc) T + i]) ker[(kid C + oc) T + i]
// with in_s = 0, kid = s for K > 1 (one input system fanned out to K kernels) and in_s = s,
// kid = 0 otherwise (C = 1 for the C2C scalar case; C > 1 is the ND real path's
// independent coordinates); a shared kernel is one tensor for every (kid, oc).  prep
// conjugates the sequence (Sequence policy) and the product is divided by its modulus
// with cross-power normalisation.
struct ConvMultiply {
    const void *src;
    void *dst;
    const void *ker;
    int64_t T;            // tensor elements
    int64_t total;        // output elements: out_systems * C * T
    int32_t C;            // coordinates per system
    int32_t K;            // kernels
    int32_t matrix;       // 0 (scalar) or the matrix size
    int32_t symmetric;
    int32_t planes;       // kernel planes per kernel set
    int32_t conj_seq;
    int32_t cross_power;
    int32_t shared_kernel;  // scalar: one kernel tensor for every output system
};

// DCT / DST of one axis (r2r_ir.rs:621-1110) as pre pass -> complex FFT of length L ->
// post pass, the reductions of the reference's FFT-reduction IR (r2r_ir.rs:1282-1500):
//   DCT-I   L = 2(N-1) even extension, forward      X_k = Re Y_k
//   DST-I   L = 2(N+1) odd extension, forward       X_k = -Im Y_{k+1}
//   DCT-II  L = N  even/odd reorder, forward         X_k = 2 Re(Y_k e^{-i pi k/2N})
//   DCT-III L = N  half-shifted spectrum, inverse     unreorder Re
//   DST-II/III: the same with alternating signs and reversed index
//   IV, N even: L = N/2 packed pairs with pre/post twiddles, inverse
//   IV, N odd:  L = 2N  pre-twiddled zero-extended, forward
// The tensor is [outer][N][inner]; the complex work array is [outer][L][inner], so a
// thread index with `inner` fastest reads and writes coalesced lines for every axis.
// kind: 0..3 DCT-I..IV, 4..7 DST-I..IV (the effective transform: II and III swap
// for the inverse direction).  tb: the reduction's twiddles by FFT position, [A | B]
// (A the pre-processing, B the post-processing factor; lower.cpp table_r2r).
struct R2rPass {
    const void *src;
    void *dst;
    const void *tb;
    int64_t outer;  // batch x product of the slower dims
    int64_t inner;  // product of the faster dims
    int64_t n;      // logical length of the axis
    int64_t L;      // FFT length
    int64_t total;  // threads: outer * L * inner (pre) or outer * n * inner (post)
    int32_t kind;
    int32_t pre;    // 1: real tensor -> complex work array, 0: spectrum -> real tensor
    double scale;
    double scale_lo;  // double-double programs: low word of the scale
};

// Boundary copy between a caller's buffer and a dense scratch tensor, with the
// zero-padding interval applied (zero_pad_ir.rs: elements whose coordinate on any padded
// axis lies in [pad_lo, pad_hi) become zero) and formatted buffer strides
// (config.rs:893-1002: per-axis stored-element strides and a batch stride).  Element L of
// the batch-major logical tensor has coordinates (batch, c_0 .. c_{rank-1}), fastest last.
constexpr int kMaxCopyRank = 8;
struct BoundaryCopy {
    const void *src;
    void *dst;
    int64_t total;       // logical elements over all batches
    int32_t rank;
    int32_t scalars;     // scalars per element: 1 (real) or 2 (complex)
    int32_t src_bytes;   // bytes per scalar of the source: 2 (f16), 4 (f32), 8 (f64)
    int32_t dst_bytes;   // ... of the destination (a conversion when they differ)
    int64_t dims[kMaxCopyRank];
    int64_t src_stride[kMaxCopyRank], dst_stride[kMaxCopyRank];
    int64_t src_batch, dst_batch;
    int64_t pad_lo[kMaxCopyRank], pad_hi[kMaxCopyRank];
};

}  // namespace b200fft
