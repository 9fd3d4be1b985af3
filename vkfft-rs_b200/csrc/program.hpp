// Executable form of a transform: the launch list the B200 runtime replays.
// Built on the host from an FftPlan (lower.cpp); tables are generated in f64 on
// the host and uploaded once per context (runtime.cpp).
#pragma once

#include <complex>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "core.hpp"
#include "pass_desc.hpp"
#include "reg_kernels.hpp"

namespace b200fft {

enum BufId : int {
    BUF_IN = 0,
    BUF_OUT = 1,
    BUF_SCRATCH0 = 2,  // four-step / Bluestein intermediate
    BUF_SCRATCH1 = 3,  // ND C2R / convolution working copy
    BUF_SCRATCH2 = 4,  // real even-half child output
    BUF_SCRATCH3 = 5,  // pass-level Rader lines
    BUF_SCRATCH4 = 6,  // dense input behind a boundary copy (zero padding / formatted strides)
    BUF_SCRATCH5 = 7,  // dense output in front of a boundary copy
    BUF_SCRATCH6 = 8,  // convolution: spectrum of the input systems
    BUF_SCRATCH7 = 9,  // convolution: product spectra of the output systems
};
constexpr int kScratchBuffers = 8;

struct HostTable {
    std::string key;      // cache key: the table's kind and parameters (empty: uncached)
    bool is_int = false;
    bool is_raw = false;  // already in the pass precision (user-supplied convolution spectra)
    std::vector<std::complex<double>> c;   // values (double-double programs: the high words)
    std::vector<std::complex<double>> lo;  // double-double programs: the low words (c + lo)
    std::vector<int32_t> i;
    std::vector<unsigned char> raw;
    // bytes on the device for complex elements of `cbytes` bytes (8 f32, 16 f64, 32 dd)
    size_t bytes(int cbytes) const {
        if (is_raw) return raw.size();
        return is_int ? i.size() * 4 : c.size() * (size_t)cbytes;
    }
};

enum KernelKind : int { KERNEL_PASS = 0, KERNEL_REG = 1, KERNEL_COPY = 2, KERNEL_CMUL = 3, KERNEL_R2R = 4 };

struct PassPlan {
    int kernel = KERNEL_PASS;     // KERNEL_REG: register-resident Stockham (reg_kernels.cu)
    RegParams rp{};               // KERNEL_REG parameters (pointers patched at launch)
    int reg_variant = -1;
    int reg_table = -1;           // twiddle table id of a KERNEL_REG pass
    int reg_table2 = -1;          // KERNEL_REG HALF modes: the W_2h table
    int reg_table3 = -1;          // KERNEL_REG Bluestein four-step modes: the W_M twiddles
    int reg_variant_plain = -1;   // persistent reg_variant: the ordinary variant, used when the
                                  // input is not 16-byte aligned for the bulk copies
    bool reg_in_real = false, reg_out_real = false;
    PassParams p{};               // device pointers are patched at upload / launch
    BoundaryCopy bc{};            // KERNEL_COPY parameters (pointers patched at launch)
    ConvMultiply cm{};            // KERNEL_CMUL parameters; reg_table holds the kernel spectrum
    R2rPass rr{};                 // KERNEL_R2R parameters
    int op_tables[kMaxOps][3];    // table ids per op (lut, lut2, lut3) or -1
    int src_buf = BUF_IN, dst_buf = BUF_OUT;
    int64_t src_off = 0, dst_off = 0;  // element offsets (units of the side's element type)
    bool peer_scatter = false;    // the final store goes to the ranks' exchange buffers
    int64_t peer_es = 0;          // output distance between consecutive logical elements
    int64_t grid = 0;
    int threads = 0;
    size_t smem = 0;
    std::string label;
};

struct Program {
    bool is_double = false;  // compute in f64 (or in double-double when is_dd)
    bool is_dd = false;      // compute in double-double (DoubleDouble precisions)
    std::vector<PassPlan> passes;
    std::vector<HostTable> tables;
    std::map<std::string, int> table_cache;
    size_t scratch_elems[kScratchBuffers] = {};  // complex elements of the compute precision
    size_t input_elems = 0, output_elems = 0;
    bool input_real = false, output_real = false;
    double algorithmic_flops = 0;  // 5 N log2 N per complex transform (for reports)
    int storage_scalar_bytes = 0;  // bytes of one stored scalar of the caller's buffers: 2 (f16),
                                   // 4, 8; 0 = the compute precision's
    // Packed device image of `tables` (256-byte aligned entries), built on the first
    // static-workspace execution and kept for the program's lifetime: the source of that
    // entry point's per-call table upload (static_workspace.cu).
    mutable std::shared_ptr<const std::vector<unsigned char>> static_table_image;

    int rbytes() const { return is_dd ? 16 : (is_double ? 8 : 4); }  // one compute scalar
    int cbytes() const { return 2 * rbytes(); }                        // one compute complex
    int scalar_kind() const { return is_dd ? 2 : (is_double ? 1 : 0); }  // kernel type: f32, f64, dd
    size_t io_scalar_bytes() const { return storage_scalar_bytes ? (size_t)storage_scalar_bytes : (size_t)rbytes(); }
    size_t input_bytes() const { return input_elems * io_scalar_bytes() * (input_real ? 1 : 2); }
    size_t output_bytes() const { return output_elems * io_scalar_bytes() * (output_real ? 1 : 2); }

    size_t scratch_offset(int k) const {  // byte offset of scratch buffer k (256-byte aligned)
        size_t off = 0;
        for (int i = 0; i < k; i++) off += (scratch_elems[i] * (size_t)cbytes() + 255) & ~size_t(255);
        return off;
    }
    size_t scratch_bytes() const { return scratch_offset(kScratchBuffers); }
};

// Device image of a table in the program's precision: raw / int tables verbatim,
// complex tables as f32 pairs, f64 pairs or double-double quadruples (re.hi, re.lo,
// im.hi, im.lo, the reference's 32-byte DD complex layout).  `dst` holds t.bytes(cbytes).
inline void pack_table(const HostTable &t, const Program &prog, unsigned char *dst) {
    if (t.is_raw) {
        std::memcpy(dst, t.raw.data(), t.raw.size());
    } else if (t.is_int) {
        std::memcpy(dst, t.i.data(), t.i.size() * 4);
    } else if (prog.is_dd) {
        double *d = reinterpret_cast<double *>(dst);
        const bool has_lo = t.lo.size() == t.c.size();
        for (size_t m = 0; m < t.c.size(); m++) {
            d[4 * m] = t.c[m].real();
            d[4 * m + 1] = has_lo ? t.lo[m].real() : 0.0;
            d[4 * m + 2] = t.c[m].imag();
            d[4 * m + 3] = has_lo ? t.lo[m].imag() : 0.0;
        }
    } else if (prog.is_double) {
        std::memcpy(dst, t.c.data(), t.c.size() * 16);
    } else {
        float *f = reinterpret_cast<float *>(dst);
        for (size_t m = 0; m < t.c.size(); m++) {
            f[2 * m] = (float)t.c[m].real();
            f[2 * m + 1] = (float)t.c[m].imag();
        }
    }
}

FastDiv make_fastdiv(uint32_t d);

// Tables (host f64).  All roots are forward: W_N^m = exp(-2 pi i m / N).
int table_twiddle(Program &prog, size_t n);
int table_reg_twiddles(Program &prog, size_t n, int variant);
// Fails unless every register pass (and its misaligned-input fallback variant) that reads
// stage twiddles reads the table of its own variant's length and radix split.
void check_reg_twiddle_tables(const Program &prog);
int table_bluestein_chirp(Program &prog, size_t n);
int table_bluestein_spectrum(Program &prog, size_t n, size_t m);
int table_bluestein_spectrum_rows(Program &prog, size_t n, size_t m, size_t m1, size_t m2);
int table_r2r(Program &prog, int type, size_t n, size_t L);  // DCT/DST reduction twiddles [A | B]
void host_fft_inplace(std::vector<std::complex<double>> &x, bool inverse);

// Lowering of a whole transform (TransformIr families) into a Program.
struct LoweredTransform;

}  // namespace b200fft
