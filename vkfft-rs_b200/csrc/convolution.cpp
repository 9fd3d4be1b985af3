// FFT convolution applications: the C2C ConvolutionIr / NdConvolutionIr (build_c2c_convolution)
// and the ND real independent-coordinate path of NdRealConvolutionIr (convolution_ir.rs:3867-4250).
//
// Reference semantics: the C coordinate images are R2C-transformed (batch C), every
// output system (kernel k, coordinate c) is out[(k C + c) L + i] =
// policy(seq[c L + i]) * ker[(k C + c) L + i] (optional sequence conjugation and
// cross-power normalisation, convolution_ir.rs:36-86), and the K C systems are
// inverse-transformed by a normalised C2R.
//
// B200 program for K = 1: R2C rows into scratch, forward passes of the middle axes, ONE
// fused pass on the outermost axis (forward FFT, spectrum multiply, inverse FFT in shared
// memory), inverse middle axes, normalised C2R rows into the output.  K > 1 fans out
// through an explicit multiply pass.  The reference requires K C copies of the kernel
// spectrum; a single copy is accepted too and broadcast to every coordinate.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>

#include "transform.hpp"

namespace b200fft {

// PassBuilder-level helpers from lower.cpp
void lower_convolution_axis0(Program &prog, size_t H, const AxisAlgorithm *alg, const PlannerTuning &tuning,
                             int64_t systems, int64_t inner, int buf, int spec_table, int64_t spec_outer_stride,
                             bool conj_sequence, bool cross_power, double scale);
void lower_convolution_multiply(Program &prog, int64_t L, int64_t C, int64_t K, int in_buf, int out_buf,
                                int spec_table, int64_t spec_copies, bool conj_sequence, bool cross_power);

static size_t prod(const std::vector<size_t> &v, size_t a, size_t b) {
    size_t r = 1;
    for (size_t i = a; i < b; i++) r = checked_mul(r, v[i], "convolution tensor size");
    return r;
}

// Appends the passes and tables of `src` to `dst`, renaming buffers through `remap`.
static void append_program(Program &dst, const Program &src, const int (&remap)[2 + kScratchBuffers]) {
    const int off = (int)dst.tables.size();
    dst.tables.insert(dst.tables.end(), src.tables.begin(), src.tables.end());
    for (PassPlan pp : src.passes) {
        for (auto &row : pp.op_tables)
            for (int &id : row)
                if (id >= 0) id += off;
        if (pp.reg_table >= 0) pp.reg_table += off;
        if (pp.reg_table2 >= 0) pp.reg_table2 += off;
        if (pp.reg_table3 >= 0) pp.reg_table3 += off;
        pp.src_buf = remap[pp.src_buf];
        pp.dst_buf = remap[pp.dst_buf];
        dst.passes.push_back(pp);
    }
    for (int k = 0; k < kScratchBuffers; k++) dst.scratch_elems[k] = std::max(dst.scratch_elems[k], src.scratch_elems[k]);
}

// C2C convolution: ConvolutionIr (rank 1, convolution_ir.rs:2520-3626) and NdConvolutionIr
// (rank >= 2, :3627-3866).  Forward transform of the batch x coordinate systems (into the
// output buffer), the multiply (scalar, K-kernel fan-out or 2x2 / 3x3 matrix, with the
// conjugation / cross-power policy) into scratch 4, normalised inverse transform of the
// output systems.  The kernel spectrum holds `planes x K` tensors of T elements.
static std::unique_ptr<Convolution> build_c2c_convolution(const FftConfig &c, const DeviceProfile &device,
                                                          const void *spectrum, uint64_t copies) {
    const size_t R = c.dimensions.size();
    const size_t T = prod(c.dimensions, 0, R);
    const int M = c.matrix_convolution > 1 ? (int)c.matrix_convolution : 0;
    if (M && M != 2 && M != 3) fail_invalid_ir("matrix convolution IR requires a 2x2 or 3x3 matrix");
    if (M == 3 && c.symmetric_convolution_kernel)
        fail_unsupported(
            "pinned VkFFT 1.3.4 3x3 symmetric-kernel code aliases yz and zz while the API guide documents six planes");
    if (c.convolution_conjugation == ConvolutionConjugation::Kernel)
        fail_unsupported("kernel-conjugated convolution is not executable in the pinned VkFFT codegen");
    const size_t C = M ? (size_t)M : c.coordinate_features, K = c.convolution_kernel_count, B = c.batch_count;
    bool padded = c.has_formatted_strides();
    for (auto &z : c.zero_padding) padded |= z.has_value();
    for (size_t a = 0; a < R; a++) padded |= c.omit_dimension.size() > a && c.omit_dimension[a];
    if (R >= 2) {
        const bool scalar_ok = !M && C == 1 && (K == 1 || B == 1);
        const bool matrix_ok = M && B == 1 && K == 1;
        if (!scalar_ok && !matrix_ok)
            fail_unsupported(
                "multidimensional performConvolution IR supports scalar K=1/K>1 ownership or batch1/K1 matrix "
                "coordinates");
        if (padded) fail_unsupported("multidimensional performConvolution currently requires dense unpadded active dimensions");
    } else {
        if ((!M && C != 1) || (K > 1 && B != 1))
            fail_unsupported("performConvolution supports one coordinate plane (or matrix coordinates) and K > 1 "
                             "kernels on one input batch");
        if (padded) fail_unsupported("B200 engine: padded or formatted performConvolution is not implemented");
    }
    const size_t planes = M ? (c.symmetric_convolution_kernel ? (size_t)(M * (M + 1) / 2) : (size_t)(M * M)) : 1;
    if (copies * T != T * planes * K)
        fail_invalid_ir("convolution kernel spectrum length must match its scalar/independent/matrix plane layout");
    const bool dbl = c.precision == Precision::F64;
    const size_t esz = dbl ? 16 : 8;
    const size_t n_scalars = copies * T * 2;
    for (size_t k = 0; k < n_scalars; k++) {
        const double v = dbl ? static_cast<const double *>(spectrum)[k] : (double)static_cast<const float *>(spectrum)[k];
        if (!std::isfinite(v)) fail_invalid_ir("convolution kernel spectrum contains non-finite values");
    }
    auto conv = std::make_unique<Convolution>();
    static std::atomic<uint64_t> next_id{1ull << 42};
    conv->id = next_id++;
    conv->config = c;
    conv->device = device;
    conv->spectrum_elems = T;
    const size_t out_systems = K > 1 ? K : B;
    FftConfig fc = c;
    fc.perform_convolution = false;
    fc.convolution_conjugation = ConvolutionConjugation::None;
    fc.cross_power_spectrum_normalization = false;
    fc.coordinate_features = 1;
    fc.matrix_convolution = 1;
    fc.symmetric_convolution_kernel = false;
    fc.convolution_kernel_count = 1;
    fc.batch_count = B * C;
    fc.normalize_inverse = false;
    conv->forward = build_transform(fc, B200FFT_FORWARD, device);
    FftConfig ic = fc;
    ic.batch_count = out_systems * C;
    ic.normalize_inverse = true;
    conv->inverse = build_transform(ic, B200FFT_INVERSE, device);

    Program &prog = conv->prog;
    prog.is_double = dbl;
    prog.input_elems = conv->logical_in_elems = B * C * T;
    prog.output_elems = conv->logical_out_elems = out_systems * C * T;
    int same[2 + kScratchBuffers];
    for (int k = 0; k < 2 + kScratchBuffers; k++) same[k] = k;
    append_program(prog, conv->forward->prog, same);  // spectrum of the input systems -> out
    HostTable st;
    st.is_raw = true;
    st.raw.assign(static_cast<const unsigned char *>(spectrum),
                  static_cast<const unsigned char *>(spectrum) + copies * T * esz);
    prog.tables.push_back(std::move(st));
    PassPlan mp{};
    mp.kernel = KERNEL_CMUL;
    mp.reg_table = (int)prog.tables.size() - 1;
    mp.cm.T = (int64_t)T;
    mp.cm.total = (int64_t)(out_systems * C * T);
    mp.cm.C = (int32_t)C;
    mp.cm.K = (int32_t)K;
    mp.cm.matrix = M;
    mp.cm.symmetric = c.symmetric_convolution_kernel ? 1 : 0;
    mp.cm.planes = (int32_t)planes;
    mp.cm.conj_seq = c.convolution_conjugation == ConvolutionConjugation::Sequence ? 1 : 0;
    mp.cm.cross_power = c.cross_power_spectrum_normalization ? 1 : 0;
    mp.src_buf = BUF_OUT;
    mp.dst_buf = BUF_SCRATCH4;
    mp.label = "convolution multiply";
    for (auto &row : mp.op_tables) row[0] = row[1] = row[2] = -1;
    prog.passes.push_back(mp);
    prog.scratch_elems[4] = std::max(prog.scratch_elems[4], out_systems * C * T);
    int inv_map[2 + kScratchBuffers];
    for (int k = 0; k < 2 + kScratchBuffers; k++) inv_map[k] = k;
    inv_map[BUF_IN] = BUF_SCRATCH4;
    append_program(prog, conv->inverse->prog, inv_map);  // normalised inverse -> out
    return conv;
}

// Checks a user kernel spectrum of `n_scalars` values for non-finite entries.
static void check_spectrum_finite(const void *spectrum, size_t n_scalars, bool dbl) {
    for (size_t k = 0; k < n_scalars; k++) {
        const double v = dbl ? static_cast<const double *>(spectrum)[k] : (double)static_cast<const float *>(spectrum)[k];
        if (!std::isfinite(v)) fail_invalid_ir("convolution kernel spectrum contains non-finite values");
    }
}

// ND real convolution in its general ownerships (NdRealConvolutionIr::build_from_spectrum,
// convolution_ir.rs:3884-4059): 2x2 / 3x3 matrix coordinates, zero padding (matrix,
// independent or scalar ownership) and formatted buffer strides (scalar, K = 1).  As the
// reference composes it: the forward R2C of the C coordinate systems (the config's zero
// padding and input strides, output dense), the multiply of the compact spectra into the
// K * C output systems (matrix, independent or scalar, with the conjugation / cross-power
// policy), the normalised C2R of the output systems (zero padding, output strides).  The
// three programs are concatenated into one launch list: forward output -> scratch 6,
// multiply -> scratch 7, inverse input <- scratch 7.  The unpadded independent case keeps
// the fused program of build_convolution below.
static std::unique_ptr<Convolution> build_real_convolution_generic(const FftConfig &c, const DeviceProfile &device,
                                                                   const void *spectrum, uint64_t copies) {
    const size_t rank = c.dimensions.size();
    const int M = c.matrix_convolution > 1 ? (int)c.matrix_convolution : 0;
    const size_t C = c.coordinate_features, K = c.convolution_kernel_count;
    const size_t W = c.dimensions[rank - 1];
    std::vector<size_t> compact = c.dimensions;
    compact[rank - 1] = W / 2 + 1;
    const size_t L = prod(compact, 0, rank);
    const size_t planes = M ? (c.symmetric_convolution_kernel ? (size_t)(M * (M + 1) / 2) : (size_t)(M * M)) : 1;
    const size_t expect = M ? K * planes : K * C;
    const bool shared = !M && copies == 1 && expect > 1;
    if (copies != expect && !shared)
        throw FftError(B200FFT_INPUT_LENGTH_MISMATCH, "input contains " + std::to_string(copies * L) +
                                                          " complex elements but kernel expects " +
                                                          std::to_string(expect * L));
    const bool dbl = c.precision == Precision::F64;
    const size_t esz = dbl ? 16 : 8;
    check_spectrum_finite(spectrum, copies * L * 2, dbl);
    auto conv = std::make_unique<Convolution>();
    static std::atomic<uint64_t> next_id{1ull << 43};
    conv->id = next_id++;
    conv->config = c;
    conv->device = device;
    conv->spectrum_elems = L;
    FftConfig fc = c;
    fc.perform_convolution = false;
    fc.convolution_conjugation = ConvolutionConjugation::None;
    fc.cross_power_spectrum_normalization = false;
    fc.coordinate_features = 1;
    fc.matrix_convolution = 1;
    fc.symmetric_convolution_kernel = false;
    fc.convolution_kernel_count = 1;
    fc.batch_count = C;
    fc.normalize_inverse = false;
    fc.output_buffer_axis_strides.assign(rank, std::nullopt);
    fc.output_buffer_batch_stride.reset();
    conv->forward = build_transform(fc, B200FFT_FORWARD, device);
    FftConfig ic = fc;
    ic.transform = TransformKind::C2R;
    ic.batch_count = K * C;
    ic.normalize_inverse = true;
    ic.input_buffer_axis_strides.assign(rank, std::nullopt);
    ic.input_buffer_batch_stride.reset();
    ic.output_buffer_axis_strides = c.output_buffer_axis_strides;
    ic.output_buffer_batch_stride = c.output_buffer_batch_stride;
    conv->inverse = build_transform(ic, B200FFT_INVERSE, device);

    Program &prog = conv->prog;
    prog.is_double = dbl;
    prog.input_real = prog.output_real = true;
    prog.input_elems = conv->forward->prog.input_elems;
    prog.output_elems = conv->inverse->prog.output_elems;
    conv->logical_in_elems = conv->forward->logical_in_elems;
    conv->logical_out_elems = conv->inverse->logical_out_elems;
    int fwd_map[2 + kScratchBuffers], inv_map[2 + kScratchBuffers];
    for (int k = 0; k < 2 + kScratchBuffers; k++) fwd_map[k] = inv_map[k] = k;
    fwd_map[BUF_OUT] = BUF_SCRATCH6;
    inv_map[BUF_IN] = BUF_SCRATCH7;
    append_program(prog, conv->forward->prog, fwd_map);
    HostTable st;
    st.is_raw = true;
    st.raw.assign(static_cast<const unsigned char *>(spectrum),
                  static_cast<const unsigned char *>(spectrum) + copies * L * esz);
    prog.tables.push_back(std::move(st));
    PassPlan mp{};
    mp.kernel = KERNEL_CMUL;
    mp.reg_table = (int)prog.tables.size() - 1;
    mp.cm.T = (int64_t)L;
    mp.cm.total = (int64_t)(K * C * L);
    mp.cm.C = (int32_t)C;
    mp.cm.K = (int32_t)K;
    mp.cm.matrix = M;
    mp.cm.symmetric = c.symmetric_convolution_kernel ? 1 : 0;
    mp.cm.planes = (int32_t)planes;
    mp.cm.conj_seq = c.convolution_conjugation == ConvolutionConjugation::Sequence ? 1 : 0;
    mp.cm.cross_power = c.cross_power_spectrum_normalization ? 1 : 0;
    mp.cm.shared_kernel = shared ? 1 : 0;
    mp.src_buf = BUF_SCRATCH6;
    mp.dst_buf = BUF_SCRATCH7;
    mp.label = "convolution multiply";
    for (auto &row : mp.op_tables) row[0] = row[1] = row[2] = -1;
    prog.passes.push_back(mp);
    append_program(prog, conv->inverse->prog, inv_map);
    prog.scratch_elems[6] = std::max(prog.scratch_elems[6], std::max(C * L, conv->forward->prog.output_elems));
    prog.scratch_elems[7] = std::max(prog.scratch_elems[7], std::max(K * C * L, conv->inverse->prog.input_elems));
    if (c.has_formatted_strides()) {
        FftConfig dense = c;
        dense.input_buffer_axis_strides.assign(rank, std::nullopt);
        dense.output_buffer_axis_strides.assign(rank, std::nullopt);
        dense.input_buffer_batch_stride.reset();
        dense.output_buffer_batch_stride.reset();
        conv->dense_twin = build_real_convolution_generic(dense, device, spectrum, copies);
    }
    return conv;
}

std::unique_ptr<Convolution> build_convolution(const FftConfig &config_in, const DeviceProfile &device,
                                               const void *spectrum, uint64_t copies) {
    config_in.validate();
    if (config_in.perform_convolution && config_in.transform == TransformKind::C2C) {
        if (!(config_in.precision == Precision::F32 || config_in.precision == Precision::F64))
            fail_precision("B200 engine", precision_name(config_in.precision));
        auto conv = build_c2c_convolution(config_in.resolve_tuning_for_device(device), device, spectrum, copies);
        check_reg_twiddle_tables(conv->prog);
        return conv;
    }
    if (!config_in.perform_convolution || config_in.transform != TransformKind::R2C ||
        config_in.dimensions.size() < 2 || config_in.batch_count != 1)
        fail_unsupported(
            "multidimensional real performConvolution IR requires batch1 ND R2C application ownership");
    // ownership rules of NdRealConvolutionIr::build_from_spectrum (convolution_ir.rs:3899-3937)
    const int Mx = config_in.matrix_convolution > 1 ? (int)config_in.matrix_convolution : 0;
    if (Mx && Mx != 2 && Mx != 3) fail_invalid_ir("matrix convolution IR requires a 2x2 or 3x3 matrix");
    if (Mx == 3 && config_in.symmetric_convolution_kernel)
        fail_unsupported(
            "pinned VkFFT 1.3.4 3x3 symmetric-kernel code aliases yz and zz while the API guide documents six planes");
    if (Mx && config_in.coordinate_features != (size_t)Mx)
        fail_unsupported(
            "multidimensional real performConvolution IR supports batch1 independent-coordinate or matrix K=1/K>1 "
            "ownership");
    for (size_t a = 0; a < config_in.omit_dimension.size(); a++)
        if (config_in.omit_dimension[a])
            fail_unsupported(
                "multidimensional real performConvolution currently requires active dimensions without omitDimension");
    if (config_in.has_formatted_strides() &&
        (config_in.coordinate_features != 1 || config_in.convolution_kernel_count != 1 || Mx))
        fail_unsupported("multidimensional real formatted performConvolution currently requires scalar batch1 K1");
    bool padded = false;
    for (auto &z : config_in.zero_padding) padded |= z.has_value();
    if (padded && Mx && config_in.symmetric_convolution_kernel)
        fail_unsupported(
            "multidimensional real performConvolution zero padding requires batch1/K1 nonsymmetric matrix ownership");
    if (config_in.convolution_conjugation == ConvolutionConjugation::Kernel)
        fail_unsupported("kernel-conjugated convolution is not executable in the pinned VkFFT codegen");
    if (!(config_in.precision == Precision::F32 || config_in.precision == Precision::F64))
        fail_precision("B200 engine", precision_name(config_in.precision));
    if (Mx || padded || config_in.has_formatted_strides()) {
        auto conv = build_real_convolution_generic(config_in.resolve_tuning_for_device(device), device, spectrum, copies);
        check_reg_twiddle_tables(conv->prog);
        return conv;
    }
    const FftConfig c = config_in.resolve_tuning_for_device(device);
    auto conv = std::make_unique<Convolution>();
    static std::atomic<uint64_t> next_id{1ull << 40};
    conv->id = next_id++;
    conv->config = c;
    conv->device = device;
    const bool dbl = c.precision == Precision::F64;
    const size_t rank = c.dimensions.size();
    const size_t C = c.coordinate_features, K = c.convolution_kernel_count;
    const size_t W = c.dimensions[rank - 1], half = W / 2 + 1;
    std::vector<size_t> compact = c.dimensions;
    compact[rank - 1] = half;
    const size_t L = prod(compact, 0, rank);        // compact tensor of one system
    const size_t full = prod(c.dimensions, 0, rank);  // real tensor of one system
    if (!(copies == 1 || copies == K * C))
        throw FftError(B200FFT_INPUT_LENGTH_MISMATCH,
                       "input contains " + std::to_string(copies * L) + " complex elements but kernel expects " +
                           std::to_string(K * C * L));
    conv->spectrum_elems = L;
    const bool conj_seq = c.convolution_conjugation == ConvolutionConjugation::Sequence;
    const bool cross = c.cross_power_spectrum_normalization;

    // forward / inverse plans as the reference builds them (convolution_ir.rs:3955-4001)
    FftConfig fc = c;
    fc.perform_convolution = false;
    fc.convolution_conjugation = ConvolutionConjugation::None;
    fc.cross_power_spectrum_normalization = false;
    fc.coordinate_features = 1;
    fc.matrix_convolution = 1;
    fc.symmetric_convolution_kernel = false;
    fc.convolution_kernel_count = 1;
    fc.batch_count = C;
    fc.normalize_inverse = false;
    conv->forward = build_transform(fc, B200FFT_FORWARD, device);
    FftConfig ic = fc;
    ic.transform = TransformKind::C2R;
    ic.batch_count = K * C;
    ic.normalize_inverse = true;
    conv->inverse = build_transform(ic, B200FFT_INVERSE, device);

    Program &prog = conv->prog;
    prog.is_double = dbl;
    prog.input_real = true;
    prog.output_real = true;
    prog.input_elems = conv->logical_in_elems = C * full;
    prog.output_elems = conv->logical_out_elems = K * C * full;
    HostTable st;
    st.is_raw = true;
    const size_t esz = dbl ? 16 : 8;
    st.raw.assign(static_cast<const unsigned char *>(spectrum),
                  static_cast<const unsigned char *>(spectrum) + copies * L * esz);
    prog.tables.push_back(std::move(st));
    const int spec_table = (int)prog.tables.size() - 1;

    const Transform &F = *conv->forward, &I = *conv->inverse;
    const PlannerTuning &tuning = F.plan.config.tuning;
    // forward R2C of the last axis: input -> scratch 1 (compact, C systems)
    prog.scratch_elems[1] = C * L;
    RealAxisJob rj;
    rj.N = W;
    rj.lines = (int64_t)(C * prod(c.dimensions, 0, rank - 1));
    rj.full_complex = F.real_algorithm == RealAlgorithm::FullComplex;
    rj.alg = &F.children[rank - 1]->axes[0].algorithm;
    rj.tuning = tuning;
    rj.in_buf = BUF_IN;
    rj.out_buf = BUF_SCRATCH1;
    lower_r2c_axis(prog, rj);
    auto complex_axis = [&](const Transform &T, size_t a, int64_t systems, bool inverse, int buf) {
        const size_t len = compact[a];
        const size_t inner = prod(compact, a + 1, rank);
        AxisJob job;
        job.N = len;
        job.alg = &T.children[a]->axes[0].algorithm;
        job.tuning = tuning;
        job.no = (int64_t)(systems * prod(compact, 0, a));
        job.S = (int64_t)inner;
        job.inverse = inverse;
        job.scale = inverse ? 1.0 / (double)len : 1.0;
        job.in_buf = job.out_buf = buf;
        job.in_os = job.out_os = (int64_t)(len * inner);
        lower_c2c_axis(prog, job);
    };
    // middle axes forward (rank-2 .. 1)
    for (size_t a = rank - 1; a-- > 1;) complex_axis(F, a, (int64_t)C, false, BUF_SCRATCH1);
    int spec_buf = BUF_SCRATCH1;
    if (K == 1) {
        // fused outermost axis: forward FFT, multiply, normalised inverse FFT
        lower_convolution_axis0(prog, compact[0], &F.children[0]->axes[0].algorithm, tuning, (int64_t)C,
                                (int64_t)prod(compact, 1, rank), BUF_SCRATCH1, spec_table,
                                copies == 1 ? 0 : (int64_t)L, conj_seq, cross, 1.0 / (double)compact[0]);
    } else {
        complex_axis(F, 0, (int64_t)C, false, BUF_SCRATCH1);
        prog.scratch_elems[2] = K * C * L;
        lower_convolution_multiply(prog, (int64_t)L, (int64_t)C, (int64_t)K, BUF_SCRATCH1, BUF_SCRATCH2, spec_table,
                                   (int64_t)copies, conj_seq, cross);
        spec_buf = BUF_SCRATCH2;
        complex_axis(I, 0, (int64_t)(K * C), true, spec_buf);
    }
    // middle axes inverse (1 .. rank-2)
    for (size_t a = 1; a + 1 < rank; a++) complex_axis(I, a, (int64_t)(K * C), true, spec_buf);
    // normalised C2R of the last axis: scratch -> output
    RealAxisJob cj;
    cj.N = W;
    cj.lines = (int64_t)(K * C * prod(c.dimensions, 0, rank - 1));
    cj.normalize = true;
    cj.full_complex = I.real_algorithm == RealAlgorithm::FullComplex;
    cj.alg = &I.children[rank - 1]->axes[0].algorithm;
    cj.tuning = tuning;
    cj.in_buf = spec_buf;
    cj.out_buf = BUF_OUT;
    lower_c2r_axis(prog, cj);
    check_reg_twiddle_tables(prog);
    return conv;
}

}  // namespace b200fft
