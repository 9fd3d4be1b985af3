// FFT convolution application: the ND real independent-coordinate path of
// NdRealConvolutionIr (convolution_ir.rs:3867-4250).
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

std::unique_ptr<Convolution> build_convolution(const FftConfig &config_in, const DeviceProfile &device,
                                               const void *spectrum, uint64_t copies) {
    config_in.validate();
    if (!config_in.perform_convolution || config_in.transform != TransformKind::R2C ||
        config_in.dimensions.size() < 2 || config_in.batch_count != 1)
        fail_unsupported(
            "multidimensional real performConvolution IR requires batch1 ND R2C application ownership");
    if (config_in.matrix_convolution > 1)
        fail_unsupported("B200 engine: matrix convolution is not implemented yet");
    if (!(config_in.precision == Precision::F32 || config_in.precision == Precision::F64))
        fail_precision("B200 engine", precision_name(config_in.precision));
    for (auto &z : config_in.zero_padding)
        if (z) fail_unsupported("B200 engine: zero padding is not implemented yet");
    if (config_in.has_formatted_strides()) fail_unsupported("B200 engine: formatted buffer strides are not implemented yet");
    const FftConfig c = config_in.resolve_tuning_for_device(device);
    auto conv = std::make_unique<Convolution>();
    static uint64_t next_id = 1ull << 40;
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
    prog.input_elems = C * full;
    prog.output_elems = K * C * full;
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
    return conv;
}

}  // namespace b200fft
