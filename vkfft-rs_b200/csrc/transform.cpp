// TransformIr::build analogue (application.rs:47-167): resolve device tuning, run the
// device-scored planner, build the per-axis child plans exactly as the reference's IR
// builders do (nd_ir.rs:676-708, real_ir.rs:282-345, nd_real_ir.rs:88-225) and lower the
// executed plans to the B200 launch program.
#include <atomic>
#include <cmath>
#include <cstring>

#include "transform.hpp"

namespace b200fft {

static std::atomic<uint64_t> g_next_id{1};

const char *precision_name(Precision p) {
    switch (p) {
        case Precision::F16StorageF32Compute: return "f16-storage/f32-compute";
        case Precision::F32: return "f32";
        case Precision::F64: return "f64";
        case Precision::F64ComputeF32Storage: return "f64-compute/f32-storage";
        case Precision::DoubleDouble: return "double-double";
        case Precision::DoubleDoubleF64Storage: return "double-double/f64-storage";
    }
    return "unknown";
}

static size_t product(const std::vector<size_t> &v, size_t from, size_t to) {
    size_t acc = 1;
    for (size_t i = from; i < to; i++) acc = checked_mul(acc, v[i], "tensor element count");
    return acc;
}

// Bytes of one compute / stored scalar of a precision (config.rs:107-161 layouts).
static bool compute_is_dd(Precision p) {
    return p == Precision::DoubleDouble || p == Precision::DoubleDoubleF64Storage;
}
static bool compute_is_f64(Precision p) {
    return p == Precision::F64 || p == Precision::F64ComputeF32Storage || compute_is_dd(p);
}
static int storage_scalar_bytes(Precision p) {
    switch (p) {
        case Precision::F16StorageF32Compute: return 2;
        case Precision::F64:
        case Precision::DoubleDoubleF64Storage: return 8;
        case Precision::DoubleDouble: return 16;
        default: return 4;
    }
}

static void check_executable(const FftConfig &) {}

// Double-double programs: every scale of the lowering is the reciprocal of an integer
// k (1/N, 1/M, 1/(2(N-1)), ...), passed as the nearest double; its low word is the
// exact residual (1 - s k) / k, formed with one FMA.
static double dd_scale_residual(double s) {
    if (s == 0.0 || s == 1.0) return 0.0;
    const double k = std::nearbyint(1.0 / s);
    if (k < 1.0 || std::fabs(s * k - 1.0) > 1e-12) return 0.0;
    return std::fma(-s, k, 1.0) / k;
}

static void finalize_dd_scales(Program &prog) {
    if (!prog.is_dd) return;
    for (PassPlan &pp : prog.passes) {
        for (int k = 0; k < pp.p.nops; k++) pp.p.ops[k].scale_lo = dd_scale_residual(pp.p.ops[k].scale);
        pp.rr.scale_lo = dd_scale_residual(pp.rr.scale);
    }
}

static bool is_r2r(TransformKind k) {
    return !(k == TransformKind::C2C || k == TransformKind::R2C || k == TransformKind::C2R);
}

// Effective R2R kind index (0..3 DCT-I..IV, 4..7 DST-I..IV) of a transform and direction:
// inverse_partner (r2r_ir.rs) swaps II and III, the others are their own inverses.
static int r2r_effective_kind(TransformKind k, bool inverse) {
    int kind = 0;
    switch (k) {
        case TransformKind::Dct1: kind = 0; break;
        case TransformKind::Dct2: kind = 1; break;
        case TransformKind::Dct3: kind = 2; break;
        case TransformKind::Dct4: kind = 3; break;
        case TransformKind::Dst1: kind = 4; break;
        case TransformKind::Dst2: kind = 5; break;
        case TransformKind::Dst3: kind = 6; break;
        default: kind = 7; break;
    }
    if (inverse && ((kind & 3) == 1 || (kind & 3) == 2)) kind ^= 3;
    return kind;
}

// inverse_pair_scale (r2r_ir.rs): 1/(2(N-1)) for DCT-I, 1/(2(N+1)) for DST-I, 1/(2N) otherwise.
static double r2r_inverse_pair_scale(TransformKind k, size_t n) {
    if (k == TransformKind::Dct1) return 1.0 / (2.0 * (double)(n - 1));
    if (k == TransformKind::Dst1) return 1.0 / (2.0 * (double)(n + 1));
    return 1.0 / (2.0 * (double)n);
}

// r2r_fft_reduction_expected_len (r2r_ir.rs:355-385) and the FFT direction of each
// reduction (r2r_ir.rs:705-716, 819, 916): III and even IV run the inverse FFT.
static size_t r2r_fft_len(int kind, size_t n) {
    switch (kind & 3) {
        case 0: return kind == 0 ? checked_mul(n - 1, 2, "DCT-I FFT reduction length")
                                 : checked_mul(n + 1, 2, "DST-I FFT reduction length");
        case 3: return n % 2 == 0 ? n / 2 : checked_mul(n, 2, "odd DCT/DST-IV FFT reduction length");
        default: return n;
    }
}
static bool r2r_fft_inverse(int kind, size_t n) { return (kind & 3) == 2 || ((kind & 3) == 3 && n % 2 == 0); }

static std::vector<int64_t> dense_strides(const std::vector<size_t> &dims) {
    std::vector<int64_t> st(dims.size(), 1);
    for (size_t a = dims.size() - 1; a-- > 0;) st[a] = st[a + 1] * (int64_t)dims[a + 1];
    return st;
}

// Zero padding (zero_pad_ir.rs) and formatted buffer strides (config.rs:893-1002,
// nd_ir.rs:1190-1260) at the transform's boundary: the lowered program reads a dense
// scratch copy of the input gathered from the caller's buffer (padding of the input
// boundary applied) and/or writes a dense scratch result scattered to the caller's
// buffer (padding of the output boundary applied).  Spatial padding owns the forward
// input / inverse output, frequency padding the forward output / inverse input; real
// transforms pad their real side.
static void add_boundaries(Transform &t) {
    const FftConfig &c = t.plan.config;
    Program &prog = t.prog;
    const bool r2c = c.transform == TransformKind::R2C, c2r = c.transform == TransformKind::C2R;
    const bool r2r = is_r2r(c.transform);
    const bool inverse = t.direction == B200FFT_INVERSE;
    std::vector<size_t> compact = c.dimensions;
    compact.back() = compact.back() / 2 + 1;
    const std::vector<size_t> &in_dims = c2r ? compact : c.dimensions;
    const std::vector<size_t> &out_dims = r2c ? compact : c.dimensions;
    bool any_pad = false;
    for (auto &z : c.zero_padding) any_pad |= z.has_value();
    bool pad_in = false, pad_out = false;
    if (any_pad) {
        if (r2r)  // spatial masking of the forward input / inverse output (r2r_ir.rs:1241-1277)
            (inverse ? pad_out : pad_in) = true;
        else if (r2c || c2r)
            (r2c ? pad_in : pad_out) = true;
        else
            ((c.zero_padding_domain == ZeroPaddingDomain::Spatial) != inverse ? pad_in : pad_out) = true;
    }
    bool fmt_in = c.input_buffer_batch_stride.has_value(), fmt_out = c.output_buffer_batch_stride.has_value();
    for (auto &v : c.input_buffer_axis_strides) fmt_in |= v.has_value();
    for (auto &v : c.output_buffer_axis_strides) fmt_out |= v.has_value();
    t.logical_in_elems = prog.input_elems;
    t.logical_out_elems = prog.output_elems;
    t.formatted = fmt_in || fmt_out;
    // mixed precision (F16 storage / F32 compute, F64 compute / F32 storage): the caller's
    // buffers hold the storage type, converted at the boundary copies
    const int sbytes = storage_scalar_bytes(c.precision), cbytes = prog.rbytes();
    const bool mixed = sbytes != cbytes;
    if (mixed) prog.storage_scalar_bytes = sbytes;
    if (!pad_in && !pad_out && !fmt_in && !fmt_out && !mixed) return;
    if (c.dimensions.size() > (size_t)kMaxCopyRank) fail_unsupported("boundary copies support rank <= 8");
    const size_t batch = c.kernel_preparation_system_count();
    const size_t esz = (size_t)prog.cbytes();
    auto copy = [&](const std::vector<size_t> &dims, bool input, bool pad, size_t elem_bytes, int src, int dst) {
        PassPlan pp{};
        pp.kernel = KERNEL_COPY;
        BoundaryCopy &b = pp.bc;
        const std::vector<size_t> fst = c.resolved_axis_strides(dims, input);
        const size_t fbatch = c.resolved_batch_stride(dims, input);
        const std::vector<int64_t> dst_dense = dense_strides(dims);
        size_t tensor = 1;
        for (size_t d : dims) tensor *= d;
        b.total = (int64_t)(tensor * batch);
        b.rank = (int32_t)dims.size();
        b.scalars = (int32_t)(elem_bytes / (size_t)cbytes);
        b.src_bytes = input ? sbytes : cbytes;
        b.dst_bytes = input ? cbytes : sbytes;
        for (size_t a = 0; a < dims.size(); a++) {
            b.dims[a] = (int64_t)dims[a];
            const int64_t formatted = (int64_t)fst[a], dense = dst_dense[a];
            b.src_stride[a] = input ? formatted : dense;
            b.dst_stride[a] = input ? dense : formatted;
            b.pad_lo[a] = b.pad_hi[a] = 0;
            if (pad && c.zero_padding[a]) {
                b.pad_lo[a] = (int64_t)c.zero_padding[a]->left;
                b.pad_hi[a] = (int64_t)c.zero_padding[a]->right;
            }
        }
        b.src_batch = input ? (int64_t)fbatch : (int64_t)tensor;
        b.dst_batch = input ? (int64_t)tensor : (int64_t)fbatch;
        pp.src_buf = src;
        pp.dst_buf = dst;
        pp.label = input ? "boundary gather" : "boundary scatter";
        for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
        return std::make_pair(pp, fbatch * batch);
    };
    if (pad_in || fmt_in || mixed) {
        const size_t eb = (r2c || r2r) ? esz / 2 : esz;
        for (PassPlan &pp : prog.passes)
            if (pp.src_buf == BUF_IN) pp.src_buf = BUF_SCRATCH4;
        auto [pp, physical] = copy(in_dims, true, pad_in, eb, BUF_IN, BUF_SCRATCH4);
        prog.scratch_elems[4] = (prog.input_elems * eb + esz - 1) / esz;
        prog.passes.insert(prog.passes.begin(), pp);
        prog.input_elems = physical;
    }
    if (pad_out || fmt_out || mixed) {
        const size_t eb = (c2r || r2r) ? esz / 2 : esz;
        for (PassPlan &pp : prog.passes) {
            if (pp.src_buf == BUF_OUT) pp.src_buf = BUF_SCRATCH5;
            if (pp.dst_buf == BUF_OUT) pp.dst_buf = BUF_SCRATCH5;
        }
        auto [pp, physical] = copy(out_dims, false, pad_out, eb, BUF_SCRATCH5, BUF_OUT);
        prog.scratch_elems[5] = (prog.output_elems * eb + esz - 1) / esz;
        prog.passes.push_back(pp);
        prog.output_elems = physical;
    }
}

static std::unique_ptr<Transform> build_transform_core(const FftConfig &config_in, int direction,
                                                       const DeviceProfile &device);

std::unique_ptr<Transform> build_transform(const FftConfig &config_in, int direction, const DeviceProfile &device) {
    auto t = build_transform_core(config_in, direction, device);
    add_boundaries(*t);
    finalize_dd_scales(t->prog);
    check_reg_twiddle_tables(t->prog);
    return t;
}

static std::unique_ptr<Transform> build_transform_core(const FftConfig &config_in, int direction,
                                                       const DeviceProfile &device) {
    if (config_in.transform == TransformKind::R2C && direction != B200FFT_FORWARD)
        fail_unsupported("RealToComplex is a forward transform; use Direction::Forward");
    if (config_in.transform == TransformKind::C2R && direction != B200FFT_INVERSE)
        fail_unsupported("ComplexToReal is an inverse transform; use Direction::Inverse");
    auto t = std::make_unique<Transform>();
    t->id = g_next_id++;
    t->direction = direction;
    t->device = device;
    t->config = config_in.resolve_tuning_for_device(device);
    t->plan = FftPlan::build_for_device(t->config, device);
    const FftConfig &c = t->plan.config;
    check_executable(c);
    const bool inverse = direction == B200FFT_INVERSE;
    const size_t rank = c.dimensions.size();
    const size_t batch = c.kernel_preparation_system_count();
    t->children.assign(rank, std::nullopt);
    Program &prog = t->prog;
    prog.is_double = compute_is_f64(c.precision);
    prog.is_dd = compute_is_dd(c.precision);

    if (c.transform == TransformKind::C2C) {
        const size_t tensor = product(c.dimensions, 0, rank);
        prog.input_elems = prog.output_elems = checked_mul(tensor, batch, "transform element count");
        if (rank == 1) {
            t->family = B200FFT_FAMILY_COMPLEX_1D;
            t->children[0] = t->plan;
            const size_t n = c.dimensions[0];
            AxisJob job;
            job.N = n;
            job.alg = &t->children[0]->axes[0].algorithm;
            job.no = (int64_t)batch;
            job.S = 1;
            job.inverse = inverse;
            job.scale = (inverse && c.normalize_inverse) ? 1.0 / (double)n : 1.0;
            job.in_os = job.out_os = (int64_t)n;
            job.tuning = c.tuning;
            lower_c2c_axis(prog, job);
            return t;
        }
        t->family = B200FFT_FAMILY_COMPLEX_ND;
        bool first = true;
        for (size_t a = rank; a-- > 0;) {
            if (c.axis_is_omitted(a)) continue;
            const size_t len = c.dimensions[a];
            const size_t inner = product(c.dimensions, a + 1, rank);
            const size_t lines = tensor / len;
            FftConfig ac = FftConfig::make({len});
            ac.batch_count = checked_mul(batch, lines, "multidimensional recursive transform batch count");
            ac.precision = c.precision;
            ac.normalize_inverse = c.normalize_inverse;
            ac.bandwidth_boost = c.bandwidth_boost;
            ac.with_tuning(c.tuning);
            if (auto gb = c.grouped_batch_for_axis(a)) ac.grouped_batch[0] = gb;
            t->children[a] = FftPlan::build_c2c_child_for_device(ac, device,
                                                                 inner == 1 ? AxisClass::Contiguous : AxisClass::Strided);
            AxisJob job;
            job.N = len;
            job.alg = &t->children[a]->axes[0].algorithm;
            job.no = (int64_t)(batch * product(c.dimensions, 0, a));
            job.S = (int64_t)inner;
            job.inverse = inverse;
            job.scale = (inverse && c.normalize_inverse) ? 1.0 / (double)len : 1.0;
            job.in_buf = first ? BUF_IN : BUF_OUT;
            job.out_buf = BUF_OUT;
            job.in_os = job.out_os = (int64_t)(len * inner);
            job.tuning = c.tuning;
            lower_c2c_axis(prog, job);
            first = false;
        }
        return t;
    }

    if (is_r2r(c.transform)) {
        // DCT / DST (application.rs:134-165): R2rIr for rank 1, NdR2rIr (r2r_ir.rs:1795-2017)
        // otherwise, one FFT reduction per non-omitted axis from the last to the first.
        // Each axis runs pre pass (tensor -> complex work array [outer][L][inner]),
        // the internal FFT as a strided (or, for the last axis, contiguous) axis of the
        // work array, and post pass (work array -> tensor); the first axis reads the
        // input, every post pass writes the output.
        const size_t tensor = product(c.dimensions, 0, rank);
        prog.input_elems = prog.output_elems = checked_mul(tensor, batch, "DCT/DST element count");
        prog.input_real = prog.output_real = true;
        t->family = rank == 1 ? B200FFT_FAMILY_REAL_TO_REAL : B200FFT_FAMILY_REAL_TO_REAL_ND;
        bool first = true;
        for (size_t a = rank; a-- > 0;) {
            if (c.axis_is_omitted(a)) continue;
            const size_t n = c.dimensions[a];
            if (c.transform == TransformKind::Dct1 && n < 2)
                throw FftError(B200FFT_INVALID_TRANSFORM_LENGTH,
                               "axis " + std::to_string(a) + " length " + std::to_string(n) + " is invalid for DCT-I");
            const size_t inner = product(c.dimensions, a + 1, rank);
            const size_t outer = checked_mul(batch, product(c.dimensions, 0, a), "DCT/DST axis batch count");
            const int kind = r2r_effective_kind(c.transform, inverse);
            const size_t L = r2r_fft_len(kind, n);
            const double scale = (inverse && c.normalize_inverse) ? r2r_inverse_pair_scale(c.transform, n) : 1.0;
            FftConfig ac = FftConfig::make({L});
            ac.batch_count = checked_mul(outer, inner, "DCT/DST internal FFT batch count");
            ac.precision = c.precision == Precision::F16StorageF32Compute ? Precision::F32
                           : c.precision == Precision::F64ComputeF32Storage ? Precision::F64
                                                                            : c.precision;
            ac.normalize_inverse = false;
            ac.bandwidth_boost = c.bandwidth_boost;
            ac.with_tuning(c.tuning);
            if (auto gb = c.grouped_batch_for_axis(a)) ac.grouped_batch[0] = gb;
            t->children[a] = FftPlan::build_c2c_child_for_device(ac, device,
                                                                 inner == 1 ? AxisClass::Contiguous : AxisClass::Strided);
            {
                R2rAxisJob rj;
                rj.n = n;
                rj.L = L;
                rj.kind = kind;
                rj.fft_inverse = r2r_fft_inverse(kind, n);
                rj.alg = &t->children[a]->axes[0].algorithm;
                rj.outer = (int64_t)outer;
                rj.inner = (int64_t)inner;
                rj.scale = scale;
                rj.in_buf = first ? BUF_IN : BUF_OUT;
                rj.out_buf = BUF_OUT;
                if (lower_r2r_axis_register(prog, rj)) {
                    first = false;
                    continue;
                }
            }
            const size_t work = checked_mul(checked_mul(outer, L, "DCT/DST work array"), inner, "DCT/DST work array");
            prog.scratch_elems[1] = std::max(prog.scratch_elems[1], work);
            auto r2r_pass = [&](bool pre) {
                PassPlan pp{};
                pp.kernel = KERNEL_R2R;
                R2rPass &r = pp.rr;
                r.outer = (int64_t)outer;
                r.inner = (int64_t)inner;
                r.n = (int64_t)n;
                r.L = (int64_t)L;
                r.total = (int64_t)(outer * (pre ? L : n) * inner);
                r.kind = kind;
                r.pre = pre ? 1 : 0;
                r.scale = scale;
                if ((kind & 3) != 0) pp.reg_table2 = table_r2r(prog, kind & 3, n, L);
                pp.src_buf = pre ? (first ? BUF_IN : BUF_OUT) : BUF_SCRATCH1;
                pp.dst_buf = pre ? BUF_SCRATCH1 : BUF_OUT;
                pp.label = pre ? "r2r pre-process" : "r2r post-process";
                for (auto &row : pp.op_tables) row[0] = row[1] = row[2] = -1;
                prog.passes.push_back(pp);
            };
            r2r_pass(true);
            AxisJob job;
            job.N = L;
            job.alg = &t->children[a]->axes[0].algorithm;
            job.no = (int64_t)outer;
            job.S = (int64_t)inner;
            job.inverse = r2r_fft_inverse(kind, n);
            job.scale = 1.0;
            job.in_buf = job.out_buf = BUF_SCRATCH1;
            job.in_os = job.out_os = (int64_t)(L * inner);
            job.tuning = c.tuning;
            lower_c2c_axis(prog, job);
            r2r_pass(false);
            first = false;
        }
        return t;
    }

    // Real transforms
    const bool r2c = c.transform == TransformKind::R2C;
    const size_t n = c.dimensions[rank - 1];
    const size_t half = n / 2 + 1;
    const size_t outer = product(c.dimensions, 0, rank - 1);
    const size_t lines = checked_mul(batch, outer, "multidimensional real FFT last-axis batch count");
    // The real axis child: RealFftIr::build_for_device_plan / build_with_shape_policy
    // (real_ir.rs:282-345); the ND builder plans it portably first (nd_real_ir.rs:118-131).
    t->real_algorithm = real_fft_algorithm_for_device(n, lines, c.precision, c.tuning, device);
    t->real_transform_len = t->real_algorithm == RealAlgorithm::FullComplex ? n : n / 2;
    {
        FftConfig rc = FftConfig::make({t->real_transform_len});
        rc.batch_count = lines;
        rc.precision = c.precision;
        rc.normalize_inverse = !r2c && c.normalize_inverse;
        rc.bandwidth_boost = c.bandwidth_boost;
        rc.with_tuning(c.tuning);
        t->children[rank - 1] = FftPlan::build_c2c_child_for_device(rc, device, AxisClass::Contiguous);
    }
    const size_t full_tensor = checked_mul(outer * n, batch, "real tensor element count");
    const size_t compact_tensor = checked_mul(outer * half, batch, "compact tensor element count");
    prog.input_real = r2c;
    prog.output_real = !r2c;
    prog.input_elems = r2c ? full_tensor : compact_tensor;
    prog.output_elems = r2c ? compact_tensor : full_tensor;
    std::vector<size_t> compact = c.dimensions;
    compact[rank - 1] = half;
    RealAxisJob rj;
    rj.N = n;
    rj.lines = (int64_t)lines;
    rj.normalize = !r2c && c.normalize_inverse;
    rj.full_complex = t->real_algorithm == RealAlgorithm::FullComplex;
    rj.alg = &t->children[rank - 1]->axes[0].algorithm;
    rj.tuning = c.tuning;

    t->family = rank == 1 ? B200FFT_FAMILY_REAL : B200FFT_FAMILY_REAL_ND;
    // complex axes on the compact tensor (always strided: the real axis is the last one)
    std::vector<size_t> caxes;
    for (size_t a = rank - 1; a-- > 0;)
        if (!c.axis_is_omitted(a)) caxes.push_back(a);
    for (size_t a : caxes) {
        const size_t len = compact[a];
        const size_t inner = product(compact, a + 1, rank);
        const size_t clines = product(compact, 0, rank) / len;
        FftConfig ac = FftConfig::make({len});
        ac.batch_count = checked_mul(batch, clines, "multidimensional real FFT complex-axis batch count");
        ac.precision = c.precision;
        ac.normalize_inverse = !r2c && c.normalize_inverse;
        ac.bandwidth_boost = c.bandwidth_boost;
        ac.with_tuning(c.tuning);
        t->children[a] = FftPlan::build_c2c_child_for_device(ac, device, AxisClass::Strided);
    }
    auto complex_axis = [&](size_t a, int in_buf, int out_buf) {
        const size_t len = compact[a];
        const size_t inner = product(compact, a + 1, rank);
        AxisJob job;
        job.N = len;
        job.alg = &t->children[a]->axes[0].algorithm;
        job.no = (int64_t)(batch * product(compact, 0, a));
        job.S = (int64_t)inner;
        job.inverse = !r2c;
        job.scale = (!r2c && c.normalize_inverse) ? 1.0 / (double)len : 1.0;
        job.in_buf = in_buf;
        job.out_buf = out_buf;
        job.in_os = job.out_os = (int64_t)(len * inner);
        job.tuning = c.tuning;
        lower_c2c_axis(prog, job);
    };
    if (r2c) {
        rj.in_buf = BUF_IN;
        rj.out_buf = BUF_OUT;
        lower_r2c_axis(prog, rj);
        for (size_t a : caxes) complex_axis(a, BUF_OUT, BUF_OUT);
    } else {
        if (caxes.empty()) {
            rj.in_buf = BUF_IN;
        } else {
            // inverse complex axes on a scratch copy of the compact input (copy semantics)
            prog.scratch_elems[1] = compact_tensor;
            bool first = true;
            for (size_t k = caxes.size(); k-- > 0;) {
                complex_axis(caxes[k], first ? BUF_IN : BUF_SCRATCH1, BUF_SCRATCH1);
                first = false;
            }
            rj.in_buf = BUF_SCRATCH1;
        }
        rj.out_buf = BUF_OUT;
        lower_c2r_axis(prog, rj);
    }
    return t;
}

}  // namespace b200fft
