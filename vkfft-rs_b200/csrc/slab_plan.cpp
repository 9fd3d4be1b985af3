// Slab decomposition plans (host only): the per-rank launch programs of a slab transform
// (see slab.cu for the data flow and the exchange).
#include <atomic>

#include "slab.hpp"

namespace b200fft {

namespace {

size_t prod(const std::vector<size_t> &v, size_t a, size_t b) {
    size_t r = 1;
    for (size_t i = a; i < b; i++) r = checked_mul(r, v[i], "slab tensor size");
    return r;
}

uint64_t next_slab_id() {  // ids id and id + 1 (the two directions' programs)
    static std::atomic<uint64_t> next{1ull << 41};
    return next.fetch_add(2);
}

// Marks the last pass a lowering appended (it must write the axis output) as the
// exchange pass and records its distance between consecutive logical elements.
void mark_exchange_pass(Program &prog, size_t first, int out_buf) {
    if (prog.passes.size() <= first) fail_runtime("slab lowering produced no exchange pass");
    PassPlan &pp = prog.passes.back();
    if (pp.dst_buf != out_buf || pp.dst_off != 0) fail_runtime("slab exchange pass does not write the axis output");
    pp.peer_scatter = true;
    if (pp.kernel == KERNEL_REG) {
        // from the ordinary variant: a persistent twin has no peer-scatter form, and its
        // misaligned-input fallback must not be the non-scattering kernel
        const int twin = reg_variant_peer_twin(pp.reg_variant_plain >= 0 ? pp.reg_variant_plain : pp.reg_variant);
        if (twin < 0) fail_runtime("slab exchange pass has no peer-scatter register kernel");
        pp.reg_variant = twin;
        pp.reg_variant_plain = -1;
        // the twin may split the line into other radices than the variant the lowering
        // chose, and its stage twiddles follow its own radix sequence
        pp.reg_table = table_reg_twiddles(prog, (size_t)pp.rp.n, twin);
        pp.peer_es = pp.rp.dst.es;
        return;
    }
    const Side &s = pp.p.out;
    if (s.real || s.em <= 0 || s.es % s.em) fail_runtime("slab exchange pass has a non-linear output side");
    const int64_t es_l = s.es / s.em;
    if (s.cs != (int64_t)s.cm * es_l) fail_runtime("slab exchange pass has a non-linear output side");
    pp.peer_es = es_l;
}

}  // namespace

std::unique_ptr<Slab> build_slab(const FftConfig &config_in, int direction, int nranks, int rank,
                                 const DeviceProfile &device) {
    config_in.validate();
    const FftConfig c = config_in.resolve_tuning_for_device(device);
    if (nranks < 1 || nranks > kMaxPeers) fail_unsupported("slab transforms support 1 to 8 ranks");
    if (rank < 0 || rank >= nranks) fail_unsupported("slab rank is out of range");
    if (!(c.precision == Precision::F32 || c.precision == Precision::F64))
        fail_precision("B200 engine", precision_name(c.precision));
    const bool real = c.transform != TransformKind::C2C;
    if (c.transform == TransformKind::R2C && direction != B200FFT_FORWARD)
        fail_unsupported("RealToComplex is a forward transform; use Direction::Forward");
    if (c.transform == TransformKind::C2R && direction != B200FFT_INVERSE)
        fail_unsupported("ComplexToReal is an inverse transform; use Direction::Inverse");
    if (!(c.transform == TransformKind::C2C || real)) fail_unsupported("slab transforms are C2C, R2C or C2R");
    const size_t R = c.dimensions.size();
    if (R < 2 || (real && R < 3)) fail_unsupported("slab transforms need rank >= 2 (C2C) or rank >= 3 (R2C/C2R)");
    if (c.batch_count != 1) fail_unsupported("slab transforms take batch 1");
    for (size_t a = 0; a < R; a++)
        if (c.axis_is_omitted(a)) fail_unsupported("slab transforms transform every axis");
    for (auto &z : c.zero_padding)
        if (z) fail_unsupported("B200 engine: zero padding is not implemented yet");
    if (c.has_formatted_strides()) fail_unsupported("B200 engine: formatted buffer strides are not implemented yet");
    if (c.perform_convolution || c.kernel_convolution) fail_unsupported("slab transforms do not run convolutions");
    const size_t D0 = c.dimensions[0], D1 = c.dimensions[1];
    if (D0 % nranks || D1 % nranks)
        fail_unsupported("slab transforms need the two outermost dimensions divisible by the rank count");

    auto s = std::make_unique<Slab>();
    const uint64_t id = next_slab_id();
    s->id_pre = id;
    s->id_post = id + 1;
    s->config = c;
    s->direction = direction;
    s->nranks = nranks;
    s->rank = rank;
    s->device = device;
    const bool dbl = c.precision == Precision::F64;
    const bool inverse = direction == B200FFT_INVERSE;
    const bool norm = inverse && c.normalize_inverse;
    std::vector<size_t> cd = c.dimensions;  // compact dims
    const size_t W = c.dimensions[R - 1];
    if (real) cd[R - 1] = W / 2 + 1;
    const size_t L0 = D0 / nranks, C1 = D1 / nranks;
    const size_t H = prod(cd, 2, R);
    s->planes_per_rank = L0;
    s->columns_per_rank = C1;
    const size_t slab_complex = checked_mul(L0 * D1, H, "slab element count");
    s->exchange_elems = slab_complex;
    const size_t real_slab = checked_mul(L0, prod(c.dimensions, 1, R), "slab element count");

    // executed child plans per axis, planned for the global tensor as the single-GPU
    // transform plans them
    s->children.assign(R, std::nullopt);
    const size_t global_compact = prod(cd, 0, R);
    for (size_t a = 0; a < R; a++) {
        if (real && a == R - 1) continue;
        FftConfig ac = FftConfig::make({cd[a]});
        ac.batch_count = global_compact / cd[a];
        ac.precision = c.precision;
        ac.normalize_inverse = c.normalize_inverse;
        ac.bandwidth_boost = c.bandwidth_boost;
        ac.with_tuning(c.tuning);
        const size_t inner = prod(cd, a + 1, R);
        s->children[a] =
            FftPlan::build_c2c_child_for_device(ac, device, inner == 1 ? AxisClass::Contiguous : AxisClass::Strided);
    }
    if (real) {
        const size_t lines = prod(c.dimensions, 0, R - 1);
        s->real_algorithm = real_fft_algorithm_for_device(W, lines, c.precision, c.tuning, device);
        FftConfig rc = FftConfig::make({s->real_algorithm == RealAlgorithm::FullComplex ? W : W / 2});
        rc.batch_count = lines;
        rc.precision = c.precision;
        rc.normalize_inverse = inverse && c.normalize_inverse;
        rc.bandwidth_boost = c.bandwidth_boost;
        rc.with_tuning(c.tuning);
        s->children[R - 1] = FftPlan::build_c2c_child_for_device(rc, device, AxisClass::Contiguous);
    }
    auto axis_job = [&](size_t a, int64_t no, int in_buf, int out_buf) {
        AxisJob job;
        job.N = cd[a];
        job.alg = &s->children[a]->axes[0].algorithm;
        job.tuning = c.tuning;
        job.no = no;
        job.S = (int64_t)prod(cd, a + 1, R);
        job.inverse = inverse;
        job.scale = norm ? 1.0 / (double)cd[a] : 1.0;
        job.in_buf = in_buf;
        job.out_buf = out_buf;
        job.in_os = job.out_os = (int64_t)(cd[a] * job.S);
        return job;
    };
    auto real_job = [&](int in_buf, int out_buf) {
        RealAxisJob rj;
        rj.N = W;
        rj.lines = (int64_t)(L0 * prod(c.dimensions, 1, R - 1));
        rj.normalize = norm;
        rj.full_complex = s->real_algorithm == RealAlgorithm::FullComplex;
        rj.alg = &s->children[R - 1]->axes[0].algorithm;
        rj.tuning = c.tuning;
        rj.in_buf = in_buf;
        rj.out_buf = out_buf;
        return rj;
    };
    Program &pre = s->pre, &post = s->post;
    pre.is_double = post.is_double = dbl;
    s->peer.n = nranks;
    if (!inverse) {
        // pre: last axis (R2C or C2C) in -> out, middle axes in place on out, axis 1
        // from out (or in, for rank 2) scattered to the ranks
        bool on_out = false;
        if (R > 2) {
            if (real) {
                lower_r2c_axis(pre, real_job(BUF_IN, BUF_OUT));
            } else {
                lower_c2c_axis(pre, axis_job(R - 1, (int64_t)(L0 * prod(cd, 1, R - 1)), BUF_IN, BUF_OUT));
            }
            on_out = true;
            for (size_t a = R - 2; a >= 2; a--) lower_c2c_axis(pre, axis_job(a, (int64_t)(L0 * prod(cd, 1, a)), BUF_OUT, BUF_OUT));
        }
        AxisJob x = axis_job(1, (int64_t)L0, on_out ? BUF_OUT : BUF_IN, BUF_OUT);
        x.out_os = (int64_t)(C1 * H);  // pencil layout [D0, C1, H] of the owner rank
        const size_t first = pre.passes.size();
        lower_c2c_axis(pre, x);
        mark_exchange_pass(pre, first, BUF_OUT);
        s->peer.chunk = (int32_t)C1;
        s->peer.off = (int64_t)(rank * L0 * C1 * H);
        // post: axis 0 on the pencils [D0, C1, H], exchange (in) -> out
        AxisJob z = axis_job(0, 1, BUF_IN, BUF_OUT);
        z.S = (int64_t)(C1 * H);
        z.in_os = z.out_os = (int64_t)(D0 * C1 * H);
        lower_c2c_axis(post, z);
        pre.input_real = real;
        pre.input_elems = real ? real_slab : slab_complex;
        post.output_elems = slab_complex;
    } else {
        // pre: axis 0 on the pencils [D0, C1, H], in -> the ranks' slabs [L0, D1, H]
        AxisJob z = axis_job(0, 1, BUF_IN, BUF_OUT);
        z.S = (int64_t)(C1 * H);
        z.in_os = (int64_t)(D0 * C1 * H);
        z.out_os = (int64_t)(L0 * D1 * H);
        z.out_S = (int64_t)(D1 * H);
        const size_t first = pre.passes.size();
        lower_c2c_axis(pre, z);
        mark_exchange_pass(pre, first, BUF_OUT);
        s->peer.chunk = (int32_t)L0;
        s->peer.off = (int64_t)(rank * C1 * H);
        // post: axes 1 .. R-2 in place on the exchange buffer, last axis exchange -> out
        for (size_t a = 1; a + 1 < R; a++)
            lower_c2c_axis(post, axis_job(a, (int64_t)(L0 * prod(cd, 1, a)), BUF_IN, BUF_IN));
        if (real) {
            lower_c2r_axis(post, real_job(BUF_IN, BUF_OUT));
        } else {
            lower_c2c_axis(post, axis_job(R - 1, (int64_t)(L0 * prod(cd, 1, R - 1)), BUF_IN, BUF_OUT));
        }
        pre.input_elems = slab_complex;
        post.output_real = real;
        post.output_elems = real ? real_slab : slab_complex;
    }
    s->peer.div = make_fastdiv((uint32_t)s->peer.chunk);
    s->input_elems = pre.input_elems;
    s->output_elems = post.output_elems;
    s->input_real = pre.input_real;
    s->output_real = post.output_real;
    check_reg_twiddle_tables(pre);
    check_reg_twiddle_tables(post);
    return s;
}

Slab::~Slab() { release_slab_device(this); }

size_t Slab::buffer_bytes() const { return ((exchange_elems * (config.precision == Precision::F64 ? 16 : 8)) + 255) & ~size_t(255); }

}  // namespace b200fft
