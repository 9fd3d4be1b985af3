// Per-axis algorithm planner: Stockham / Rader / Bluestein selection.
//
// Restates vkfft-rs src/planner.rs (and the parts of src/scheduler.rs and
// src/real_ir.rs that change algorithm selection) so that every plan decision is
// bit-identical to the reference planner: same factorisation, same Rader gates
// and shared-memory reservations, same Bluestein padding tables and search.
// Block/register geometry of the reference's scheduler is not ported: the B200
// kernels choose their own tiling (see lower.cpp).
#include <algorithm>
#include <cstring>

#include "core.hpp"

namespace b200fft {

static const size_t STOCKHAM_PRIMES[] = {2, 3, 5, 7, 11, 13};                    // planner.rs:10
static const size_t DOUBLE_DOUBLE_STOCKHAM_PRIMES[] = {2, 3, 5, 7};              // planner.rs:11
static const size_t MERGED_RADICES[] = {32, 16, 15, 14, 12, 10, 9, 8, 6, 4};     // planner.rs:14
static const std::vector<size_t> BLUESTEIN_SMOOTH_PRIMES = {2, 3, 5, 7};         // planner.rs:17

// ---- planner.rs:581-733 ---------------------------------------------------

std::vector<size_t> prime_factorization(size_t value) {
    std::vector<size_t> f;
    if (value < 2) return f;
    while (value % 2 == 0) {
        f.push_back(2);
        value /= 2;
    }
    size_t d = 3;
    while (d <= value / d) {
        while (value % d == 0) {
            f.push_back(d);
            value /= d;
        }
        d += 2;
    }
    if (value > 1) f.push_back(value);
    return f;
}

bool is_smooth(size_t value, const std::vector<size_t> &primes) {
    if (value == 0) return false;
    for (size_t p : primes)
        while (value % p == 0) value /= p;
    return value == 1;
}

std::vector<size_t> merged_radix_schedule(size_t value) {
    std::vector<size_t> stages;
    if (value <= 1) return stages;
    static const size_t FALLBACK[] = {13, 11, 7, 5, 3, 2};
    while (value > 1) {
        size_t selected = 0;
        for (size_t r : MERGED_RADICES)
            if (value % r == 0) {
                selected = r;
                break;
            }
        if (!selected)
            for (size_t r : FALLBACK)
                if (value % r == 0) {
                    selected = r;
                    break;
                }
        if (!selected) break;
        stages.push_back(selected);
        value /= selected;
    }
    return stages;
}

static size_t mod_pow(size_t base, size_t exponent, size_t modulus) {
    unsigned __int128 result = 1, b = base % modulus, m = modulus;
    while (exponent > 0) {
        if (exponent & 1) result = (result * b) % m;
        b = (b * b) % m;
        exponent >>= 1;
    }
    return static_cast<size_t>(result);
}

size_t primitive_root(size_t prime) {
    if (prime == 2) return 1;
    if (prime < 2 || prime_factorization(prime).size() != 1) return 0;
    size_t phi = prime - 1;
    auto uf = prime_factorization(phi);
    uf.erase(std::unique(uf.begin(), uf.end()), uf.end());
    for (size_t g = 2; g < prime; g++) {
        bool ok = true;
        for (size_t f : uf)
            if (mod_pow(g, phi / f, prime) == 1) {
                ok = false;
                break;
            }
        if (ok) return g;
    }
    return 0;
}

static void smooth_visit(const std::vector<size_t> &primes, size_t index, size_t current, size_t target, size_t &best) {
    if (current >= best) return;
    if (index == primes.size()) {
        if (current >= target) best = current;
        return;
    }
    size_t prime = primes[index];
    size_t value = current;
    for (;;) {
        smooth_visit(primes, index + 1, value, target, best);
        size_t next;
        if (__builtin_mul_overflow(value, prime, &next) || next >= best) break;
        value = next;
    }
}

size_t next_smooth_at_least(size_t target, const std::vector<size_t> &primes_in) {
    if (target <= 1) return 1;
    if (primes_in.empty() || std::any_of(primes_in.begin(), primes_in.end(), [](size_t p) { return p < 2; }))
        fail_tuning("smooth-number prime set must contain values >= 2");
    std::vector<size_t> ordered = primes_in;
    std::sort(ordered.begin(), ordered.end());
    ordered.erase(std::unique(ordered.begin(), ordered.end()), ordered.end());
    size_t best = SIZE_MAX;
    if (std::binary_search(ordered.begin(), ordered.end(), (size_t)2)) {
        size_t p = 1;
        while (p < target && p <= (SIZE_MAX >> 1)) p <<= 1;
        best = p >= target ? p : SIZE_MAX;
    }
    smooth_visit(ordered, 0, 1, target, best);
    if (best == SIZE_MAX) fail_overflow("smooth convolution length");
    return best;
}

static size_t checked_product(const std::vector<size_t> &v, const char *op) {
    size_t acc = 1;
    for (size_t x : v) acc = checked_mul(acc, x, op);
    return acc;
}

// ---- planner.rs:244-276 ---------------------------------------------------

static size_t effective_axis_len(TransformKind t, size_t len, size_t axis) {
    switch (t) {
        case TransformKind::Dct1:
            if (len > SIZE_MAX / 2 || len * 2 < 2) fail_overflow("DCT-I effective FFT length");
            return len * 2 - 2;
        case TransformKind::Dst1:
            if (len > (SIZE_MAX - 2) / 2) fail_overflow("DST-I effective FFT length");
            return len * 2 + 2;
        case TransformKind::Dct4:
        case TransformKind::Dst4:
            if (len % 2 == 0) {
                if (len / 2 == 0)
                    throw FftError(B200FFT_INVALID_TRANSFORM_LENGTH, "axis " + std::to_string(axis) + " length " +
                                                                          std::to_string(len) +
                                                                          " is invalid for DCT/DST-IV");
                return len / 2;
            }
            return len;
        default: return len;
    }
}

// ---- Rader gates (planner.rs:465-529) -------------------------------------

static bool in_list(size_t v, const size_t *list, size_t n) {
    for (size_t i = 0; i < n; i++)
        if (list[i] == v) return true;
    return false;
}

static bool rader_fft_passes_upstream_safe_prime_gate(size_t prime, const PlannerTuning &t) {
    if (prime <= 2) return false;
    for (size_t f : prime_factorization(prime - 1))
        if (f >= t.min_rader_direct_prime) return false;
    return true;
}

static RaderPrimePlan rader_fft_mode(size_t prime) {
    RaderPrimePlan r;
    r.prime = prime;
    r.fft_convolution = true;
    r.convolution.prime_factors = prime_factorization(prime - 1);
    r.convolution.merged_radices = merged_radix_schedule(prime - 1);
    return r;
}

static RaderPrimePlan rader_direct_mode(size_t prime) {
    RaderPrimePlan r;
    r.prime = prime;
    r.fft_convolution = false;
    return r;
}

static bool rader_mode_with_stockham_primes(size_t prime, const PlannerTuning &t, const size_t *sp, size_t nsp,
                                            RaderPrimePlan *out);

static bool rader_convolution_is_recursively_plannable(size_t len, const PlannerTuning &t, const size_t *sp,
                                                       size_t nsp) {
    for (size_t p : prime_factorization(len)) {
        if (in_list(p, sp, nsp)) continue;
        if (!rader_mode_with_stockham_primes(p, t, sp, nsp, nullptr)) return false;
    }
    return true;
}

// planner.rs:479-510
static bool rader_mode_with_stockham_primes(size_t prime, const PlannerTuning &t, const size_t *sp, size_t nsp,
                                            RaderPrimePlan *out) {
    bool fft_eligible = prime >= t.min_rader_fft_prime && prime < t.max_rader_fft_prime;
    if (fft_eligible && rader_fft_passes_upstream_safe_prime_gate(prime, t)) {
        if (out) *out = rader_fft_mode(prime);
        return true;
    }
    if (prime >= t.min_rader_direct_prime && prime < t.max_rader_direct_prime) {
        if (out) *out = rader_direct_mode(prime);
        return true;
    }
    if (t.allow_recursive_fft_rader && fft_eligible &&
        rader_convolution_is_recursively_plannable(prime - 1, t, sp, nsp)) {
        if (out) *out = rader_fft_mode(prime);
        return true;
    }
    return false;
}

// planner.rs:531-548
static AxisAlgorithm plan_bluestein(size_t len) {
    if (len > SIZE_MAX / 2 || len * 2 < 1) fail_overflow("Bluestein minimum convolution length");
    size_t m = next_smooth_at_least(len * 2 - 1, BLUESTEIN_SMOOTH_PRIMES);
    AxisAlgorithm a;
    a.kind = AlgorithmKind::Bluestein;
    a.convolution_len = m;
    a.radix.merged_radices = merged_radix_schedule(m);
    a.radix.prime_factors = prime_factorization(m);
    return a;
}

// planner.rs:282-347.  select returns: 1 = Rader mode chosen (filled), 0 = fall back
// to Bluestein.
template <typename Select>
static AxisAlgorithm plan_axis_algorithm_with_rader_selector(size_t len, const PlannerTuning &tuning,
                                                             const size_t *sp, size_t nsp, Select select) {
    tuning.validate();
    if (len == 0) throw FftError(B200FFT_ZERO_LENGTH, "FFT axis 0 has zero length");
    AxisAlgorithm a;
    if (len == 1) {
        a.kind = AlgorithmKind::Stockham;
        return a;
    }
    auto factors = prime_factorization(len);
    std::vector<size_t> stockham_factors;
    std::vector<RaderPrimePlan> rader;
    size_t cursor = 0;
    while (cursor < factors.size()) {
        size_t prime = factors[cursor];
        size_t mult = 1;
        while (cursor + mult < factors.size() && factors[cursor + mult] == prime) mult++;
        if (in_list(prime, sp, nsp)) {
            for (size_t i = 0; i < mult; i++) stockham_factors.push_back(prime);
        } else {
            RaderPrimePlan r;
            if (select(prime, r)) {
                r.prime = prime;
                r.multiplicity = mult;
                r.generator = primitive_root(prime);
                rader.push_back(r);
            } else {
                return plan_bluestein(len);
            }
        }
        cursor += mult;
    }
    size_t stockham_len = checked_product(stockham_factors, "Stockham radix product");
    a.radix.prime_factors = stockham_factors;
    a.radix.merged_radices = merged_radix_schedule(stockham_len);
    if (rader.empty()) {
        a.kind = AlgorithmKind::Stockham;
    } else {
        a.kind = AlgorithmKind::Rader;
        a.primes = rader;
    }
    return a;
}

AxisAlgorithm plan_axis_algorithm(size_t len, const PlannerTuning &tuning) {
    return plan_axis_algorithm_with_rader_selector(len, tuning, STOCKHAM_PRIMES, 6, [&](size_t prime, RaderPrimePlan &r) {
        return rader_mode_with_stockham_primes(prime, tuning, STOCKHAM_PRIMES, 6, &r);
    });
}

// planner.rs:442-463
static size_t c2c_rader_fft_shared_limit(size_t available, size_t fft_len, AxisClass cls, size_t complex_bytes,
                                         size_t coalesced_bytes, size_t configured) {
    size_t shared = available / complex_bytes;
    size_t strided = coalesced_bytes > complex_bytes ? available / coalesced_bytes : shared;
    size_t device_limit = (cls == AxisClass::Contiguous && fft_len <= shared) ? shared : strided;
    return std::min(device_limit, configured);
}

// planner.rs:349-440
static AxisAlgorithm plan_c2c_axis_algorithm_for_device(size_t len, size_t batch_count, const PlannerTuning &tuning,
                                                        Precision precision, AxisClass cls, const DeviceProfile &d) {
    size_t complex_bytes = compute_complex_bytes(precision);
    size_t coalesced = upstream_coalesced_memory_bytes_for_precision(d, precision);
    size_t used_shared = is_pow2(len) ? d.shared_memory_pow2_bytes : d.shared_memory_bytes;
    size_t fft_rader_limit =
        c2c_rader_fft_shared_limit(used_shared, len, cls, complex_bytes, coalesced, tuning.max_rader_fft_prime);
    PlannerTuning effective = upstream_effective_rader_tuning(tuning, d, precision);
    size_t direct_limit = effective.max_rader_direct_prime;
    const size_t *sp = is_double_double(precision) ? DOUBLE_DOUBLE_STOCKHAM_PRIMES : STOCKHAM_PRIMES;
    size_t nsp = is_double_double(precision) ? 4 : 6;

    AxisAlgorithm a = plan_axis_algorithm_with_rader_selector(len, tuning, sp, nsp, [&](size_t prime, RaderPrimePlan &r) {
        bool in_fft_scan =
            prime >= tuning.min_rader_direct_prime && prime >= tuning.min_rader_fft_prime && prime < fft_rader_limit;
        if (in_fft_scan) {
            if (rader_fft_passes_upstream_safe_prime_gate(prime, tuning)) {
                r = rader_fft_mode(prime);
                return true;
            }
            size_t reservation = checked_mul(prime - 1, complex_bytes,
                                             "device-scored direct Rader shared-memory reservation");
            size_t avail = used_shared > reservation ? used_shared - reservation : 0;  // saturating_sub
            fft_rader_limit =
                c2c_rader_fft_shared_limit(avail, len, cls, complex_bytes, coalesced, tuning.max_rader_fft_prime);
        }
        if (prime >= tuning.min_rader_direct_prime && prime < direct_limit) {
            r = rader_direct_mode(prime);
            return true;
        }
        bool fft_eligible = prime >= tuning.min_rader_fft_prime && prime < tuning.max_rader_fft_prime;
        if (tuning.allow_recursive_fft_rader && fft_eligible &&
            rader_convolution_is_recursively_plannable(prime - 1, effective, sp, nsp)) {
            r = rader_fft_mode(prime);
            return true;
        }
        return false;
    });
    if (a.kind == AlgorithmKind::Bluestein) {
        size_t m = upstream_bluestein_auto_padding(len, batch_count, precision, d);
        a.convolution_len = m;
        a.radix.prime_factors = prime_factorization(m);
        a.radix.merged_radices = merged_radix_schedule(m);
    }
    return a;
}

// planner.rs:550-579
static size_t scratch_estimate(const AxisAlgorithm &a) {
    switch (a.kind) {
        case AlgorithmKind::Stockham: return 0;
        case AlgorithmKind::Rader: {
            size_t total = 0;
            for (auto &p : a.primes)
                total = checked_add(total, checked_mul(p.prime - 1, p.multiplicity, "Rader scratch estimate"),
                                    "Rader scratch estimate");
            return total;
        }
        case AlgorithmKind::Bluestein: return checked_mul(a.convolution_len, 3, "Bluestein scratch estimate");
    }
    return 0;
}

// planner.rs:168-242
static FftPlan build_inner(const FftConfig &config, const DeviceProfile *device, int cls_override) {
    config.validate();
    if (config.perform_convolution)
        fail_unsupported(
            "performConvolution is an application pipeline; build ConvolutionIr instead of a plain FftPlan");
    size_t exec_batch = config.kernel_preparation_system_count();
    FftPlan plan;
    plan.config = config;
    plan.axis_class_override = cls_override;
    for (size_t axis = 0; axis < config.dimensions.size(); axis++) {
        size_t logical = config.dimensions[axis];
        bool omitted = config.axis_is_omitted(axis);
        size_t eff = omitted ? logical : effective_axis_len(config.transform, logical, axis);
        AxisAlgorithm alg;
        if (omitted) {
            alg = plan_axis_algorithm(logical, config.tuning);
        } else if (config.transform == TransformKind::C2C && device &&
                   has_fixed_upstream_gpu_scheduler_profile(*device)) {
            AxisClass cls = cls_override >= 0 ? static_cast<AxisClass>(cls_override)
                                              : (axis + 1 == config.dimensions.size() ? AxisClass::Contiguous
                                                                                      : AxisClass::Strided);
            alg = plan_c2c_axis_algorithm_for_device(eff, exec_batch, config.tuning, config.precision, cls, *device);
        } else {
            alg = plan_axis_algorithm(eff, config.tuning);
        }
        AxisPlan ap;
        ap.axis = axis;
        ap.logical_len = logical;
        ap.effective_fft_len = eff;
        ap.algorithm = alg;
        ap.estimated_scratch_complex = omitted ? 0 : scratch_estimate(alg);
        plan.axes.push_back(ap);
    }
    return plan;
}

FftPlan FftPlan::build(const FftConfig &c) { return build_inner(c, nullptr, -1); }

FftPlan FftPlan::build_for_device(const FftConfig &c, const DeviceProfile &d) {
    return build_inner(c.resolve_tuning_for_device(d), &d, -1);
}

FftPlan FftPlan::build_c2c_child_for_device(const FftConfig &c, const DeviceProfile &d, AxisClass cls) {
    if (c.transform != TransformKind::C2C || c.dimensions.size() != 1)
        fail_unsupported("device-scored C2C child planning requires a one-dimensional C2C config");
    return build_inner(c.resolve_tuning_for_device(d), &d, static_cast<int>(cls));
}

// ---- scheduler.rs:17-208: fixed upstream Bluestein auto-padding tables -----

struct PadEntry {
    size_t threshold, padded;
};
static const PadEntry NVIDIA_WIDE[] = {
    {17, 36},     {19, 40},     {23, 48},     {29, 64},     {34, 70},     {37, 80},     {41, 90},     {46, 96},
    {51, 104},    {53, 128},    {67, 144},    {73, 160},    {82, 256},    {129, 288},   {145, 512},   {257, 625},
    {314, 750},   {376, 756},   {379, 768},   {386, 1024},  {513, 1056},  {529, 1200},  {601, 1225},  {614, 1250},
    {626, 1296},  {649, 1331},  {667, 1440},  {721, 1456},  {730, 1560},  {781, 2048},  {1025, 2187}, {1095, 2304},
    {1153, 2688}, {1345, 2730}, {1366, 2925}, {1464, 3000}, {1501, 4096}, {2049, 4368}, {2185, 4608}, {2305, 4900},
    {2364, 4900}, {2451, 5184}, {2593, 5625}, {2814, 5760}, {2881, 6000}, {3001, 6048}, {3026, 6144}, {3073, 6561},
    {3282, 8192}};
static const PadEntry NVIDIA_F32[] = {
    {17, 36},     {19, 40},     {23, 48},     {29, 64},     {34, 70},     {37, 80},     {41, 96},     {51, 104},
    {53, 112},    {57, 120},    {61, 128},    {67, 144},    {73, 150},    {76, 160},    {82, 256},    {129, 384},
    {193, 512},   {257, 567},   {285, 625},   {314, 768},   {386, 832},   {417, 1024},  {513, 1152},  {577, 1200},
    {601, 1296},  {649, 1536},  {769, 2048},  {1025, 2187}, {1095, 2304}, {1153, 2500}, {1251, 2592}, {1297, 2816},
    {1409, 3072}, {1537, 4096}, {2049, 4368}, {2185, 4563}, {2283, 4576}, {2289, 4608}, {2305, 5184}, {2593, 5625},
    {2814, 5632}, {2817, 6000}, {3001, 6144}, {3073, 6561}, {3282, 8192}};
static const PadEntry OTHER_WIDE[] = {
    {17, 36},     {19, 40},     {23, 56},     {29, 64},     {34, 70},     {37, 78},     {41, 81},     {43, 90},
    {46, 125},    {67, 150},    {76, 175},    {89, 189},    {97, 198},    {101, 243},   {123, 256},   {129, 270},
    {136, 512},   {257, 625},   {314, 640},   {321, 702},   {353, 750},   {376, 756},   {379, 768},   {386, 875},
    {439, 1024},  {513, 1296},  {649, 1300},  {651, 1323},  {663, 1344},  {673, 1512},  {757, 1792},  {897, 2016},
    {1009, 2048}, {1025, 2187}, {1095, 3136}, {1569, 3159}, {1581, 3430}, {1717, 3584}, {1793, 4096}, {2049, 4224},
    {2113, 4375}, {2189, 4480}, {2241, 4704}, {2353, 4928}, {2465, 4992}, {2497, 5005}, {2504, 5103}, {2553, 5376},
    {2689, 5632}, {2817, 5824}, {2913, 6048}, {3026, 6144}, {3073, 6875}, {3439, 8192}};
static const PadEntry OTHER_F32[] = {
    {17, 36},     {19, 42},     {23, 64},     {34, 81},     {43, 88},     {46, 125},    {67, 150},    {76, 162},
    {82, 175},    {89, 256},    {129, 512},   {257, 625},   {314, 768},   {386, 1024},  {513, 1296},  {649, 2048},
    {1025, 2187}, {1095, 2304}, {1153, 2500}, {1251, 2592}, {1297, 3072}, {1537, 3125}, {1564, 3136}, {1569, 4096},
    {2049, 4375}, {2189, 4608}, {2305, 5184}, {2593, 6561}, {3282, 8192}};

// scheduler.rs:228-237
static bool precision_uses_lut(Precision p) {
    return p == Precision::F64 || p == Precision::F64ComputeF32Storage || p == Precision::DoubleDouble ||
           p == Precision::DoubleDoubleF64Storage;
}

// scheduler.rs:242-270; returns 0 for "no table entry"
static size_t bluestein_padding_from_table(size_t seq, Precision p, const DeviceProfile &d) {
    if (!has_fixed_upstream_gpu_scheduler_profile(d)) return 0;
    bool wide = precision_uses_lut(p);
    const PadEntry *t;
    size_t n;
    if (d.vendor == Vendor::Nvidia) {
        t = wide ? NVIDIA_WIDE : NVIDIA_F32;
        n = wide ? sizeof(NVIDIA_WIDE) / sizeof(PadEntry) : sizeof(NVIDIA_F32) / sizeof(PadEntry);
    } else {
        t = wide ? OTHER_WIDE : OTHER_F32;
        n = wide ? sizeof(OTHER_WIDE) / sizeof(PadEntry) : sizeof(OTHER_F32) / sizeof(PadEntry);
    }
    if (seq > SIZE_MAX / 2 || seq * 2 < 1) return 0;
    size_t required = seq * 2 - 1;
    for (size_t i = 0; i < n; i++) {
        if (seq < t[i].threshold) break;
        if (i + 1 == n || seq < t[i + 1].threshold) return required <= t[i].padded ? t[i].padded : 0;
    }
    return 0;
}

// ---- scheduler.rs register "goodness" tables (VkFFTGetRegistersPerThread) ----
static const int RT = 33;  // VKFFT_RADIX_TABLE_LEN (scheduler.rs:637)
typedef size_t RegTable[RT];

static void derive_composites(RegTable r) {  // scheduler.rs:10334-10370
    r[32] = r[2] % 32 == 0 ? r[2] : 0;
    r[16] = r[2] % 16 == 0 ? r[2] : 0;
    r[8] = r[2] % 8 == 0 ? r[2] : 0;
    r[4] = r[2] % 4 == 0 ? r[2] : 0;
    if (r[2] >= 12 && r[3] >= 12) {
        size_t v = std::min(r[2], r[3]);
        r[12] = v % 12 == 0 ? v : 0;
    } else {
        r[12] = 0;
    }
    r[6] = std::min(r[2], r[3]);
    r[9] = r[3] % 9 == 0 ? r[3] : 0;
    r[10] = std::min(r[2], r[5]);
    r[14] = std::min(r[2], r[7]);
    r[15] = std::min(r[3], r[5]);
}

// scheduler.rs:10639-10798 optimize_radix_kernels (register_boost 1 on this path)
static void optimize_radix_kernels(RegTable reg, RegTable m) {
    if ((reg[32] > 0 || reg[2] % 32 == 0) && reg[32] % 32 == 0 && m[2] >= 5) {
        m[32] = m[2] / 5;
        m[2] -= m[32] * 5;
        if (reg[2] % 32 == 0) reg[32] = reg[2];
    }
    if ((reg[16] > 0 || reg[2] % 16 == 0) && reg[16] % 16 == 0 && m[2] >= 4) {
        m[16] = m[2] / 4;
        m[2] -= m[16] * 4;
        if (reg[2] % 16 == 0) reg[16] = reg[2];
    }
    if (reg[15] > 0 && reg[15] % 15 == 0 && m[3] >= 1 && m[5] >= 1) {
        m[15] = std::min(m[3], m[5]);
        m[3] -= m[15];
        m[5] -= m[15];
    }
    if (reg[14] > 0 && reg[14] % 14 == 0 && m[2] >= 1 && m[7] >= 1) {
        m[14] = std::min(m[2], m[7]);
        m[2] -= m[14];
        m[7] -= m[14];
    }
    if (reg[12] > 0 && reg[12] % 12 == 0 && m[2] >= 2 && m[3] >= 1) {
        m[12] = std::min(m[3], m[2] / 2);
        m[2] -= 2 * m[12];
        m[3] -= m[12];
    }
    if (reg[10] > 0 && reg[10] % 10 == 0 && m[2] >= 1 && m[5] >= 1) {
        m[10] = std::min(m[2], m[5]);
        m[2] -= m[10];
        m[5] -= m[10];
    }
    if (reg[9] > 0 && reg[9] % 9 == 0 && m[3] >= 2) {
        m[9] = m[3] / 2;
        m[3] -= m[9] * 2;
    }
    if ((reg[8] > 0 || reg[2] % 8 == 0) && reg[8] % 8 == 0 && m[2] >= 3) {
        m[8] = m[2] / 3;
        m[2] -= m[8] * 3;
        if (reg[2] % 8 == 0) reg[8] = reg[2];
    }
    if (reg[6] > 0 && reg[6] % 6 == 0 && m[2] >= 1 && m[3] >= 1) {
        m[6] = std::min(m[2], m[3]);
        m[2] -= m[6];
        m[3] -= m[6];
    }
    if ((reg[4] > 0 || reg[2] % 4 == 0) && reg[4] % 4 == 0 && m[2] >= 2) {
        m[4] = m[2] / 2;
        m[2] -= m[4] * 2;
        if (reg[2] % 4 == 0) reg[4] = reg[2];
    }
}

// scheduler.rs:10800-10818 over the optimised stage list; returns is_good_sequence
static bool stage_goodness(const RegTable reg, const RegTable m) {
    size_t mx = 0, mn = SIZE_MAX;
    for (int radix = RT - 1; radix >= 2; radix--)
        if (m[radix] > 0 && reg[radix] > 0) {
            mx = std::max(mx, reg[radix]);
            mn = std::min(mn, reg[radix]);
        }
    if (mx == 0) fail_invalid_ir("mixed-radix scheduler produced no executable stages");
    return !(mx > 16 || mx >= 2 * mn);
}

static size_t ceil_div_sz(size_t v, size_t d) { return (v + d - 1) / d; }

// scheduler.rs:10854-10949 power_of_two_register_table -> is_good_sequence
static bool pow2_is_good(size_t fft_len, size_t rhs) {
    if (fft_len == 1) return true;
    size_t exponent = __builtin_ctzll(fft_len);
    RegTable r = {0};
    size_t ay = std::max<size_t>(rhs / 64, 1);
    size_t test_min = SIZE_MAX, max_radix_min_stages = 1;
    for (size_t c = 1; c <= 3; c++) {
        size_t st = ceil_div_sz(exponent, c);
        if (st < test_min) {
            test_min = st;
            max_radix_min_stages = c;
        }
    }
    size_t mlm = 0;
    for (size_t c = max_radix_min_stages; c >= 1; c--) {
        size_t ax = checked_mul(ay, fft_len, "power-of-two register scheduler active thread estimate") >> c;
        if (ax >= 128) {
            mlm = c;
            break;
        }
    }
    mlm = std::max<size_t>(mlm, 3);
    size_t fin = 1, min_stages = exponent;
    for (size_t c = 2; c <= mlm; c++) {
        size_t st = ceil_div_sz(exponent, c);
        if (st < min_stages) {
            fin = c;
            min_stages = st;
        }
    }
    size_t re = exponent > fin ? fin : exponent;
    r[2] = (size_t)1 << re;
    if (exponent < 3) r[2] = (size_t)1 << exponent;
    r[32] = r[2] % 32 == 0 ? r[2] : 0;
    r[16] = r[2] % 16 == 0 ? r[2] : 0;
    r[8] = r[2] % 8 == 0 ? r[2] : 0;
    r[4] = r[2] % 4 == 0 ? r[2] : 0;
    r[6] = std::min(r[2], r[3]);
    r[9] = r[3] % 9 == 0 ? r[3] : 0;
    r[10] = std::min(r[2], r[5]);
    r[14] = std::min(r[2], r[7]);
    r[15] = std::min(r[3], r[5]);
    size_t mx = 0, mn = SIZE_MAX;
    for (int i = 0; i < RT; i++)
        if (r[i] > 0) {
            mx = std::max(mx, r[i]);
            mn = std::min(mn, r[i]);
        }
    if (mn == SIZE_MAX) {
        mn = 2;
        mx = 2;
    }
    return !(mx > 16 || mx >= 2 * mn);
}

// scheduler.rs:9882-9988 (2^a 3^b) and :10318-10463 (remaining smooth families)
static bool mixed_is_good(size_t fft_len, size_t rhs) {
    (void)rhs;
    static const size_t primes[6] = {2, 3, 5, 7, 11, 13};
    size_t rem = fft_len;
    size_t e[6] = {0};
    for (int i = 0; i < 6; i++)
        while (rem % primes[i] == 0) {
            rem /= primes[i];
            e[i]++;
        }
    if (rem != 1) fail_unsupported("mixed-radix register slice requires factors from 2/3/5/7/11/13 only");
    int mask = 0;
    for (int i = 0; i < 6; i++)
        if (e[i]) mask |= 1 << i;
    RegTable r = {0};
    RegTable m = {0};
    for (int i = 0; i < 6; i++) m[primes[i]] = e[i];
    auto has = [&](int i) { return (mask >> i) & 1; };
    const int B2 = 1, B3 = 2, B5 = 4, B7 = 8, B11 = 16, B13 = 32;
    if (mask == B2 || mask == 0)
        fail_unsupported("power-of-two or empty factorization belongs to a different scheduler branch");
    if (mask == (B2 | B3)) {
        // scheduler.rs:9882-9988
        size_t prim = (e[0] == e[1] || e[0] == 1) ? 6 : 12;
        r[2] = r[3] = prim;
        r[32] = r[2] % 32 == 0 ? r[2] : 0;
        r[16] = r[2] % 16 == 0 ? r[2] : 0;
        r[8] = r[2] % 8 == 0 ? r[2] : 0;
        r[4] = r[2] % 4 == 0 ? r[2] : 0;
        if (r[2] >= 12 && r[3] >= 12) {
            r[12] = std::min(r[2], r[3]);
            if (r[12] % 12 != 0) r[12] = 0;
        }
        r[6] = std::min(r[2], r[3]);
        r[9] = r[3] % 9 == 0 ? r[3] : 0;
        optimize_radix_kernels(r, m);
        return stage_goodness(r, m);
    }
    const int S11_13 = B11 | B13;
    int core = mask & ~S11_13;  // the 2/3/5/7 part
    bool has11 = has(4), has13 = has(5);
    auto add1113 = [&]() {
        if (has11) r[11] = 11;
        if (has13) r[13] = 13;
    };
    if (mask == B3) {
        r[3] = e[1] == 1 ? 3 : 9;
    } else if (mask == B5) {
        r[5] = 5;
    } else if (mask == B7) {
        r[7] = 7;
    } else if (mask == B11) {
        r[11] = 11;
    } else if (mask == B13) {
        r[13] = 13;
    } else if (mask == (B2 | B5)) {
        r[2] = e[0] <= 2 ? 10 : 8;
        r[5] = 10;
    } else if (mask == (B2 | B7)) {
        if (e[0] <= 2) {
            r[2] = 14;
            r[7] = 14;
        } else {
            r[2] = 8;
            r[7] = 7;
        }
    } else if (mask == (B2 | B11)) {
        r[2] = e[0] == 1 ? 10 : 8;
        r[11] = 11;
    } else if (mask == (B2 | B13)) {
        r[2] = e[0] <= 2 ? 12 : 8;
        r[13] = 13;
    } else if (mask == (B3 | B5)) {
        r[3] = 15;
        r[5] = 15;
    } else if (mask == (B3 | B7)) {
        r[3] = e[1] == 1 ? 6 : 9;
        r[7] = 7;
    } else if (mask == (B3 | B11)) {
        r[3] = 9;
        r[11] = 11;
    } else if (mask == (B3 | B13)) {
        r[3] = e[1] == 1 ? 12 : 9;
        r[13] = 13;
    } else if (core == (B2 | B5) && (has11 || has13)) {
        // [0,2,4] | [0,2,5] | [0,2,4,5]
        r[2] = e[0] <= 2 ? 10 : 8;
        r[5] = 10;
        add1113();
    } else if (core == (B2 | B7) && (has11 || has13)) {
        r[2] = (e[0] == 1 || e[0] == 2) ? 14 : (e[0] == 3 ? 8 : 16);
        r[7] = 14;
        add1113();
    } else if (mask == (B2 | B11 | B13)) {
        r[2] = e[0] <= 2 ? 12 : 8;
        r[11] = 11;
        r[13] = 13;
    } else if (core == (B2 | B5 | B7) && (has11 || has13)) {
        r[2] = (e[0] == 1 || e[0] == 2) ? 10 : (e[0] == 3 ? 8 : 16);
        r[5] = 10;
        r[7] = 14;
        add1113();
    } else if (core == (B3 | B5) && (has11 || has13)) {
        r[3] = 15;
        r[5] = 15;
        add1113();
    } else if (core == (B3 | B7) && (has11 || has13)) {
        if (e[1] == 1) {
            r[3] = 12;
            r[7] = 14;
        } else {
            r[3] = 9;
            r[7] = 7;
        }
        add1113();
    } else if (mask == (B3 | B11 | B13)) {
        r[3] = e[1] == 1 ? 12 : 9;
        r[11] = 11;
        r[13] = 13;
    } else if (core == (B3 | B5 | B7) && (has11 || has13)) {
        r[3] = 15;
        r[5] = 15;
        r[7] = 14;
        add1113();
    } else if (mask == (B2 | B3 | B11 | B13)) {
        if (e[0] == 1) {
            r[2] = 6;
            r[3] = 6;
        } else {
            r[2] = 12;
            r[3] = 12;
        }
        r[11] = 11;
        r[13] = 13;
    } else if (core == (B2 | B3 | B5) && (has11 || has13)) {
        if (e[0] == 1) {
            r[2] = 10;
            r[3] = 15;
        } else {
            r[2] = 12;
            r[3] = 12;
        }
        r[5] = 10;
        add1113();
    } else if (core == (B2 | B3 | B7) && (has11 || has13)) {
        r[2] = 12;
        r[3] = 12;
        r[7] = 14;
        add1113();
    } else if (core == (B2 | B3 | B5 | B7) && (has11 || has13)) {
        if (e[0] == 1) {
            r[2] = 14;
            r[3] = 15;
        } else if (e[0] == 2 || e[0] == 3) {
            r[2] = 12;
            r[3] = 12;
        } else {
            r[2] = 16;
            r[3] = 12;
        }
        r[5] = 15;
        r[7] = 14;
        add1113();
    } else if (mask == (B2 | B3 | B5)) {
        if (e[0] == 1) {
            r[2] = 6;
            r[3] = 6;
            r[5] = 5;
        } else {
            r[2] = 12;
            r[3] = 12;
            r[5] = 10;
        }
    } else if (mask == (B2 | B3 | B7)) {
        if (e[0] <= 2) {
            r[2] = 6;
            r[3] = 6;
            r[7] = 7;
        } else {
            r[2] = 8;
            r[3] = 6;
            r[7] = 7;
        }
    } else if (mask == (B2 | B3 | B11)) {
        if (e[0] == 1) {
            r[2] = 6;
            r[3] = 6;
        } else {
            r[2] = 12;
            r[3] = 12;
        }
        r[11] = 11;
    } else if (mask == (B2 | B3 | B13)) {
        if (e[0] == 1) {
            r[2] = 6;
            r[3] = 6;
        } else {
            r[2] = 12;
            r[3] = 12;
        }
        r[13] = 13;
    } else if (mask == (B2 | B5 | B7)) {
        r[2] = e[0] <= 2 ? 10 : 8;
        r[5] = 10;
        r[7] = 7;
    } else if (mask == (B3 | B5 | B7)) {
        r[3] = 15;
        r[5] = 15;
        r[7] = 14;
    } else if (mask == (B2 | B3 | B5 | B7)) {
        if (e[0] == 1) {
            r[2] = 14;
            r[3] = 15;
        } else if (e[0] == 2 || e[0] == 3) {
            r[2] = 12;
            r[3] = 12;
        } else {
            r[2] = 16;
            r[3] = 12;
        }
        r[5] = 15;
        r[7] = 14;
    } else if ((mask & (B2 | B3)) == 0) {
        // every active factor index >= 2 (5/7/11/13 only)
        for (int i = 2; i < 6; i++)
            if (has(i)) r[primes[i]] = primes[i];
    } else {
        fail_invalid_ir("exhaustive smooth-factor register-table dispatch missed a supported factor subset");
    }
    derive_composites(r);
    optimize_radix_kernels(r, m);
    return stage_goodness(r, m);
}

// scheduler.rs:2267-2460 plan_gpu_double_double_quad_registers -> is_good_sequence
static bool dd_quad_is_good(size_t fft_len, size_t rhs) {
    size_t rem = fft_len, e2 = 0, e3 = 0, e5 = 0, e7 = 0;
    while (rem % 2 == 0) rem /= 2, e2++;
    while (rem % 3 == 0) rem /= 3, e3++;
    while (rem % 5 == 0) rem /= 5, e5++;
    while (rem % 7 == 0) rem /= 7, e7++;
    if (rem != 1) fail_unsupported("fixed-upstream Quad register table supports only factors 2/3/5/7");
    RegTable r = {0};
    if (e2 > 0) {
        if (e3 > 0) {
            if (e5 > 0) {
                r[2] = 6;
                r[3] = 6;
                r[5] = 5;
                if (e7 > 0) r[7] = 7;
            } else if (e7 > 0) {
                r[2] = e2 <= 2 ? 6 : 8;
                r[3] = 6;
                r[7] = 7;
            } else {
                r[2] = 6;
                r[3] = 6;
            }
        } else if (e5 > 0) {
            if (e7 > 0) {
                r[2] = e2 == 1 ? 6 : 8;
                r[5] = 5;
                r[7] = 7;
            } else {
                r[2] = 4;
                r[5] = 5;
            }
        } else if (e7 > 0) {
            r[2] = 8;
            r[7] = 7;
        } else {
            size_t ay = std::max<size_t>(rhs / 64, 1);
            size_t test_min = SIZE_MAX, mrms = 1;
            for (size_t c = 1; c <= 3; c++) {
                size_t st = ceil_div_sz(e2, c);
                if (st < test_min) {
                    test_min = st;
                    mrms = c;
                }
            }
            size_t mm = 0;
            for (size_t c = mrms; c >= 1; c--) {
                size_t ax = checked_mul(ay, fft_len, "double-double Quad active thread estimate") >> c;
                if (ax >= 128) {
                    mm = c;
                    break;
                }
            }
            mm = std::max<size_t>(mm, 3);
            size_t fin = 1, min_st = e2;
            for (size_t c = 2; c <= mm; c++) {
                size_t st = ceil_div_sz(e2, c);
                if (st < min_st) {
                    fin = c;
                    min_st = st;
                }
            }
            size_t used = std::min(e2, fin);
            r[2] = (size_t)1 << used;
            if (e2 < 3) r[2] = (size_t)1 << e2;
        }
    } else if (e3 > 0) {
        if (e5 > 0) {
            if (e7 > 0) {
                r[3] = 6;
                r[5] = 5;
                r[7] = 7;
            } else {
                r[3] = 3;
                r[5] = 5;
            }
        } else if (e7 > 0) {
            r[3] = 6;
            r[7] = 7;
        } else {
            r[3] = e3 == 1 ? 3 : 9;
        }
    } else if (e5 > 0) {
        r[5] = 5;
        if (e7 > 0) r[7] = 7;
    } else if (e7 > 0) {
        r[7] = 7;
    } else {
        fail_unsupported("double-double Quad factorization produced no supported radix");
    }
    r[32] = r[2] % 32 == 0 ? r[2] : 0;
    r[16] = r[2] % 16 == 0 ? r[2] : 0;
    r[8] = r[2] % 8 == 0 ? r[2] : 0;
    r[4] = r[2] % 4 == 0 ? r[2] : 0;
    if (r[2] >= 12 && r[3] >= 12) {
        r[12] = std::min(r[2], r[3]);
        if (r[12] % 12 != 0) r[12] = 0;
    }
    r[6] = std::min(r[2], r[3]);
    r[9] = r[3] % 9 == 0 ? r[3] : 0;
    r[10] = std::min(r[2], r[5]);
    r[14] = std::min(r[2], r[7]);
    r[15] = std::min(r[3], r[5]);
    size_t mx = 0, mn = SIZE_MAX;
    for (int i = 0; i < RT; i++)
        if (r[i]) {
            mx = std::max(mx, r[i]);
            mn = std::min(mn, r[i]);
        }
    if (mx == 0) fail_invalid_ir("double-double Quad register table produced no executable radix");
    return !(mx > 16 || mx >= 2 * mn);
}

static bool small_radix_smooth(size_t v) {  // scheduler.rs:272-280
    for (size_t p : {2, 3, 5, 7})
        while (v % p == 0) v /= p;
    return v == 1;
}

// scheduler.rs:283-357 generic good-sequence search
static size_t bluestein_generic_padding(size_t seq, size_t batch, Precision p, const DeviceProfile &d) {
    if (!has_fixed_upstream_gpu_scheduler_profile(d))
        fail_unsupported("fixed upstream Bluestein padding requires a known GPU scheduler profile");
    if (seq > SIZE_MAX / 2 || seq * 2 < 1) fail_overflow("fixed upstream Bluestein minimum padded length");
    size_t required = seq * 2 - 1;
    size_t max_rhs = checked_mul(seq, batch, "fixed upstream Bluestein RHS estimate");
    size_t cb = compute_complex_bytes(p);
    size_t used = is_pow2(seq) ? d.shared_memory_pow2_bytes : d.shared_memory_bytes;
    size_t max_shared = used / cb;
    size_t cand = required;
    for (;;) {
        size_t np = 1;
        while (np < cand) {
            if (np > (SIZE_MAX >> 1)) fail_overflow("fixed upstream Bluestein next power of two");
            np <<= 1;
        }
        bool tq = (unsigned __int128)np * 3 <= (unsigned __int128)cand * 4;
        bool fits = np <= max_shared || required > max_shared;
        if (seq < 128 || (tq && fits)) cand = np;
        if (small_radix_smooth(cand)) {
            size_t rhs = std::max<size_t>(max_rhs / cand, 1);
            bool good;
            if (is_double_double(p))
                good = dd_quad_is_good(cand, rhs);
            else if (is_pow2(cand))
                good = pow2_is_good(cand, rhs);
            else
                good = mixed_is_good(cand, rhs);
            if (good) return cand;
        }
        cand = checked_add(cand, 1, "fixed upstream Bluestein padding search");
    }
}

size_t upstream_bluestein_auto_padding(size_t seq, size_t batch, Precision p, const DeviceProfile &d) {
    size_t t = bluestein_padding_from_table(seq, p, d);
    if (t) return t;
    return bluestein_generic_padding(seq, batch, p, d);
}

// scheduler.rs:1758-1782
static bool force_rader_two_upload(size_t seq, const std::vector<size_t> &fft_primes, const DeviceProfile &d) {
    if (seq == 0 || d.max_threads_per_block == 0) fail_invalid_ir("Rader upload pressure requires non-zero dimensions");
    if (d.backend == Backend::CpuReference) return false;
    for (size_t p : fft_primes) {
        if (p < 2 || seq % p != 0) fail_invalid_ir("FFT-Rader prime does not divide the scheduled axis");
        size_t containers = seq / p;
        if (containers > 512 || containers > d.max_threads_per_block) return true;
    }
    return false;
}

// real_ir.rs:1124-1207 (FixedUpstreamDevice shape policy)
RealAlgorithm real_fft_algorithm_for_device(size_t length, size_t batch, Precision p, const PlannerTuning &tuning,
                                            const DeviceProfile &d) {
    if (length < 2 || length % 2 != 0) return RealAlgorithm::FullComplex;
    if (!has_fixed_upstream_gpu_scheduler_profile(d)) return RealAlgorithm::EvenHalfSize;
    if (d.vendor == Vendor::Apple) return RealAlgorithm::FullComplex;
    size_t cb = compute_complex_bytes(p);
    size_t used = is_pow2(length) ? d.shared_memory_pow2_bytes : d.shared_memory_bytes;
    size_t max_ns = used / cb;
    if (length > max_ns) return RealAlgorithm::EvenHalfSize;
    PlannerTuning up = tuning;
    up.allow_recursive_fft_rader = false;
    FftConfig sc = FftConfig::make({length});
    sc.precision = p;
    sc.with_tuning(up);
    FftPlan scoring = FftPlan::build_c2c_child_for_device(sc, d, AxisClass::Contiguous);
    const AxisAlgorithm &alg = scoring.axes[0].algorithm;
    if (alg.kind == AlgorithmKind::Stockham) return RealAlgorithm::FullComplex;
    if (alg.kind == AlgorithmKind::Bluestein) {
        size_t padded = upstream_bluestein_auto_padding(length, batch, p, d);
        return padded > max_ns ? RealAlgorithm::EvenHalfSize : RealAlgorithm::FullComplex;
    }
    size_t largest_direct = 0;
    std::vector<size_t> fft_primes;
    for (auto &r : alg.primes) {
        if (!r.fft_convolution)
            largest_direct = std::max(largest_direct, r.prime);
        else
            fft_primes.push_back(r.prime);
    }
    size_t reserved = used;
    if (largest_direct) {
        size_t res = (largest_direct - 1) * cb;
        reserved = used > res ? used - res : 0;
    }
    size_t reserved_limit = reserved / cb;
    bool two = force_rader_two_upload(length, fft_primes, d);
    return (length > reserved_limit || two) ? RealAlgorithm::EvenHalfSize : RealAlgorithm::FullComplex;
}

void fill_axis_info(const AxisPlan &a, b200fft_axis_info &o) {
    std::memset(&o, 0, sizeof(o));
    o.axis = a.axis;
    o.logical_len = a.logical_len;
    o.effective_fft_len = a.effective_fft_len;
    o.estimated_scratch_complex = a.estimated_scratch_complex;
    o.algorithm = static_cast<int32_t>(a.algorithm.kind);
    o.convolution_len = a.algorithm.convolution_len;
    o.prime_factor_count = (uint32_t)std::min<size_t>(a.algorithm.radix.prime_factors.size(), B200FFT_MAX_FACTORS);
    for (uint32_t i = 0; i < o.prime_factor_count; i++) o.prime_factors[i] = a.algorithm.radix.prime_factors[i];
    o.merged_radix_count = (uint32_t)std::min<size_t>(a.algorithm.radix.merged_radices.size(), B200FFT_MAX_FACTORS);
    for (uint32_t i = 0; i < o.merged_radix_count; i++) o.merged_radices[i] = a.algorithm.radix.merged_radices[i];
    o.rader_prime_count = (uint32_t)std::min<size_t>(a.algorithm.primes.size(), B200FFT_MAX_RADER_PRIMES);
    for (uint32_t i = 0; i < o.rader_prime_count; i++) {
        auto &r = a.algorithm.primes[i];
        auto &dst = o.rader_primes[i];
        dst.prime = r.prime;
        dst.multiplicity = r.multiplicity;
        dst.generator = r.generator;
        dst.mode = r.fft_convolution ? B200FFT_RADER_FFT_CONVOLUTION : B200FFT_RADER_DIRECT;
        dst.convolution_factor_count =
            (uint32_t)std::min<size_t>(r.convolution.prime_factors.size(), B200FFT_MAX_FACTORS);
        for (uint32_t k = 0; k < dst.convolution_factor_count; k++)
            dst.convolution_factors[k] = r.convolution.prime_factors[k];
    }
}

}  // namespace b200fft
