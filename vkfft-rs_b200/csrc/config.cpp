// FftConfig, PlannerTuning and DeviceProfile: validation and device resolution.
// Restates vkfft-rs src/config.rs (line references per function) so validation
// accepts and rejects exactly the same configurations with the same messages.
#include <algorithm>
#include <cstring>

#include "core.hpp"

namespace b200fft {

[[noreturn]] void fail_overflow(const char *operation) {
    throw FftError(B200FFT_ARITHMETIC_OVERFLOW, std::string("integer overflow while computing ") + operation);
}
[[noreturn]] void fail_invalid_ir(const char *message) {
    throw FftError(B200FFT_INVALID_KERNEL_IR, std::string("invalid kernel IR: ") + message);
}
[[noreturn]] void fail_unsupported(const char *message) {
    throw FftError(B200FFT_UNSUPPORTED_KERNEL_PATH, std::string("unsupported kernel path: ") + message);
}
[[noreturn]] void fail_tuning(const char *message) {
    throw FftError(B200FFT_INVALID_PLANNER_TUNING, std::string("invalid planner tuning: ") + message);
}
[[noreturn]] void fail_value_range(const char *field) {
    throw FftError(B200FFT_VALUE_OUT_OF_RANGE,
                   std::string(field) + " cannot be represented by the current backend index type");
}
[[noreturn]] void fail_runtime(const std::string &message) {
    throw FftError(B200FFT_NATIVE_RUNTIME, "CUDA runtime error: " + message);
}
[[noreturn]] void fail_unavailable(const std::string &message) {
    throw FftError(B200FFT_NATIVE_UNAVAILABLE, "CUDA runtime is unavailable: " + message);
}
[[noreturn]] void fail_precision(const char *backend, const char *precision) {
    throw FftError(B200FFT_UNSUPPORTED_PRECISION,
                   std::string(backend) + " backend does not yet support precision " + precision);
}
[[noreturn]] void fail_input_length(size_t expected, size_t actual) {
    throw FftError(B200FFT_INPUT_LENGTH_MISMATCH, "input contains " + std::to_string(actual) +
                                                      " complex elements but kernel expects " +
                                                      std::to_string(expected));
}
[[noreturn]] void fail_resource(const char *resource, size_t required, size_t available) {
    throw FftError(B200FFT_RESOURCE_LIMIT_EXCEEDED, std::string(resource) + " requires " +
                                                        std::to_string(required) +
                                                        " bytes/units but only " +
                                                        std::to_string(available) + " are available");
}

size_t checked_mul(size_t a, size_t b, const char *operation) {
    size_t r;
    if (__builtin_mul_overflow(a, b, &r)) fail_overflow(operation);
    return r;
}
size_t checked_add(size_t a, size_t b, const char *operation) {
    size_t r;
    if (__builtin_add_overflow(a, b, &r)) fail_overflow(operation);
    return r;
}

// config.rs:107-161
size_t compute_complex_bytes(Precision p) {
    switch (p) {
        case Precision::F16StorageF32Compute:
        case Precision::F32: return 8;
        case Precision::F64:
        case Precision::F64ComputeF32Storage: return 16;
        case Precision::DoubleDouble:
        case Precision::DoubleDoubleF64Storage: return 32;
    }
    return 8;
}
size_t storage_complex_bytes(Precision p) {
    switch (p) {
        case Precision::F16StorageF32Compute: return 4;
        case Precision::F32:
        case Precision::F64ComputeF32Storage: return 8;
        case Precision::F64:
        case Precision::DoubleDoubleF64Storage: return 16;
        case Precision::DoubleDouble: return 32;
    }
    return 8;
}
bool is_double_double(Precision p) {
    return p == Precision::DoubleDouble || p == Precision::DoubleDoubleF64Storage;
}

// config.rs:505-543
void PlannerTuning::validate() const {
    if (min_rader_direct_prime < 2 || min_rader_fft_prime < 2) fail_tuning("minimum Rader prime must be at least 2");
    if (min_rader_direct_prime > 33)
        fail_tuning("direct Rader minimum must not exceed upstream loc_multipliers capacity (33)");
    if (max_rader_direct_prime < min_rader_direct_prime)
        fail_tuning("direct Rader maximum must not be smaller than its minimum");
    if (max_rader_fft_prime < min_rader_fft_prime) fail_tuning("FFT Rader maximum must not be smaller than its minimum");
}

// config.rs:267-282
DeviceProfile DeviceProfile::generic(Backend b, Vendor v, uint32_t other) {
    DeviceProfile d;
    d.backend = b;
    d.vendor = v;
    d.vendor_other_id = other;
    d.shared_memory_bytes = 32 * 1024;
    d.shared_memory_pow2_bytes = 32 * 1024;
    d.max_threads_per_block = 256;
    d.max_workgroup_size[0] = d.max_workgroup_size[1] = d.max_workgroup_size[2] = 256;
    d.coalesced_memory_bytes = 32;
    d.shared_banks = 32;
    d.supports_f64 = b != Backend::Metal;
    d.subgroup = SubgroupProfile{};
    return d;
}

// The profile the reference derives from a CUDA device's attributes
// (backend/cuda/runtime.rs:1204-1225): shared memory per block and its power-of-two
// floor, the thread limits, 32-byte coalescing, 32 banks, 32-lane subgroups.
DeviceProfile cuda_device_profile(size_t shared_per_block, size_t max_threads, size_t dim_x, size_t dim_y,
                                  size_t dim_z, bool supports_f64) {
    DeviceProfile d = DeviceProfile::generic(Backend::Cuda, Vendor::Nvidia);
    size_t pow2 = 1;
    while (pow2 * 2 <= shared_per_block) pow2 *= 2;
    d.shared_memory_bytes = shared_per_block;
    d.shared_memory_pow2_bytes = shared_per_block ? pow2 : 0;
    d.max_threads_per_block = max_threads;
    d.max_workgroup_size[0] = dim_x;
    d.max_workgroup_size[1] = dim_y;
    d.max_workgroup_size[2] = dim_z;
    d.coalesced_memory_bytes = 32;
    d.shared_banks = 32;
    d.supports_f64 = supports_f64;
    d.subgroup.size = d.subgroup.min_size = d.subgroup.max_size = 32;
    d.subgroup.compute_supported = d.subgroup.basic_supported = d.subgroup.shuffle_supported = true;
    d.subgroup.shuffle_relative_supported = d.subgroup.compute_full_subgroups = true;
    return d;
}

// config.rs:287-299
bool has_fixed_upstream_gpu_scheduler_profile(const DeviceProfile &d) {
    switch (d.backend) {
        case Backend::Vulkan:
        case Backend::OpenCl:
            return d.vendor == Vendor::Nvidia || d.vendor == Vendor::Amd || d.vendor == Vendor::Intel;
        case Backend::Cuda: return d.vendor == Vendor::Nvidia;
        case Backend::Hip: return d.vendor == Vendor::Amd;
        case Backend::LevelZero: return d.vendor == Vendor::Intel;
        case Backend::Metal: return d.vendor == Vendor::Apple;
        case Backend::CpuReference: return false;
    }
    return false;
}

// config.rs:305-319
static size_t upstream_coalesced_memory_bytes(const DeviceProfile &d) {
    switch (d.backend) {
        case Backend::Vulkan:
        case Backend::OpenCl: return (d.vendor == Vendor::Nvidia || d.vendor == Vendor::Amd) ? 32 : 64;
        case Backend::Cuda:
        case Backend::Hip: return 32;
        case Backend::LevelZero:
        case Backend::Metal: return 64;
        case Backend::CpuReference: return d.coalesced_memory_bytes;
    }
    return 32;
}

// config.rs:324-333
size_t upstream_coalesced_memory_bytes_for_precision(const DeviceProfile &d, Precision p) {
    size_t base = upstream_coalesced_memory_bytes(d);
    return p == Precision::F16StorageF32Compute ? base * 2 : base;
}

// config.rs:337-346
static size_t upstream_direct_rader_thread_cap(const DeviceProfile &d, Precision p) {
    size_t complex_size = compute_complex_bytes(p);
    size_t per = std::max<size_t>(upstream_coalesced_memory_bytes_for_precision(d, p) / complex_size, 1);
    size_t v = d.max_threads_per_block / per;
    size_t doubled = (v > SIZE_MAX / 2) ? SIZE_MAX : v * 2;  // saturating_mul
    return doubled == 0 ? 0 : doubled - 1;                    // saturating_sub
}

// config.rs:350-360
PlannerTuning upstream_effective_rader_tuning(PlannerTuning t, const DeviceProfile &d, Precision p) {
    t.max_rader_direct_prime =
        std::max(std::min(t.max_rader_direct_prime, upstream_direct_rader_thread_cap(d, p)), t.min_rader_direct_prime);
    return t;
}

// config.rs:396-420
PlannerTuning tuning_for_device(const DeviceProfile &d, Precision p) {
    PlannerTuning t = PlannerTuning::portable();
    if (is_double_double(p)) {
        t.min_rader_direct_prime = 11;
        t.max_rader_direct_prime = 29;
    } else {
        t.max_rader_direct_prime = (d.vendor == Vendor::Nvidia || d.vendor == Vendor::Amd) ? 89 : 17;
    }
    if (d.vendor == Vendor::Amd) {
        if (is_double_double(p))
            t.min_rader_fft_prime = 19;
        else if (p == Precision::F64 || p == Precision::F64ComputeF32Storage)
            t.min_rader_fft_prime = 29;
        else
            t.min_rader_fft_prime = 17;
    }
    return t;
}

// config.rs:678-710 (FftConfig::new)
FftConfig FftConfig::make(const std::vector<size_t> &dims) {
    FftConfig c;
    c.dimensions = dims;
    size_t n = dims.size();
    c.zero_padding.assign(n, std::nullopt);
    c.omit_dimension.assign(n, false);
    c.grouped_batch.assign(n, std::nullopt);
    c.input_buffer_axis_strides.assign(n, std::nullopt);
    c.output_buffer_axis_strides.assign(n, std::nullopt);
    return c;
}

static TransformKind kind_from_c(int32_t v) {
    switch (v) {
        case B200FFT_C2C: return TransformKind::C2C;
        case B200FFT_R2C: return TransformKind::R2C;
        case B200FFT_C2R: return TransformKind::C2R;
        case B200FFT_DCT1: return TransformKind::Dct1;
        case B200FFT_DCT2: return TransformKind::Dct2;
        case B200FFT_DCT3: return TransformKind::Dct3;
        case B200FFT_DCT4: return TransformKind::Dct4;
        case B200FFT_DST1: return TransformKind::Dst1;
        case B200FFT_DST2: return TransformKind::Dst2;
        case B200FFT_DST3: return TransformKind::Dst3;
        case B200FFT_DST4: return TransformKind::Dst4;
    }
    fail_value_range("transform kind");
}

static Precision precision_from_c(int32_t v) {
    if (v < 0 || v > 5) fail_value_range("precision");
    return static_cast<Precision>(v);
}

FftConfig FftConfig::from_c(const b200fft_config &c) {
    if (c.rank > B200FFT_MAX_DIMS) fail_value_range("FFT rank");
    std::vector<size_t> dims(c.dimensions, c.dimensions + c.rank);
    FftConfig f = make(dims);
    f.batch_count = c.batch_count;
    f.transform = kind_from_c(c.transform);
    f.precision = precision_from_c(c.precision);
    f.normalize_inverse = c.normalize_inverse != 0;
    f.perform_convolution = c.perform_convolution != 0;
    f.kernel_convolution = c.kernel_convolution != 0;
    if (c.convolution_conjugation < 0 || c.convolution_conjugation > 2) fail_value_range("conjugateConvolution");
    f.convolution_conjugation = static_cast<ConvolutionConjugation>(c.convolution_conjugation);
    f.cross_power_spectrum_normalization = c.cross_power_spectrum_normalization != 0;
    f.symmetric_convolution_kernel = c.symmetric_convolution_kernel != 0;
    f.coordinate_features = c.coordinate_features;
    f.matrix_convolution = c.matrix_convolution;
    f.convolution_kernel_count = c.convolution_kernel_count;
    f.tuning.min_rader_direct_prime = c.tuning.min_rader_direct_prime;
    f.tuning.max_rader_direct_prime = c.tuning.max_rader_direct_prime;
    f.tuning.min_rader_fft_prime = c.tuning.min_rader_fft_prime;
    f.tuning.max_rader_fft_prime = c.tuning.max_rader_fft_prime;
    f.tuning.allow_recursive_fft_rader = c.tuning.allow_recursive_fft_rader != 0;
    f.use_device_tuning = c.use_device_tuning != 0;
    f.zero_padding_domain = c.zero_padding_domain ? ZeroPaddingDomain::Frequency : ZeroPaddingDomain::Spatial;
    for (uint32_t a = 0; a < c.rank; a++) {
        if (c.has_zero_padding[a] && c.zero_padding_left[a] != c.zero_padding_right[a])
            f.zero_padding[a] = ZeroPaddingRange{c.zero_padding_left[a], c.zero_padding_right[a]};
        f.omit_dimension[a] = c.omit_dimension[a] != 0;
        if (c.grouped_batch[a]) f.grouped_batch[a] = c.grouped_batch[a];
        if (c.input_buffer_axis_strides[a]) f.input_buffer_axis_strides[a] = c.input_buffer_axis_strides[a];
        if (c.output_buffer_axis_strides[a]) f.output_buffer_axis_strides[a] = c.output_buffer_axis_strides[a];
    }
    f.bandwidth_boost = c.bandwidth_boost;
    if (c.input_buffer_batch_stride) f.input_buffer_batch_stride = c.input_buffer_batch_stride;
    if (c.output_buffer_batch_stride) f.output_buffer_batch_stride = c.output_buffer_batch_stride;
    return f;
}

void FftConfig::to_c(b200fft_config &c) const {
    std::memset(&c, 0, sizeof(c));
    c.rank = static_cast<uint32_t>(dimensions.size());
    for (size_t a = 0; a < dimensions.size() && a < B200FFT_MAX_DIMS; a++) {
        c.dimensions[a] = dimensions[a];
        if (zero_padding[a]) {
            c.has_zero_padding[a] = 1;
            c.zero_padding_left[a] = zero_padding[a]->left;
            c.zero_padding_right[a] = zero_padding[a]->right;
        }
        c.omit_dimension[a] = omit_dimension[a];
        c.grouped_batch[a] = grouped_batch[a].value_or(0);
        c.input_buffer_axis_strides[a] = input_buffer_axis_strides[a].value_or(0);
        c.output_buffer_axis_strides[a] = output_buffer_axis_strides[a].value_or(0);
    }
    c.batch_count = batch_count;
    c.transform = static_cast<int32_t>(transform);
    c.precision = static_cast<int32_t>(precision);
    c.normalize_inverse = normalize_inverse;
    c.perform_convolution = perform_convolution;
    c.kernel_convolution = kernel_convolution;
    c.convolution_conjugation = static_cast<int32_t>(convolution_conjugation);
    c.cross_power_spectrum_normalization = cross_power_spectrum_normalization;
    c.symmetric_convolution_kernel = symmetric_convolution_kernel;
    c.coordinate_features = coordinate_features;
    c.matrix_convolution = matrix_convolution;
    c.convolution_kernel_count = convolution_kernel_count;
    c.tuning.min_rader_direct_prime = tuning.min_rader_direct_prime;
    c.tuning.max_rader_direct_prime = tuning.max_rader_direct_prime;
    c.tuning.min_rader_fft_prime = tuning.min_rader_fft_prime;
    c.tuning.max_rader_fft_prime = tuning.max_rader_fft_prime;
    c.tuning.allow_recursive_fft_rader = tuning.allow_recursive_fft_rader;
    c.use_device_tuning = use_device_tuning;
    c.zero_padding_domain = zero_padding_domain == ZeroPaddingDomain::Frequency;
    c.bandwidth_boost = bandwidth_boost;
    c.input_buffer_batch_stride = input_buffer_batch_stride.value_or(0);
    c.output_buffer_batch_stride = output_buffer_batch_stride.value_or(0);
}

// config.rs:834-839
FftConfig FftConfig::resolve_tuning_for_device(const DeviceProfile &d) const {
    FftConfig c = *this;
    if (c.use_device_tuning) c.tuning = tuning_for_device(d, c.precision);
    return c;
}

// config.rs:809-818
size_t FftConfig::kernel_preparation_system_count() const {
    if (!kernel_convolution) return batch_count;
    return checked_mul(batch_count, coordinate_features, "kernelConvolution batch x coordinate system count");
}

// config.rs:855-867
bool FftConfig::axis_is_omitted(size_t axis) const {
    if (axis < omit_dimension.size() && omit_dimension[axis]) return true;
    if (dimensions.size() <= 1 || axis >= dimensions.size() || dimensions[axis] != 1) return false;
    size_t fastest = dimensions.size() - 1;
    bool real = transform == TransformKind::R2C || transform == TransformKind::C2R;
    return !real || axis != fastest;
}

std::optional<size_t> FftConfig::grouped_batch_for_axis(size_t axis) const {
    if (axis < grouped_batch.size()) return grouped_batch[axis];
    return std::nullopt;
}

bool FftConfig::has_formatted_strides() const {
    if (input_buffer_batch_stride || output_buffer_batch_stride) return true;
    for (auto &s : input_buffer_axis_strides)
        if (s) return true;
    for (auto &s : output_buffer_axis_strides)
        if (s) return true;
    return false;
}

// config.rs:1463-1499 resolve_formatted_axis_strides
static std::vector<size_t> resolve_axis_strides(const std::vector<size_t> &dims,
                                                const std::vector<std::optional<size_t>> &ov,
                                                const char *field) {
    if (dims.empty()) throw FftError(B200FFT_EMPTY_DIMENSIONS, "FFT dimensions must not be empty");
    if (ov.size() != dims.size()) fail_invalid_ir("formatted axis-stride metadata must match the FFT dimensionality");
    size_t rank = dims.size(), fastest = rank - 1;
    if (ov[fastest] && *ov[fastest] != 1) fail_invalid_ir("formatted fastest-axis stride must remain one stored element");
    std::vector<size_t> strides(rank, 1);
    for (size_t a = fastest; a-- > 0;) {
        size_t minimum = checked_mul(strides[a + 1], dims[a + 1], field);
        size_t s = ov[a].value_or(minimum);
        if (s < minimum) fail_invalid_ir("formatted axis stride overlaps the next faster logical axis");
        strides[a] = s;
    }
    return strides;
}

// config.rs:1501-1522 resolve_formatted_batch_stride
static size_t resolve_batch_stride(const std::vector<size_t> &dims, const std::vector<size_t> &axis_strides,
                                   std::optional<size_t> ov, const char *field) {
    if (dims.empty() || axis_strides.size() != dims.size())
        fail_invalid_ir("formatted batch-stride metadata must match the FFT dimensionality");
    size_t minimum = checked_mul(axis_strides[0], dims[0], field);
    size_t s = ov.value_or(minimum);
    if (s < minimum) fail_invalid_ir("formatted batch stride overlaps the logical tensor");
    return s;
}

std::vector<size_t> FftConfig::resolved_axis_strides(const std::vector<size_t> &dims, bool input) const {
    return resolve_axis_strides(dims, input ? input_buffer_axis_strides : output_buffer_axis_strides,
                                input ? "formatted input axis stride" : "formatted output axis stride");
}

size_t FftConfig::resolved_batch_stride(const std::vector<size_t> &dims, bool input) const {
    auto s = resolved_axis_strides(dims, input);
    return resolve_batch_stride(dims, s, input ? input_buffer_batch_stride : output_buffer_batch_stride,
                                input ? "formatted input batch stride" : "formatted output batch stride");
}

// config.rs:1036-1460 FftConfig::validate
void FftConfig::validate() const {
    const bool real = transform == TransformKind::R2C || transform == TransformKind::C2R;
    const bool r2r = !(transform == TransformKind::C2C || real);
    if (dimensions.empty()) throw FftError(B200FFT_EMPTY_DIMENSIONS, "FFT dimensions must not be empty");
    if (batch_count == 0) throw FftError(B200FFT_ZERO_BATCH_COUNT, "FFT batch count must be greater than zero");
    if (zero_padding.size() != dimensions.size())
        fail_invalid_ir("zero-padding metadata must match the FFT dimensionality");
    if (omit_dimension.size() != dimensions.size())
        fail_invalid_ir("omitDimension metadata must match the FFT dimensionality");
    bool any_omit = std::any_of(omit_dimension.begin(), omit_dimension.end(), [](bool b) { return b; });
    if (any_omit) {
        if (dimensions.size() == 1) fail_unsupported("omitDimension currently supports multidimensional transforms only");
        if (real && omit_dimension[dimensions.size() - 1])
            fail_unsupported("omitDimension cannot disable the contiguous R2C/C2R axis");
    }
    if (dimensions.size() > 1 && !real) {
        bool all = true;
        for (size_t a = 0; a < dimensions.size(); a++) all = all && axis_is_omitted(a);
        if (all) fail_unsupported("multidimensional transform requires at least one active axis");
    }
    if (input_buffer_axis_strides.size() != dimensions.size() || output_buffer_axis_strides.size() != dimensions.size())
        fail_invalid_ir("formatted axis-stride metadata must match the FFT dimensionality");
    const bool formatted = has_formatted_strides();
    if (coordinate_features == 0) fail_value_range("coordinateFeatures");
    if (convolution_kernel_count == 0) fail_value_range("numberKernels");
    bool all_unpadded = std::all_of(zero_padding.begin(), zero_padding.end(), [](auto &z) { return !z; });
    bool all_padded = std::all_of(zero_padding.begin(), zero_padding.end(), [](auto &z) { return (bool)z; });
    if (kernel_convolution) {
        if (perform_convolution)
            fail_unsupported("kernelConvolution prepares a kernel spectrum and must not be combined with performConvolution");
        (void)kernel_preparation_system_count();
        bool dense_1d = dimensions.size() == 1 && all_unpadded;
        bool s52 = transform == TransformKind::R2C && dimensions.size() == 2 && batch_count == 2 &&
                   coordinate_features == 2 && all_unpadded;
        bool s51 = transform == TransformKind::R2C && dimensions.size() == 3 && batch_count == 1 &&
                   coordinate_features == 9 && all_padded && zero_padding_domain == ZeroPaddingDomain::Spatial;
        if (!(transform == TransformKind::C2C || transform == TransformKind::R2C) || (!dense_1d && !s52 && !s51) ||
            matrix_convolution != 1 || symmetric_convolution_kernel || convolution_kernel_count != 1 ||
            !(precision == Precision::F32 || precision == Precision::F64) || formatted ||
            convolution_conjugation != ConvolutionConjugation::None || cross_power_spectrum_normalization)
            fail_unsupported(
                "kernelConvolution currently requires dense 1D C2C/R2C independent batch/coordinate K1 preparation, "
                "pinned sample_52-style 2D R2C B2/C2 preparation, or pinned sample_51-style batch1 3D R2C C9 "
                "Spatial-padding preparation in ordinary F32/F64");
    }
    bool extended = coordinate_features != 1 || matrix_convolution != 1 || symmetric_convolution_kernel ||
                    convolution_kernel_count != 1;
    if (!perform_convolution && !kernel_convolution && extended)
        fail_unsupported(
            "coordinate/matrix/multi-kernel layout currently requires performConvolution or the pinned "
            "independent-coordinate kernelConvolution preparation contract");
    if (!perform_convolution &&
        (convolution_conjugation != ConvolutionConjugation::None || cross_power_spectrum_normalization))
        fail_unsupported("convolution conjugation/cross-power semantics require performConvolution");
    if (perform_convolution) {
        bool real_app = transform == TransformKind::R2C && dimensions.size() > 1;
        if (transform != TransformKind::C2C && !real_app)
            fail_unsupported("performConvolution supports C2C plus multidimensional R2C application transforms");
        if (dimensions.size() > 1) {
            bool scalar_k1 = !extended;
            bool scalar_fanout = matrix_convolution == 1 && coordinate_features == 1 && convolution_kernel_count > 1;
            if (real_app) {
                bool indep = matrix_convolution == 1;
                bool matrix_b1 = matrix_convolution > 1 && coordinate_features == matrix_convolution;
                if (batch_count != 1 || (!indep && !matrix_b1))
                    fail_unsupported(
                        "multidimensional real performConvolution supports batch1 independent-coordinate or matrix "
                        "K=1/K>1 layouts");
            } else {
                bool matrix_k1_b1 = matrix_convolution > 1 && batch_count == 1 && convolution_kernel_count == 1 &&
                                    coordinate_features == matrix_convolution;
                if (!scalar_k1 && !scalar_fanout && !matrix_k1_b1)
                    fail_unsupported(
                        "multidimensional performConvolution supports scalar K=1/K>1 layouts or a batch1/K1 matrix "
                        "layout");
            }
        }
        if (convolution_kernel_count > 1 && batch_count != 1)
            fail_unsupported(
                "pinned VkFFT numberKernels is a one-input fan-out, not a numberBatches*numberKernels Cartesian "
                "product: sample_52 fixes numberBatches=1 and convolutionStep uses kernel batchID for the "
                "batch/output stride");
        if (!(matrix_convolution >= 1 && matrix_convolution <= 3))
            fail_unsupported("matrixConvolution currently accepts pinned VkFFT sizes 1, 2, or 3");
        if (matrix_convolution == 1 && coordinate_features != 1 && !real_app)
            fail_unsupported(
                "coordinateFeatures > 1 without matrixConvolution is only materialized for multidimensional real "
                "application convolution");
        if (symmetric_convolution_kernel) {
            if (matrix_convolution == 3)
                fail_unsupported(
                    "pinned VkFFT 1.3.4 3x3 symmetric-kernel code aliases yz and zz while the API guide documents six "
                    "planes; keep this path fail-closed");
            if (matrix_convolution != 2) fail_unsupported("symmetricKernel requires matrixConvolution > 1");
        }
        if (convolution_conjugation == ConvolutionConjugation::Kernel)
            fail_unsupported(
                "pinned VkFFT documents conjugateConvolution=2 but has no executable kernel-conjugation codegen branch");
        bool mixed = precision == Precision::F16StorageF32Compute || precision == Precision::F64ComputeF32Storage;
        if (!(precision == Precision::F16StorageF32Compute || precision == Precision::F32 ||
              precision == Precision::F64 || precision == Precision::F64ComputeF32Storage))
            fail_unsupported("performConvolution currently requires ordinary or mixed F16/F32/F64 storage");
        bool mixed_c2c_k1 = transform == TransformKind::C2C && dimensions.size() == 1 && batch_count == 1 &&
                            coordinate_features == 1 && matrix_convolution == 1 && !symmetric_convolution_kernel &&
                            convolution_kernel_count == 1 && !formatted && all_unpadded &&
                            convolution_conjugation == ConvolutionConjugation::None &&
                            !cross_power_spectrum_normalization;
        bool mixed_scalar = coordinate_features == 1 && matrix_convolution == 1 &&
                            (convolution_kernel_count == 1 || !formatted);
        bool mixed_fanout =
            coordinate_features > 1 && matrix_convolution == 1 && convolution_kernel_count > 1 && !formatted;
        bool mixed_matrix = matrix_convolution == 3 && coordinate_features == 3 && !formatted;
        if (mixed && !(mixed_c2c_k1 || (real_app && batch_count == 1 && (mixed_scalar || mixed_fanout || mixed_matrix))))
            fail_unsupported(
                "mixed-storage performConvolution currently requires dense default-policy 1D C2C batch1 scalar K1, "
                "batch1 scalar Real ownership, unformatted independent-coordinate K>1 Real fan-out, or unformatted "
                "3x3 Real matrix ownership");
        if (formatted) {
            bool real_formatted_k1 = real_app && batch_count == 1 && coordinate_features == 1 &&
                                     matrix_convolution == 1 && convolution_kernel_count == 1;
            if (!real_formatted_k1)
                fail_unsupported("formatted performConvolution currently requires batch1 scalar ND Real K1");
        }
        if (!all_unpadded) {
            bool real_zp = real_app && batch_count == 1 && !symmetric_convolution_kernel &&
                           (matrix_convolution == 1 ||
                            (matrix_convolution > 1 && coordinate_features == matrix_convolution));
            if (!real_zp)
                fail_unsupported(
                    "performConvolution zero padding requires a pinned batch1 multidimensional real "
                    "scalar/independent-coordinate/nonsymmetric-matrix ownership");
        }
        if (any_omit) fail_unsupported("omitDimension does not compose with performConvolution");
    }
    if (formatted) {
        bool multi = dimensions.size() >= 2;
        if (!multi)
            fail_unsupported(
                "formatted strides currently support ordinary and double-double multidimensional C2C, real, and R2R "
                "transforms");
        if (dimensions.size() > 4) fail_unsupported("formatted custom strides follow upstream VKFFT_MAX_FFT_DIMENSIONS=4");
        std::vector<size_t> compact = dimensions;
        if (real) compact.back() = compact.back() / 2 + 1;
        const std::vector<size_t> *in_dims = &dimensions, *out_dims = &dimensions;
        if (!(perform_convolution && transform == TransformKind::R2C)) {
            if (transform == TransformKind::R2C) out_dims = &compact;
            if (transform == TransformKind::C2R) in_dims = &compact;
        }
        (void)resolved_batch_stride(*in_dims, true);
        (void)resolved_batch_stride(*out_dims, false);
    }
    if (grouped_batch.size() != dimensions.size()) fail_invalid_ir("groupedBatch metadata must match the FFT dimensionality");
    // groupedBatch: every C2C/real/R2R family in 1D or ND is accepted (config.rs:1378-1431)
    if (zero_padding_domain == ZeroPaddingDomain::Frequency && !all_unpadded && transform != TransformKind::C2C)
        fail_unsupported("frequency-domain zero padding currently supports C2C transforms only");
    for (size_t a = 0; a < dimensions.size(); a++) {
        size_t len = dimensions[a];
        if (len == 0) throw FftError(B200FFT_ZERO_LENGTH, "FFT axis " + std::to_string(a) + " has zero length");
        if (transform == TransformKind::Dct1 && !axis_is_omitted(a) && len < 2)
            throw FftError(B200FFT_INVALID_TRANSFORM_LENGTH,
                           "axis " + std::to_string(a) + " length " + std::to_string(len) + " is invalid for DCT-I");
        if (zero_padding[a]) {
            auto z = *zero_padding[a];
            if (z.left > z.right || z.right > len)
                throw FftError(B200FFT_INVALID_ZERO_PADDING_RANGE,
                               "zero-padding interval [" + std::to_string(z.left) + ", " + std::to_string(z.right) +
                                   ") is invalid for axis " + std::to_string(a) + " of length " + std::to_string(len));
        }
    }
    (void)r2r;
    tuning.validate();
}

}  // namespace b200fft
