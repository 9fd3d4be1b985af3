// Host-side core types of the B200 FFT engine: errors, configuration, device
// profile, planner tuning and plans.  These mirror the vkfft-rs Rust types field
// for field (config.rs, planner.rs, error.rs) so the planner port can make
// bit-identical algorithm choices.
#pragma once

#include <cstddef>
#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/b200fft.h"

namespace b200fft {

// VkFftError (error.rs:6-57) as a C++ exception carrying the C status code and the
// Display text (error.rs:59-125).
struct FftError : public std::exception {
    b200fft_status code;
    std::string message;
    FftError(b200fft_status c, std::string m) : code(c), message(std::move(m)) {}
    const char *what() const noexcept override { return message.c_str(); }
};

[[noreturn]] void fail_overflow(const char *operation);
[[noreturn]] void fail_invalid_ir(const char *message);
[[noreturn]] void fail_unsupported(const char *message);
[[noreturn]] void fail_tuning(const char *message);
[[noreturn]] void fail_value_range(const char *field);
[[noreturn]] void fail_runtime(const std::string &message);
[[noreturn]] void fail_unavailable(const std::string &message);
[[noreturn]] void fail_precision(const char *backend, const char *precision);
[[noreturn]] void fail_input_length(size_t expected, size_t actual);
[[noreturn]] void fail_resource(const char *resource, size_t required, size_t available);

size_t checked_mul(size_t a, size_t b, const char *operation);
size_t checked_add(size_t a, size_t b, const char *operation);
inline bool is_pow2(size_t v) { return v != 0 && (v & (v - 1)) == 0; }

enum class TransformKind { C2C, R2C, C2R, Dct1, Dct2, Dct3, Dct4, Dst1, Dst2, Dst3, Dst4 };
enum class Precision { F16StorageF32Compute, F32, F64, F64ComputeF32Storage, DoubleDouble, DoubleDoubleF64Storage };
enum class Backend { Vulkan, Cuda, Hip, OpenCl, LevelZero, Metal, CpuReference };
enum class Vendor { Nvidia, Amd, Intel, Apple, Other };
enum class ZeroPaddingDomain { Spatial, Frequency };
enum class ConvolutionConjugation { None, Sequence, Kernel };

// Precision::compute_complex_bytes (config.rs:138-152)
size_t compute_complex_bytes(Precision p);
size_t storage_complex_bytes(Precision p);
bool is_double_double(Precision p);

struct PlannerTuning {
    size_t min_rader_direct_prime = 17;
    size_t max_rader_direct_prime = 89;
    size_t min_rader_fft_prime = 17;
    size_t max_rader_fft_prime = 16384;
    bool allow_recursive_fft_rader = false;

    static PlannerTuning portable() { return PlannerTuning{}; }
    void validate() const;  // config.rs:505-543
};

struct SubgroupProfile {
    size_t size = 0, min_size = 0, max_size = 0;
    bool required_size_compute_supported = false, compute_supported = false, basic_supported = false,
         shuffle_supported = false, shuffle_relative_supported = false, compute_full_subgroups = false;
};

struct DeviceProfile {
    Backend backend = Backend::Cuda;
    Vendor vendor = Vendor::Nvidia;
    uint32_t vendor_other_id = 0;
    size_t shared_memory_bytes = 32 * 1024;
    size_t shared_memory_pow2_bytes = 32 * 1024;
    size_t max_threads_per_block = 256;
    size_t max_workgroup_size[3] = {256, 256, 256};
    size_t coalesced_memory_bytes = 32;
    size_t shared_banks = 32;
    bool supports_f64 = true;
    SubgroupProfile subgroup;

    static DeviceProfile generic(Backend b, Vendor v, uint32_t other = 0);  // config.rs:267-282
};

// DeviceProfile of a CUDA device from its attributes (backend/cuda/runtime.rs:1204-1225)
DeviceProfile cuda_device_profile(size_t shared_per_block, size_t max_threads, size_t dim_x, size_t dim_y,
                                  size_t dim_z, bool supports_f64);
PlannerTuning tuning_for_device(const DeviceProfile &d, Precision p);  // config.rs:396-420
bool has_fixed_upstream_gpu_scheduler_profile(const DeviceProfile &d); // config.rs:287-299
size_t upstream_coalesced_memory_bytes_for_precision(const DeviceProfile &d, Precision p);
PlannerTuning upstream_effective_rader_tuning(PlannerTuning t, const DeviceProfile &d, Precision p);

struct ZeroPaddingRange {
    size_t left = 0, right = 0;
};

struct FftConfig {
    std::vector<size_t> dimensions;
    size_t batch_count = 1;
    TransformKind transform = TransformKind::C2C;
    Precision precision = Precision::F32;
    bool normalize_inverse = false;
    bool perform_convolution = false;
    bool kernel_convolution = false;
    ConvolutionConjugation convolution_conjugation = ConvolutionConjugation::None;
    bool cross_power_spectrum_normalization = false;
    size_t coordinate_features = 1;
    size_t matrix_convolution = 1;
    bool symmetric_convolution_kernel = false;
    size_t convolution_kernel_count = 1;
    PlannerTuning tuning;
    bool use_device_tuning = true;
    std::vector<std::optional<ZeroPaddingRange>> zero_padding;
    std::vector<bool> omit_dimension;
    ZeroPaddingDomain zero_padding_domain = ZeroPaddingDomain::Spatial;
    std::vector<std::optional<size_t>> grouped_batch;
    size_t bandwidth_boost = 0;
    std::vector<std::optional<size_t>> input_buffer_axis_strides;
    std::vector<std::optional<size_t>> output_buffer_axis_strides;
    std::optional<size_t> input_buffer_batch_stride;
    std::optional<size_t> output_buffer_batch_stride;

    static FftConfig make(const std::vector<size_t> &dims);  // FftConfig::new
    static FftConfig from_c(const b200fft_config &c);
    void to_c(b200fft_config &c) const;

    FftConfig &with_tuning(const PlannerTuning &t) {
        tuning = t;
        use_device_tuning = false;
        return *this;
    }
    FftConfig resolve_tuning_for_device(const DeviceProfile &d) const;  // config.rs:834-839
    size_t kernel_preparation_system_count() const;                     // config.rs:809-818
    bool axis_is_omitted(size_t axis) const;                             // config.rs:855-867
    std::optional<size_t> grouped_batch_for_axis(size_t axis) const;
    bool has_formatted_strides() const;
    std::vector<size_t> resolved_axis_strides(const std::vector<size_t> &dims, bool input) const;
    size_t resolved_batch_stride(const std::vector<size_t> &dims, bool input) const;
    void validate() const;  // config.rs:1036-1460
};

// ---- planner.rs types ----
enum class AlgorithmKind { Stockham = 0, Rader = 1, Bluestein = 2 };

struct RadixPlan {
    std::vector<size_t> prime_factors;
    std::vector<size_t> merged_radices;
};

struct RaderPrimePlan {
    size_t prime = 0, multiplicity = 0, generator = 0;
    bool fft_convolution = false;  // RaderMode::FftConvolution vs DirectMultiplication
    RadixPlan convolution;         // only for FftConvolution
};

struct AxisAlgorithm {
    AlgorithmKind kind = AlgorithmKind::Stockham;
    RadixPlan radix;  // Stockham radix, Rader's stockham part, or Bluestein convolution
    std::vector<RaderPrimePlan> primes;
    size_t convolution_len = 0;
};

struct AxisPlan {
    size_t axis = 0, logical_len = 0, effective_fft_len = 0;
    AxisAlgorithm algorithm;
    size_t estimated_scratch_complex = 0;
};

enum class AxisClass { Contiguous = 0, Strided = 1 };

struct FftPlan {
    FftConfig config;
    std::vector<AxisPlan> axes;
    int axis_class_override = -1;  // -1: none
    bool use_bluestein_override = false;

    static FftPlan build(const FftConfig &c);                                        // planner.rs:106
    static FftPlan build_for_device(const FftConfig &c, const DeviceProfile &d);    // planner.rs:115
    static FftPlan build_c2c_child_for_device(const FftConfig &c, const DeviceProfile &d, AxisClass cls);
};

// planner.rs free functions
std::vector<size_t> prime_factorization(size_t value);
std::vector<size_t> merged_radix_schedule(size_t value);
size_t primitive_root(size_t prime);  // 0 if none
size_t next_smooth_at_least(size_t target, const std::vector<size_t> &primes);
bool is_smooth(size_t value, const std::vector<size_t> &primes);
AxisAlgorithm plan_axis_algorithm(size_t len, const PlannerTuning &tuning);

// scheduler.rs:361-373
size_t upstream_bluestein_auto_padding(size_t sequence_len, size_t batch_count, Precision p,
                                       const DeviceProfile &d);

// real_ir.rs:1124-1213
enum class RealAlgorithm { FullComplex = 0, EvenHalfSize = 1 };
RealAlgorithm real_fft_algorithm_for_device(size_t length, size_t batch_count, Precision p,
                                            const PlannerTuning &tuning, const DeviceProfile &d);

void fill_axis_info(const AxisPlan &a, b200fft_axis_info &out);

}  // namespace b200fft
