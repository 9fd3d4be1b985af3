/*
 * b200fft -- C ABI of the B200-native FFT engine for the vkfft-rs transform hot path.
 *
 * Every entry point below replaces one item of the vkfft-rs Rust surface
 * (file:line refer to the crate's sources).  Plain C types only: fixed-width
 * integers, plain pointers and sizes, an opaque stream pointer (cudaStream_t).
 *
 * Conventions
 *   - dimensions are ordered slowest -> fastest (config.rs:662-666); the last
 *     axis is contiguous.
 *   - complex data is interleaved (re, im), like Complex<T> (complex.rs:3-12).
 *   - every call returns a b200fft_status; on failure the message is available
 *     from b200fft_last_error_string() (thread-local), like VkFftError's Display
 *     (error.rs:59-125).  Validation errors are returned before any GPU work.
 *   - planning calls (config / plan / transform build) never touch a GPU.
 */
#ifndef B200FFT_H
#define B200FFT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200FFT_ABI_VERSION 1
#define B200FFT_MAX_DIMS 8
#define B200FFT_MAX_FACTORS 64
#define B200FFT_MAX_RADER_PRIMES 16

/* VkFftError variants, in declaration order (error.rs:6-57). */
typedef enum b200fft_status {
    B200FFT_OK = 0,
    B200FFT_EMPTY_DIMENSIONS = 1,
    B200FFT_ZERO_LENGTH = 2,
    B200FFT_ZERO_BATCH_COUNT = 3,
    B200FFT_ARITHMETIC_OVERFLOW = 4,
    B200FFT_INVALID_TRANSFORM_LENGTH = 5,
    B200FFT_INVALID_KERNEL_IR = 6,
    B200FFT_INVALID_LUT = 7,
    B200FFT_UNSUPPORTED_KERNEL_PATH = 8,
    B200FFT_UNSUPPORTED_PRECISION = 9,
    B200FFT_RESOURCE_LIMIT_EXCEEDED = 10,
    B200FFT_INPUT_LENGTH_MISMATCH = 11,
    B200FFT_VALUE_OUT_OF_RANGE = 12,
    B200FFT_INVALID_ZERO_PADDING_RANGE = 13,
    B200FFT_SHADER_COMPILATION = 14,
    B200FFT_VULKAN_UNAVAILABLE = 15,
    B200FFT_VULKAN_RUNTIME = 16,
    B200FFT_NATIVE_UNAVAILABLE = 17,
    B200FFT_NATIVE_RUNTIME = 18,
    B200FFT_INVALID_PLANNER_TUNING = 19
} b200fft_status;

/* config.rs:3-16 */
typedef enum b200fft_direction { B200FFT_FORWARD = 0, B200FFT_INVERSE = 1 } b200fft_direction;

/* config.rs:35-42 (DCT/DST kinds are accepted by the planner, rejected by execution) */
typedef enum b200fft_transform_kind {
    B200FFT_C2C = 0,
    B200FFT_R2C = 1,
    B200FFT_C2R = 2,
    B200FFT_DCT1 = 3, B200FFT_DCT2 = 4, B200FFT_DCT3 = 5, B200FFT_DCT4 = 6,
    B200FFT_DST1 = 7, B200FFT_DST2 = 8, B200FFT_DST3 = 9, B200FFT_DST4 = 10
} b200fft_transform_kind;

/* config.rs:107-115 */
typedef enum b200fft_precision {
    B200FFT_F16_STORAGE_F32_COMPUTE = 0,
    B200FFT_F32 = 1,
    B200FFT_F64 = 2,
    B200FFT_F64_COMPUTE_F32_STORAGE = 3,
    B200FFT_DOUBLE_DOUBLE = 4,
    B200FFT_DOUBLE_DOUBLE_F64_STORAGE = 5
} b200fft_precision;

/* config.rs:163-181 */
typedef enum b200fft_backend {
    B200FFT_BACKEND_VULKAN = 0, B200FFT_BACKEND_CUDA = 1, B200FFT_BACKEND_HIP = 2,
    B200FFT_BACKEND_OPENCL = 3, B200FFT_BACKEND_LEVEL_ZERO = 4, B200FFT_BACKEND_METAL = 5,
    B200FFT_BACKEND_CPU_REFERENCE = 6
} b200fft_backend;
typedef enum b200fft_vendor {
    B200FFT_VENDOR_NVIDIA = 0, B200FFT_VENDOR_AMD = 1, B200FFT_VENDOR_INTEL = 2,
    B200FFT_VENDOR_APPLE = 3, B200FFT_VENDOR_OTHER = 4
} b200fft_vendor;

/* PlannerTuning (config.rs:365-381) */
typedef struct b200fft_planner_tuning {
    uint64_t min_rader_direct_prime;
    uint64_t max_rader_direct_prime;
    uint64_t min_rader_fft_prime;
    uint64_t max_rader_fft_prime;
    int32_t allow_recursive_fft_rader;
    int32_t _reserved;
} b200fft_planner_tuning;

/* SubgroupProfile (config.rs:183-248) */
typedef struct b200fft_subgroup_profile {
    uint64_t size, min_size, max_size;
    int32_t required_size_compute_supported, compute_supported, basic_supported,
        shuffle_supported, shuffle_relative_supported, compute_full_subgroups;
} b200fft_subgroup_profile;

/* DeviceProfile (config.rs:250-282) */
typedef struct b200fft_device_profile {
    int32_t backend; /* b200fft_backend */
    int32_t vendor;  /* b200fft_vendor */
    uint32_t vendor_other_id;
    int32_t supports_f64;
    uint64_t shared_memory_bytes;
    uint64_t shared_memory_pow2_bytes;
    uint64_t max_threads_per_block;
    uint64_t max_workgroup_size[3];
    uint64_t coalesced_memory_bytes;
    uint64_t shared_banks;
    b200fft_subgroup_profile subgroup;
} b200fft_device_profile;

/* FftConfig (config.rs:609-676).  Optional<usize> fields use 0 for None. */
typedef struct b200fft_config {
    uint32_t rank; /* number of dimensions, 1..B200FFT_MAX_DIMS */
    uint32_t _pad0;
    uint64_t dimensions[B200FFT_MAX_DIMS];
    uint64_t batch_count;
    int32_t transform; /* b200fft_transform_kind */
    int32_t precision; /* b200fft_precision */
    int32_t normalize_inverse;
    int32_t perform_convolution;
    int32_t kernel_convolution;
    int32_t convolution_conjugation; /* 0 None, 1 Sequence, 2 Kernel (config.rs:592-598) */
    int32_t cross_power_spectrum_normalization;
    int32_t symmetric_convolution_kernel;
    uint64_t coordinate_features;
    uint64_t matrix_convolution;
    uint64_t convolution_kernel_count;
    b200fft_planner_tuning tuning;
    int32_t use_device_tuning;
    int32_t zero_padding_domain; /* 0 Spatial, 1 Frequency (config.rs:548-555) */
    int32_t has_zero_padding[B200FFT_MAX_DIMS];
    uint64_t zero_padding_left[B200FFT_MAX_DIMS];
    uint64_t zero_padding_right[B200FFT_MAX_DIMS];
    int32_t omit_dimension[B200FFT_MAX_DIMS];
    uint64_t grouped_batch[B200FFT_MAX_DIMS];
    uint64_t bandwidth_boost;
    uint64_t input_buffer_axis_strides[B200FFT_MAX_DIMS];
    uint64_t output_buffer_axis_strides[B200FFT_MAX_DIMS];
    uint64_t input_buffer_batch_stride;
    uint64_t output_buffer_batch_stride;
} b200fft_config;

/* AlgorithmKind (planner.rs:19-24) and RaderMode (planner.rs:32-36) */
typedef enum b200fft_algorithm { B200FFT_STOCKHAM = 0, B200FFT_RADER = 1, B200FFT_BLUESTEIN = 2 } b200fft_algorithm;
typedef enum b200fft_rader_mode { B200FFT_RADER_FFT_CONVOLUTION = 0, B200FFT_RADER_DIRECT = 1 } b200fft_rader_mode;

typedef struct b200fft_rader_prime {
    uint64_t prime, multiplicity, generator;
    int32_t mode; /* b200fft_rader_mode */
    uint32_t convolution_factor_count;
    uint64_t convolution_factors[B200FFT_MAX_FACTORS];
} b200fft_rader_prime;

/* AxisPlan (planner.rs:82-90) flattened */
typedef struct b200fft_axis_info {
    uint64_t axis, logical_len, effective_fft_len, estimated_scratch_complex;
    int32_t algorithm; /* b200fft_algorithm */
    uint32_t prime_factor_count;   /* Stockham/Rader: stockham radix; Bluestein: convolution */
    uint32_t merged_radix_count;
    uint32_t rader_prime_count;
    uint64_t convolution_len;      /* Bluestein only */
    uint64_t prime_factors[B200FFT_MAX_FACTORS];
    uint64_t merged_radices[B200FFT_MAX_FACTORS];
    b200fft_rader_prime rader_primes[B200FFT_MAX_RADER_PRIMES];
} b200fft_axis_info;

/* RealFftAlgorithm (real_ir.rs:36-40) */
typedef enum b200fft_real_algorithm { B200FFT_REAL_FULL_COMPLEX = 0, B200FFT_REAL_EVEN_HALF_SIZE = 1 } b200fft_real_algorithm;

/* TransformIr family (application.rs:31-45), the non-DD members */
typedef enum b200fft_family {
    B200FFT_FAMILY_COMPLEX_1D = 0, B200FFT_FAMILY_COMPLEX_ND = 1,
    B200FFT_FAMILY_REAL = 2, B200FFT_FAMILY_REAL_ND = 3,
    B200FFT_FAMILY_REAL_TO_REAL = 4, B200FFT_FAMILY_REAL_TO_REAL_ND = 5
} b200fft_family;

typedef struct b200fft_plan b200fft_plan;           /* FftPlan */
typedef struct b200fft_transform b200fft_transform; /* TransformIr + its device program */
typedef struct b200fft_context b200fft_context;     /* CudaExecutionContext */

/* ---- error reporting --------------------------------------------------- */
/* Display text of the last error on this thread (error.rs:59-125). */
const char *b200fft_last_error_string(void);
uint32_t b200fft_abi_version(void);

/* ---- configuration (config.rs) ------------------------------------------ */
/* FftConfig::new(dimensions) (config.rs:678-710) */
b200fft_status b200fft_config_init(b200fft_config *config, uint32_t rank, const uint64_t *dimensions);
/* FftConfig::validate (config.rs:1036-1460) */
b200fft_status b200fft_config_validate(const b200fft_config *config);
/* PlannerTuning::portable (config.rs:383-393) */
void b200fft_planner_tuning_portable(b200fft_planner_tuning *tuning);
/* PlannerTuning::for_device (config.rs:396-420) */
void b200fft_planner_tuning_for_device(const b200fft_device_profile *device, int32_t precision,
                                       b200fft_planner_tuning *tuning);
/* DeviceProfile::generic (config.rs:267-282) */
void b200fft_device_profile_generic(int32_t backend, int32_t vendor, uint32_t vendor_other_id,
                                    b200fft_device_profile *profile);

/* ---- planner (planner.rs) ------------------------------------------------ */
/* FftPlan::build (planner.rs:106-109): portable, device-neutral classification */
b200fft_status b200fft_plan_build(const b200fft_config *config, b200fft_plan **plan);
/* FftPlan::build_for_device (planner.rs:115-118) */
b200fft_status b200fft_plan_build_for_device(const b200fft_config *config,
                                             const b200fft_device_profile *device,
                                             b200fft_plan **plan);
/* FftPlan::build_c2c_child_for_device (planner.rs:122-135); axis_class 0 contiguous, 1 strided */
b200fft_status b200fft_plan_build_c2c_child_for_device(const b200fft_config *config,
                                                       const b200fft_device_profile *device,
                                                       int32_t axis_class, b200fft_plan **plan);
uint32_t b200fft_plan_axis_count(const b200fft_plan *plan);
/* plan.axes[axis] (planner.rs:82-90) */
b200fft_status b200fft_plan_axis_info(const b200fft_plan *plan, uint32_t axis, b200fft_axis_info *info);
void b200fft_plan_destroy(b200fft_plan *plan);
/* planner.rs:581-733 helpers */
uint64_t b200fft_next_smooth_at_least(uint64_t target);
uint64_t b200fft_primitive_root(uint64_t prime);
/* scheduler.rs:361-373 upstream_bluestein_auto_padding */
b200fft_status b200fft_bluestein_auto_padding(uint64_t sequence_len, uint64_t batch_count,
                                              int32_t precision,
                                              const b200fft_device_profile *device,
                                              uint64_t *padded);

/* ---- application (application.rs) ---------------------------------------- */
/* TransformIr::build(config, direction, device) (application.rs:48-167).  Host only:
 * resolves device tuning, runs the device planner and lowers the plan to the B200
 * launch program.  Device-side tables are uploaded lazily on first execution. */
b200fft_status b200fft_transform_build(const b200fft_config *config, int32_t direction,
                                       const b200fft_device_profile *device,
                                       b200fft_transform **transform);
void b200fft_transform_destroy(b200fft_transform *transform);
int32_t b200fft_transform_family(const b200fft_transform *transform);
int32_t b200fft_transform_direction(const b200fft_transform *transform);
/* TransformIr::batch_count (application.rs:185-200) */
uint64_t b200fft_transform_batch_count(const b200fft_transform *transform);
/* RealFftIr::algorithm / transform_len (real_ir.rs:266-280) of the real axis */
int32_t b200fft_transform_real_algorithm(const b200fft_transform *transform);
uint64_t b200fft_transform_real_transform_len(const b200fft_transform *transform);
/* The device-scored plan the transform executes (top level) */
const b200fft_plan *b200fft_transform_plan(const b200fft_transform *transform);
/* The 1D child plan executed for one tensor axis (nd_ir.rs:676-708 child plans;
 * real_ir.rs:326-345 internal plan for the real axis; for DCT/DST the internal FFT of
 * the axis's reduction, r2r_ir.rs:689-940) */
b200fft_status b200fft_transform_axis_child_info(const b200fft_transform *transform, uint32_t axis,
                                                 b200fft_axis_info *info);
/* Element counts (complex or real) of the logical input / output tensors: the sizes of
 * the host arrays of b200fft_execute_host, which are always dense (the reference packs
 * formatted layouts internally, nd_real_ir.rs:715-750). */
uint64_t b200fft_transform_input_elements(const b200fft_transform *transform);
uint64_t b200fft_transform_output_elements(const b200fft_transform *transform);
/* Element counts of the device buffers of b200fft_execute: with formatted buffer strides
 * (config.rs:893-1002) batch_stride x batch stored elements, otherwise the logical
 * counts.  Elements of a formatted output buffer outside the tensor are not written. */
uint64_t b200fft_transform_input_buffer_elements(const b200fft_transform *transform);
uint64_t b200fft_transform_output_buffer_elements(const b200fft_transform *transform);
int32_t b200fft_transform_input_is_real(const b200fft_transform *transform);
int32_t b200fft_transform_output_is_real(const b200fft_transform *transform);
/* Bytes of device scratch one execution needs (0 when every pass runs in place on chip). */
uint64_t b200fft_transform_workspace_bytes(const b200fft_transform *transform);
/* Generic (op-program) passes of the transform that run an ahead-of-time specialised
 * sm_100a kernel from the library's catalogue: returns their number (-1 for a null
 * transform) and stores the number of generic passes in *generic_passes; the others run
 * the precompiled interpreter kernel.  No counterpart in the reference (whose kernels
 * are generated and compiled at run time, backend/cuda/runtime.rs:300-368); nothing is
 * compiled at run time here.  Needs no GPU. */
int32_t b200fft_transform_specialised_passes(const b200fft_transform *transform, int32_t *generic_passes);
/* Number of kernel launches one execution issues. */
uint32_t b200fft_transform_launch_count(const b200fft_transform *transform);
/* The kernel kind of each launch of one execution, in order, one label per line (e.g.
 * "register stockham (tensor-map tiles)"), written NUL-terminated into buffer (at most
 * capacity bytes, truncated); returns the length the whole text needs, without the NUL.
 * No counterpart in the reference (introspection of this engine's launch list); needs no
 * GPU. */
uint64_t b200fft_transform_describe_passes(const b200fft_transform *transform, char *buffer, uint64_t capacity);

/* ---- execution runtime (backend/cuda/runtime.rs) ------------------------- */
/* CudaExecutionContext::probe (cuda/runtime.rs:979): number of CUDA devices, or
 * B200FFT_NATIVE_UNAVAILABLE when no driver/device is present. */
b200fft_status b200fft_probe(int32_t *device_count);
/* CudaExecutionContext::new(device_index) (cuda/runtime.rs:1058-1244) */
b200fft_status b200fft_context_create(int32_t device_ordinal, b200fft_context **context);
void b200fft_context_destroy(b200fft_context *context);
/* NativeRuntime::device_profile (native_runtime.rs:164); the profile the reference
 * would report for this device (cuda/runtime.rs:1204-1225). */
b200fft_status b200fft_context_device_profile(const b200fft_context *context,
                                              b200fft_device_profile *profile);
b200fft_status b200fft_context_device_name(const b200fft_context *context, char *name, size_t capacity);

/* Resident execution: device pointers, stream ordered, no host synchronisation
 * (execute_program_chain_complex32_into, cuda/runtime.rs:1775-1809).  in and out may
 * be equal.  workspace: NULL lets the context own the scratch (allocated on first
 * use), otherwise at least b200fft_transform_workspace_bytes bytes of device memory.
 * stream: a cudaStream_t, or NULL for the context's stream. */
b200fft_status b200fft_execute(b200fft_context *context, b200fft_transform *transform,
                               const void *input, void *output, void *workspace, void *stream);

/* Resident execution that allocates nothing.  No counterpart in the reference: it is
 * an addition of this engine for callers that cannot allocate device memory at call
 * time -- code running under a framework allocator that has reserved the device's
 * memory (a cudaMalloc there can fail), and latency-critical loops, where the
 * implicit device-wide synchronisation of cudaFree stalls other streams.
 * The transform's tables and scratch live in one library-owned device region of
 * B200FFT_STATIC_WORKSPACE_BYTES per device; its address is looked up on the first call
 * on each device.  A transform whose tables plus scratch
 * (b200fft_transform_workspace_bytes covers the scratch part) exceed the region is
 * rejected with B200FFT_RESOURCE_LIMIT_EXCEEDED and a message giving both sizes.
 * Nothing in the region has to start at zero.  Every call copies its transform's
 * tables in from host memory (a packed image the transform keeps from its first call)
 * ahead of its kernels, on the same stream.  The first call on a device also looks up
 * the region's address: make it before any stream capture.  Calls whose GPU work can
 * overlap -- on different streams, contexts or threads of one process -- share the
 * region and race: order them on one stream.  in and out as for b200fft_execute;
 * stream: a cudaStream_t, or NULL for the context's stream. */
#define B200FFT_STATIC_WORKSPACE_BYTES (16u << 20)
b200fft_status b200fft_execute_static_workspace(b200fft_context *context, b200fft_transform *transform,
                                                const void *input, void *output, void *stream);

/* Host execution with copy semantics: NativeRuntime::execute_transform_f32 / _f64
 * (native_runtime.rs:339-359).  Element type follows the precision (float or double);
 * real transforms take / return real arrays (NativeTransformInput32::Real).  Sizes in
 * bytes are checked (InputLengthMismatch).  Synchronous. */
b200fft_status b200fft_execute_host(b200fft_context *context, b200fft_transform *transform,
                                    const void *input, size_t input_bytes, void *output,
                                    size_t output_bytes);

/* ---- FFT convolution (convolution_ir.rs, native_runtime.rs:257-337) ----- */
typedef struct b200fft_convolution b200fft_convolution;
/* build_from_spectrum of the reference's convolution applications; config has
 * perform_convolution = 1 and selects the family:
 *  - transform R2C, rank >= 2: NdRealConvolutionIr (convolution_ir.rs:3867-4250), batch 1,
 *    coordinate_features C, K kernels: kernel_spectrum holds K*C compact R2C spectra
 *    (prod(dims[:-1]) * (dims[-1]/2+1) complex values each), or 1 broadcast to every system;
 *    spectrum_copies is 1 or K*C.
 *  - transform C2C, rank 1: ConvolutionIr (:2520-3626); rank >= 2: NdConvolutionIr
 *    (:3627-3866): kernel_spectrum holds planes*K tensors of prod(dims) complex values
 *    (planes = 1, or the 2x2 / 3x3 matrix planes, 3 for a symmetric 2x2);
 *    spectrum_copies = planes*K.
 * The input holds batch x coordinates systems, the output (K > 1 ? K : batch) x
 * coordinates systems; the inverse transform is normalised. */
b200fft_status b200fft_convolution_build(const b200fft_config *config,
                                         const b200fft_device_profile *device,
                                         const void *kernel_spectrum, uint64_t spectrum_copies,
                                         b200fft_convolution **convolution);
void b200fft_convolution_destroy(b200fft_convolution *convolution);
uint64_t b200fft_convolution_workspace_bytes(const b200fft_convolution *convolution);
/* As b200fft_transform_specialised_passes, for a convolution's launch list (no
 * counterpart in the reference). */
int32_t b200fft_convolution_specialised_passes(const b200fft_convolution *convolution, int32_t *generic_passes);
/* Element counts of the input / output arrays (real for the ND real convolution, complex
 * for ConvolutionIr / NdConvolutionIr). */
/* Logical elements of the host API's arrays (input C * full real tensor, output K * C). */
uint64_t b200fft_convolution_input_elements(const b200fft_convolution *convolution);
uint64_t b200fft_convolution_output_elements(const b200fft_convolution *convolution);
/* Elements of the device buffers b200fft_execute_convolution reads and writes: the
 * formatted layouts when the config sets buffer strides (scalar K = 1 ND real
 * convolution, convolution_ir.rs:3922-3928), else the logical counts. */
uint64_t b200fft_convolution_input_buffer_elements(const b200fft_convolution *convolution);
uint64_t b200fft_convolution_output_buffer_elements(const b200fft_convolution *convolution);
int32_t b200fft_convolution_input_is_real(const b200fft_convolution *convolution);
/* execute_nd_real_convolution_f32/f64 on device pointers (stream ordered). */
b200fft_status b200fft_execute_convolution(b200fft_context *context, b200fft_convolution *convolution,
                                           const void *input, void *output, void *workspace,
                                           void *stream);
/* Same with host arrays and copy semantics. */
b200fft_status b200fft_execute_convolution_host(b200fft_context *context,
                                                b200fft_convolution *convolution,
                                                const void *input, size_t input_bytes, void *output,
                                                size_t output_bytes);

/* ---- multi-GPU slab decomposition ---------------------------------------
 * No counterpart in the reference (a single-device crate); the multi-GPU form of
 * TransformIr::build + execute for rank >= 2 C2C and rank >= 3 R2C / C2R tensors, batch 1,
 * one process per GPU.  Rank g of P owns planes [g D0/P, (g+1) D0/P) of axis 0.
 *   forward input  [D0/P, D1, ...]        (real for R2C)
 *   forward output [D0, D1/P, ...']       axis-1 indices [g D1/P, (g+1) D1/P); the last
 *                                         axis is compact (N/2+1) for R2C
 *   inverse input / output: the forward output / input layouts.
 * D0 and D1 must be divisible by P (at most 8).  The exchange (the all-to-all transpose)
 * is done by the last FFT pass before it, which stores straight into the owner rank's
 * exchange buffer through CUDA IPC peer mappings, followed by a device-side barrier with
 * a bounded wait (b200fft_slab_set_timeout; on expiry the context's error word records
 * it, see b200fft_context_synchronize).  Set-up per rank: build, attach (allocates the
 * exchange buffers and returns this rank's handle), gather every rank's handle by any
 * means (e.g. torch.distributed.all_gather_object), connect.  Every rank must execute
 * the same sequence of slab calls; a slab must be destroyed before its context. */
#define B200FFT_SLAB_HANDLE_BYTES 128
typedef struct b200fft_slab b200fft_slab;
typedef struct b200fft_slab_info {
    uint32_t nranks, rank;
    uint64_t planes_per_rank;   /* D0 / nranks */
    uint64_t columns_per_rank;  /* D1 / nranks */
    uint64_t input_elements;    /* per rank, elements of the input's type (float/double or complex) */
    uint64_t output_elements;
    int32_t input_is_real, output_is_real;
    uint64_t exchange_bytes;    /* device memory b200fft_slab_attach allocates */
    uint32_t launch_count;      /* kernel launches of one execution (barrier included) */
} b200fft_slab_info;
b200fft_status b200fft_slab_build(const b200fft_config *config, int32_t direction, uint32_t nranks,
                                  uint32_t rank, const b200fft_device_profile *device,
                                  b200fft_slab **slab);
void b200fft_slab_destroy(b200fft_slab *slab);
b200fft_status b200fft_slab_get_info(const b200fft_slab *slab, b200fft_slab_info *info);
b200fft_status b200fft_slab_set_timeout(b200fft_slab *slab, uint64_t timeout_ns);
/* handle: B200FFT_SLAB_HANDLE_BYTES bytes written for this rank. */
b200fft_status b200fft_slab_attach(b200fft_context *context, b200fft_slab *slab, void *handle);
/* handles: nranks consecutive handles, rank order.  Fails if two ranks share a GPU. */
b200fft_status b200fft_slab_connect(b200fft_context *context, b200fft_slab *slab, const void *handles);
/* Phase timing (profiling; no counterpart in the reference): once enabled (after
 * attach), every execution records CUDA events around its phases, and
 * b200fft_slab_phase_times waits for the last execution and writes ms[4] = the local
 * passes before the exchange, the exchange pass (the FFT pass whose stores land in the
 * ranks' buffers), the barrier, and the passes after it. */
b200fft_status b200fft_slab_set_phase_timing(b200fft_slab *slab, int32_t enabled);
b200fft_status b200fft_slab_phase_times(b200fft_slab *slab, float *ms);
/* Stream ordered, device pointers; input and output must not overlap.  workspace as for
 * b200fft_execute (NULL: context-owned scratch). */
b200fft_status b200fft_execute_slab(b200fft_context *context, b200fft_slab *slab, const void *input,
                                    void *output, void *workspace, void *stream);

/* ---- asynchronous submission (NativeAsyncRuntime, native_runtime.rs:362-451) -------
 * submit_transform_f32_async / _f64_async: queues a host execution with the semantics of
 * b200fft_execute_host and returns a ticket at once.  The input array must stay alive and
 * unchanged, and the output array unread, until the ticket is waited for.  Submissions on
 * one context run in submission order on a worker thread; the transform must outlive its
 * tickets.  b200fft_ticket_wait returns the execution's status (the error text through
 * b200fft_last_error_string on the waiting thread) and frees the ticket; _destroy waits
 * and frees without reporting. */
typedef struct b200fft_ticket b200fft_ticket;
b200fft_status b200fft_submit_host(b200fft_context *context, b200fft_transform *transform,
                                   const void *input, size_t input_bytes, void *output,
                                   size_t output_bytes, b200fft_ticket **ticket);
b200fft_status b200fft_ticket_wait(b200fft_ticket *ticket);
void b200fft_ticket_destroy(b200fft_ticket *ticket);

/* Waits for the stream (NULL: the context's) and reports any error the context's kernels
 * recorded since the last check (bounded waits that expired, invalid programs) as
 * NativeRuntime, clearing it. */
b200fft_status b200fft_context_synchronize(b200fft_context *context, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* B200FFT_H */
