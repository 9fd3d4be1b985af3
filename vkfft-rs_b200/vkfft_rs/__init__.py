"""Python mirror of the vkfft-rs transform API over the B200 C ABI (include/b200fft.h).

Names and argument meaning follow the Rust crate so code and tests read like the
reference's own:

    FftConfig(dims).with_batch_count(b).with_precision(Precision.F64)   # config.rs:609-1034
    FftPlan.build(cfg) / FftPlan.build_for_device(cfg, device)           # planner.rs:106-118
    TransformIr.build(cfg, Direction.FORWARD, device)                    # application.rs:48
    ctx = CudaExecutionContext(0); ctx.execute_transform(ir, x)          # cuda/runtime.rs:2311
    ctx.execute_resident(ir, in_ptr, out_ptr, stream=...)                # resident chain "into"

Errors raise VkFftError carrying the C status (the VkFftError variant name) and the
reference's Display text.  The native library is required: there is no fallback
path, and importing this module on a machine without the built library fails.
"""
import ctypes
import enum
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_PKG = os.path.dirname(_HERE)
LIB_PATH = os.path.join(_PKG, "libb200fft.so")

MAX_DIMS = 8
MAX_FACTORS = 64
MAX_RADER = 16


class Status(enum.IntEnum):
    OK = 0
    EmptyDimensions = 1
    ZeroLength = 2
    ZeroBatchCount = 3
    ArithmeticOverflow = 4
    InvalidTransformLength = 5
    InvalidKernelIr = 6
    InvalidLut = 7
    UnsupportedKernelPath = 8
    UnsupportedPrecision = 9
    ResourceLimitExceeded = 10
    InputLengthMismatch = 11
    ValueOutOfRange = 12
    InvalidZeroPaddingRange = 13
    ShaderCompilation = 14
    VulkanUnavailable = 15
    VulkanRuntime = 16
    NativeUnavailable = 17
    NativeRuntime = 18
    InvalidPlannerTuning = 19


class VkFftError(Exception):
    """error.rs:6-57: .status is the variant, str() is the Display text."""

    def __init__(self, status, message):
        super().__init__(message)
        self.status = Status(status)
        self.message = message

    @property
    def variant(self):
        return self.status.name


class Direction(enum.IntEnum):
    FORWARD = 0
    INVERSE = 1


class TransformKind(enum.IntEnum):
    C2C = 0
    R2C = 1
    C2R = 2
    DCT1 = 3
    DCT2 = 4
    DCT3 = 5
    DCT4 = 6
    DST1 = 7
    DST2 = 8
    DST3 = 9
    DST4 = 10


class Precision(enum.IntEnum):
    F16_STORAGE_F32_COMPUTE = 0
    F32 = 1
    F64 = 2
    F64_COMPUTE_F32_STORAGE = 3
    DOUBLE_DOUBLE = 4
    DOUBLE_DOUBLE_F64_STORAGE = 5


class Backend(enum.IntEnum):
    VULKAN = 0
    CUDA = 1
    HIP = 2
    OPENCL = 3
    LEVEL_ZERO = 4
    METAL = 5
    CPU_REFERENCE = 6


class GpuVendor(enum.IntEnum):
    NVIDIA = 0
    AMD = 1
    INTEL = 2
    APPLE = 3
    OTHER = 4


class AlgorithmKind(enum.IntEnum):
    STOCKHAM = 0
    RADER = 1
    BLUESTEIN = 2


class RaderMode(enum.IntEnum):
    FFT_CONVOLUTION = 0
    DIRECT_MULTIPLICATION = 1


class ZeroPaddingDomain(enum.IntEnum):
    """config.rs:548-555: which transform boundary owns the zero-padding interval."""
    SPATIAL = 0
    FREQUENCY = 1


class RealFftAlgorithm(enum.IntEnum):
    FULL_COMPLEX = 0
    EVEN_HALF_SIZE = 1


class Family(enum.IntEnum):
    COMPLEX_1D = 0
    COMPLEX_ND = 1
    REAL = 2
    REAL_ND = 3
    REAL_TO_REAL = 4
    REAL_TO_REAL_ND = 5


u64 = ctypes.c_uint64
i32 = ctypes.c_int32
u32 = ctypes.c_uint32


class _Tuning(ctypes.Structure):
    _fields_ = [("min_rader_direct_prime", u64), ("max_rader_direct_prime", u64),
                ("min_rader_fft_prime", u64), ("max_rader_fft_prime", u64),
                ("allow_recursive_fft_rader", i32), ("_reserved", i32)]


class _Subgroup(ctypes.Structure):
    _fields_ = [("size", u64), ("min_size", u64), ("max_size", u64),
                ("required_size_compute_supported", i32), ("compute_supported", i32),
                ("basic_supported", i32), ("shuffle_supported", i32),
                ("shuffle_relative_supported", i32), ("compute_full_subgroups", i32)]


class _Device(ctypes.Structure):
    _fields_ = [("backend", i32), ("vendor", i32), ("vendor_other_id", u32), ("supports_f64", i32),
                ("shared_memory_bytes", u64), ("shared_memory_pow2_bytes", u64),
                ("max_threads_per_block", u64), ("max_workgroup_size", u64 * 3),
                ("coalesced_memory_bytes", u64), ("shared_banks", u64), ("subgroup", _Subgroup)]


class _Config(ctypes.Structure):
    _fields_ = [("rank", u32), ("_pad0", u32), ("dimensions", u64 * MAX_DIMS), ("batch_count", u64),
                ("transform", i32), ("precision", i32), ("normalize_inverse", i32),
                ("perform_convolution", i32), ("kernel_convolution", i32),
                ("convolution_conjugation", i32), ("cross_power_spectrum_normalization", i32),
                ("symmetric_convolution_kernel", i32), ("coordinate_features", u64),
                ("matrix_convolution", u64), ("convolution_kernel_count", u64), ("tuning", _Tuning),
                ("use_device_tuning", i32), ("zero_padding_domain", i32),
                ("has_zero_padding", i32 * MAX_DIMS), ("zero_padding_left", u64 * MAX_DIMS),
                ("zero_padding_right", u64 * MAX_DIMS), ("omit_dimension", i32 * MAX_DIMS),
                ("grouped_batch", u64 * MAX_DIMS), ("bandwidth_boost", u64),
                ("input_buffer_axis_strides", u64 * MAX_DIMS),
                ("output_buffer_axis_strides", u64 * MAX_DIMS),
                ("input_buffer_batch_stride", u64), ("output_buffer_batch_stride", u64)]


class _RaderPrime(ctypes.Structure):
    _fields_ = [("prime", u64), ("multiplicity", u64), ("generator", u64), ("mode", i32),
                ("convolution_factor_count", u32), ("convolution_factors", u64 * MAX_FACTORS)]


class _SlabInfo(ctypes.Structure):
    _fields_ = [("nranks", u32), ("rank", u32), ("planes_per_rank", u64), ("columns_per_rank", u64),
                ("input_elements", u64), ("output_elements", u64), ("input_is_real", i32),
                ("output_is_real", i32), ("exchange_bytes", u64), ("launch_count", u32)]


SLAB_HANDLE_BYTES = 128


class _AxisInfo(ctypes.Structure):
    _fields_ = [("axis", u64), ("logical_len", u64), ("effective_fft_len", u64),
                ("estimated_scratch_complex", u64), ("algorithm", i32), ("prime_factor_count", u32),
                ("merged_radix_count", u32), ("rader_prime_count", u32), ("convolution_len", u64),
                ("prime_factors", u64 * MAX_FACTORS), ("merged_radices", u64 * MAX_FACTORS),
                ("rader_primes", _RaderPrime * MAX_RADER)]


_lib = None


def library():
    """Load libb200fft.so (fails loudly when it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C vkfft-rs_b200` "
                          "or __graft_entry__.build()")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    vp = ctypes.c_void_p
    sigs = {
        "b200fft_last_error_string": ([], ctypes.c_char_p),
        "b200fft_abi_version": ([], u32),
        "b200fft_config_init": ([P(_Config), u32, P(u64)], i32),
        "b200fft_config_validate": ([P(_Config)], i32),
        "b200fft_planner_tuning_portable": ([P(_Tuning)], None),
        "b200fft_planner_tuning_for_device": ([P(_Device), i32, P(_Tuning)], None),
        "b200fft_device_profile_generic": ([i32, i32, u32, P(_Device)], None),
        "b200fft_plan_build": ([P(_Config), P(vp)], i32),
        "b200fft_plan_build_for_device": ([P(_Config), P(_Device), P(vp)], i32),
        "b200fft_plan_build_c2c_child_for_device": ([P(_Config), P(_Device), i32, P(vp)], i32),
        "b200fft_plan_axis_count": ([vp], u32),
        "b200fft_plan_axis_info": ([vp, u32, P(_AxisInfo)], i32),
        "b200fft_plan_destroy": ([vp], None),
        "b200fft_next_smooth_at_least": ([u64], u64),
        "b200fft_primitive_root": ([u64], u64),
        "b200fft_bluestein_auto_padding": ([u64, u64, i32, P(_Device), P(u64)], i32),
        "b200fft_transform_build": ([P(_Config), i32, P(_Device), P(vp)], i32),
        "b200fft_transform_destroy": ([vp], None),
        "b200fft_transform_family": ([vp], i32),
        "b200fft_transform_direction": ([vp], i32),
        "b200fft_transform_batch_count": ([vp], u64),
        "b200fft_transform_real_algorithm": ([vp], i32),
        "b200fft_transform_real_transform_len": ([vp], u64),
        "b200fft_transform_plan": ([vp], vp),
        "b200fft_transform_axis_child_info": ([vp, u32, P(_AxisInfo)], i32),
        "b200fft_transform_input_elements": ([vp], u64),
        "b200fft_transform_output_elements": ([vp], u64),
        "b200fft_transform_input_buffer_elements": ([vp], u64),
        "b200fft_transform_output_buffer_elements": ([vp], u64),
        "b200fft_transform_input_is_real": ([vp], i32),
        "b200fft_transform_output_is_real": ([vp], i32),
        "b200fft_transform_workspace_bytes": ([vp], u64),
        "b200fft_transform_launch_count": ([vp], u32),
        "b200fft_transform_specialised_passes": ([vp, P(i32)], i32),
        "b200fft_transform_describe_passes": ([vp, ctypes.c_char_p, ctypes.c_uint64], ctypes.c_uint64),
        "b200fft_probe": ([P(i32)], i32),
        "b200fft_context_create": ([i32, P(vp)], i32),
        "b200fft_context_destroy": ([vp], None),
        "b200fft_context_device_profile": ([vp, P(_Device)], i32),
        "b200fft_context_device_name": ([vp, ctypes.c_char_p, ctypes.c_size_t], i32),
        "b200fft_execute": ([vp, vp, vp, vp, vp, vp], i32),
        "b200fft_execute_static_workspace": ([vp, vp, vp, vp, vp], i32),
        "b200fft_execute_host": ([vp, vp, vp, ctypes.c_size_t, vp, ctypes.c_size_t], i32),
        "b200fft_convolution_build": ([P(_Config), P(_Device), vp, u64, P(vp)], i32),
        "b200fft_convolution_destroy": ([vp], None),
        "b200fft_convolution_workspace_bytes": ([vp], u64),
        "b200fft_convolution_specialised_passes": ([vp, P(i32)], i32),
        "b200fft_convolution_input_elements": ([vp], u64),
        "b200fft_convolution_output_elements": ([vp], u64),
        "b200fft_convolution_input_is_real": ([vp], i32),
        "b200fft_convolution_input_buffer_elements": ([vp], u64),
        "b200fft_convolution_output_buffer_elements": ([vp], u64),
        "b200fft_execute_convolution": ([vp, vp, vp, vp, vp, vp], i32),
        "b200fft_execute_convolution_host": ([vp, vp, vp, ctypes.c_size_t, vp, ctypes.c_size_t], i32),
        "b200fft_slab_build": ([P(_Config), i32, u32, u32, P(_Device), P(vp)], i32),
        "b200fft_slab_destroy": ([vp], None),
        "b200fft_slab_get_info": ([vp, P(_SlabInfo)], i32),
        "b200fft_slab_set_phase_timing": ([vp, i32], i32),
        "b200fft_slab_phase_times": ([vp, P(ctypes.c_float)], i32),
        "b200fft_slab_set_timeout": ([vp, u64], i32),
        "b200fft_slab_attach": ([vp, vp, vp], i32),
        "b200fft_slab_connect": ([vp, vp, vp], i32),
        "b200fft_execute_slab": ([vp, vp, vp, vp, vp, vp], i32),
        "b200fft_context_synchronize": ([vp, vp], i32),
        "b200fft_submit_host": ([vp, vp, vp, ctypes.c_size_t, vp, ctypes.c_size_t, P(vp)], i32),
        "b200fft_ticket_wait": ([vp], i32),
        "b200fft_ticket_destroy": ([vp], None),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


EXPORTED_SYMBOLS = None  # filled lazily by exported_symbols()


def _check(status):
    if status != 0:
        msg = library().b200fft_last_error_string().decode()
        raise VkFftError(status, msg)


# ---- config.rs -----------------------------------------------------------------

class PlannerTuning:
    """config.rs:365-544"""

    def __init__(self, min_rader_direct_prime=17, max_rader_direct_prime=89, min_rader_fft_prime=17,
                 max_rader_fft_prime=16384, allow_recursive_fft_rader=False):
        self.min_rader_direct_prime = min_rader_direct_prime
        self.max_rader_direct_prime = max_rader_direct_prime
        self.min_rader_fft_prime = min_rader_fft_prime
        self.max_rader_fft_prime = max_rader_fft_prime
        self.allow_recursive_fft_rader = allow_recursive_fft_rader

    @classmethod
    def portable(cls):
        return cls()

    @classmethod
    def for_device(cls, device, precision):
        t = _Tuning()
        library().b200fft_planner_tuning_for_device(ctypes.byref(device._c()), int(precision), ctypes.byref(t))
        return cls._from_c(t)

    def with_recursive_fft_rader(self, enabled):
        t = PlannerTuning(**vars(self))
        t.allow_recursive_fft_rader = enabled
        return t

    def _c(self):
        return _Tuning(self.min_rader_direct_prime, self.max_rader_direct_prime, self.min_rader_fft_prime,
                       self.max_rader_fft_prime, int(self.allow_recursive_fft_rader), 0)

    @classmethod
    def _from_c(cls, t):
        return cls(t.min_rader_direct_prime, t.max_rader_direct_prime, t.min_rader_fft_prime,
                   t.max_rader_fft_prime, bool(t.allow_recursive_fft_rader))

    def __eq__(self, other):
        return vars(self) == vars(other)

    def __repr__(self):
        return f"PlannerTuning({vars(self)})"


class DeviceProfile:
    """config.rs:250-282"""

    def __init__(self, c):
        self._s = c

    @classmethod
    def generic(cls, backend, vendor, other_id=0):
        c = _Device()
        library().b200fft_device_profile_generic(int(backend), int(vendor), other_id, ctypes.byref(c))
        return cls(c)

    def replace(self, **kw):
        c = _Device()
        ctypes.memmove(ctypes.byref(c), ctypes.byref(self._s), ctypes.sizeof(_Device))
        for k, v in kw.items():
            if k == "max_workgroup_size":
                for i, x in enumerate(v):
                    c.max_workgroup_size[i] = x
            else:
                setattr(c, k, int(v))
        return DeviceProfile(c)

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        v = getattr(self._s, name)
        if name == "max_workgroup_size":
            return list(v)
        return v

    def _c(self):
        return self._s


class FftConfig:
    """config.rs:609-1034 (builder methods return new configs, like the Rust by-value builders)."""

    def __init__(self, dimensions):
        dims = [int(d) for d in dimensions]
        self._s = _Config()
        arr = (u64 * max(1, len(dims)))(*dims) if dims else None
        _check(library().b200fft_config_init(ctypes.byref(self._s), len(dims), arr))

    def _copy(self):
        c = FftConfig.__new__(FftConfig)
        c._s = _Config()
        ctypes.memmove(ctypes.byref(c._s), ctypes.byref(self._s), ctypes.sizeof(_Config))
        return c

    def _set(self, **kw):
        c = self._copy()
        for k, v in kw.items():
            setattr(c._s, k, v)
        return c

    @property
    def dimensions(self):
        return [self._s.dimensions[i] for i in range(self._s.rank)]

    @property
    def batch_count(self):
        return self._s.batch_count

    @property
    def precision(self):
        return Precision(self._s.precision)

    @property
    def transform(self):
        return TransformKind(self._s.transform)

    @property
    def tuning(self):
        return PlannerTuning._from_c(self._s.tuning)

    def with_batch_count(self, n):
        return self._set(batch_count=int(n))

    def with_precision(self, p):
        return self._set(precision=int(p))

    def with_transform(self, t):
        return self._set(transform=int(t))

    def with_inverse_normalization(self, normalize):
        return self._set(normalize_inverse=int(bool(normalize)))

    def with_tuning(self, tuning):
        c = self._set(use_device_tuning=0)
        c._s.tuning = tuning._c()
        return c

    def with_device_tuning(self):
        c = self._set(use_device_tuning=1)
        c._s.tuning = PlannerTuning.portable()._c()
        return c

    def with_convolution(self, enabled):
        return self._set(perform_convolution=int(bool(enabled)))

    def with_kernel_convolution(self, enabled):
        return self._set(kernel_convolution=int(bool(enabled)))

    def with_coordinate_features(self, n):
        return self._set(coordinate_features=int(n))

    def with_matrix_convolution(self, m):
        c = self._set(matrix_convolution=int(m))
        if m > 1:
            c._s.coordinate_features = int(m)
        return c

    def with_convolution_kernel_count(self, k):
        return self._set(convolution_kernel_count=int(k))

    def with_convolution_conjugation(self, mode):
        return self._set(convolution_conjugation=int(mode))

    def with_cross_power_spectrum_normalization(self, enabled):
        return self._set(cross_power_spectrum_normalization=int(bool(enabled)))

    def with_symmetric_convolution_kernel(self, enabled):
        return self._set(symmetric_convolution_kernel=int(bool(enabled)))

    def with_bandwidth_boost(self, b):
        return self._set(bandwidth_boost=int(b))

    def _axis_check(self, axis, field):
        if axis >= self._s.rank:
            raise VkFftError(Status.ValueOutOfRange,
                             f"{field} cannot be represented by the current backend index type")

    def with_zero_padding(self, axis, left, right):
        if axis >= self._s.rank or left > right or right > self._s.dimensions[axis]:
            length = self._s.dimensions[axis] if axis < self._s.rank else 0
            raise VkFftError(Status.InvalidZeroPaddingRange,
                             f"zero-padding interval [{left}, {right}) is invalid for axis {axis} "
                             f"of length {length}")
        c = self._copy()
        c._s.has_zero_padding[axis] = int(left != right)
        c._s.zero_padding_left[axis] = left
        c._s.zero_padding_right[axis] = right
        return c

    def with_zero_padding_domain(self, domain):
        return self._set(zero_padding_domain=int(domain))

    def with_omit_dimension(self, axis, omit):
        self._axis_check(axis, "omitDimension axis")
        c = self._copy()
        c._s.omit_dimension[axis] = int(bool(omit))
        return c

    def with_grouped_batch(self, axis, grouped):
        self._axis_check(axis, "groupedBatch axis")
        c = self._copy()
        c._s.grouped_batch[axis] = int(grouped)
        return c

    def with_input_buffer_axis_stride(self, axis, stride):
        self._axis_check(axis, "formatted input axis stride")
        c = self._copy()
        c._s.input_buffer_axis_strides[axis] = int(stride)
        return c

    def with_output_buffer_axis_stride(self, axis, stride):
        self._axis_check(axis, "formatted output axis stride")
        c = self._copy()
        c._s.output_buffer_axis_strides[axis] = int(stride)
        return c

    def with_input_buffer_batch_stride(self, stride):
        return self._set(input_buffer_batch_stride=int(stride))

    def with_output_buffer_batch_stride(self, stride):
        return self._set(output_buffer_batch_stride=int(stride))

    def validate(self):
        _check(library().b200fft_config_validate(ctypes.byref(self._s)))


# ---- planner.rs ------------------------------------------------------------------

class RadixPlan:
    def __init__(self, prime_factors, merged_radices):
        self.prime_factors = prime_factors
        self.merged_radices = merged_radices


class RaderPrimePlan:
    def __init__(self, r):
        self.prime = r.prime
        self.multiplicity = r.multiplicity
        self.generator = r.generator
        self.mode = RaderMode(r.mode)
        self.convolution = RadixPlan(list(r.convolution_factors[:r.convolution_factor_count]), None)


class AxisPlan:
    """planner.rs:82-90 with AxisAlgorithm flattened (kind, radix, primes, convolution_len)."""

    def __init__(self, info):
        self.axis = info.axis
        self.logical_len = info.logical_len
        self.effective_fft_len = info.effective_fft_len
        self.estimated_scratch_complex = info.estimated_scratch_complex
        self.kind = AlgorithmKind(info.algorithm)
        self.radix = RadixPlan(list(info.prime_factors[:info.prime_factor_count]),
                               list(info.merged_radices[:info.merged_radix_count]))
        self.primes = [RaderPrimePlan(info.rader_primes[i]) for i in range(info.rader_prime_count)]
        self.convolution_len = info.convolution_len if self.kind == AlgorithmKind.BLUESTEIN else None

    def __repr__(self):
        extra = ""
        if self.kind == AlgorithmKind.BLUESTEIN:
            extra = f", convolution_len={self.convolution_len}"
        elif self.kind == AlgorithmKind.RADER:
            extra = ", primes=" + str([(p.prime, p.mode.name) for p in self.primes])
        return f"AxisPlan(axis={self.axis}, len={self.logical_len}, {self.kind.name}{extra})"


def _axes_of(handle):
    lib = library()
    out = []
    for a in range(lib.b200fft_plan_axis_count(handle)):
        info = _AxisInfo()
        _check(lib.b200fft_plan_axis_info(handle, a, ctypes.byref(info)))
        out.append(AxisPlan(info))
    return out


class FftPlan:
    """planner.rs:92-242"""

    def __init__(self, handle):
        self.axes = _axes_of(handle)
        library().b200fft_plan_destroy(handle)

    @classmethod
    def build(cls, config):
        h = ctypes.c_void_p()
        _check(library().b200fft_plan_build(ctypes.byref(config._s), ctypes.byref(h)))
        return cls(h)

    @classmethod
    def build_for_device(cls, config, device):
        h = ctypes.c_void_p()
        _check(library().b200fft_plan_build_for_device(ctypes.byref(config._s), ctypes.byref(device._c()),
                                                       ctypes.byref(h)))
        return cls(h)

    @classmethod
    def build_c2c_child_for_device(cls, config, device, strided):
        h = ctypes.c_void_p()
        _check(library().b200fft_plan_build_c2c_child_for_device(
            ctypes.byref(config._s), ctypes.byref(device._c()), int(bool(strided)), ctypes.byref(h)))
        return cls(h)


def next_smooth_at_least(target):
    return int(library().b200fft_next_smooth_at_least(target))


def primitive_root(prime):
    r = int(library().b200fft_primitive_root(prime))
    return r or None


def upstream_bluestein_auto_padding(sequence_len, batch_count, precision, device):
    out = u64()
    _check(library().b200fft_bluestein_auto_padding(sequence_len, batch_count, int(precision),
                                                    ctypes.byref(device._c()), ctypes.byref(out)))
    return int(out.value)


# ---- application.rs ----------------------------------------------------------------

# host-API array types (execute_transform_f32 / _f64): mixed precisions take the API type,
# the device buffers of execute_resident hold the storage type (float16 / float32)
_np_dtype = {
    (Precision.F32, True): np.float32, (Precision.F32, False): np.complex64,
    (Precision.F64, True): np.float64, (Precision.F64, False): np.complex128,
    (Precision.F16_STORAGE_F32_COMPUTE, True): np.float32, (Precision.F16_STORAGE_F32_COMPUTE, False): np.complex64,
    (Precision.F64_COMPUTE_F32_STORAGE, True): np.float64, (Precision.F64_COMPUTE_F32_STORAGE, False): np.complex128,
    # double-double: float64 words, (hi, lo) per real and (re.hi, re.lo, im.hi, im.lo) per
    # complex element (the reference's DD buffer layout, double_double.rs encode_complex_double_double)
    (Precision.DOUBLE_DOUBLE, True): np.float64, (Precision.DOUBLE_DOUBLE, False): np.float64,
    (Precision.DOUBLE_DOUBLE_F64_STORAGE, True): np.float64,
    (Precision.DOUBLE_DOUBLE_F64_STORAGE, False): np.complex128,
}


def _words(precision, real):
    """Array items per logical element: 2 (real) / 4 (complex) for double-double, else 1."""
    if precision == Precision.DOUBLE_DOUBLE:
        return 2 if real else 4
    return 1


class TransformIr:
    """application.rs:31-167.  Owns the lowered B200 launch program."""

    def __init__(self, handle, config):
        self._h = handle
        self.config = config

    @classmethod
    def build(cls, config, direction, device):
        h = ctypes.c_void_p()
        _check(library().b200fft_transform_build(ctypes.byref(config._s), int(direction),
                                                 ctypes.byref(device._c()), ctypes.byref(h)))
        return cls(h, config)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.b200fft_transform_destroy(h)
            self._h = None

    @property
    def pass_labels(self):
        """The kernel kind of each launch of one execution, in order."""
        n = library().b200fft_transform_describe_passes(self._h, None, 0)
        buf = ctypes.create_string_buffer(n + 1)
        library().b200fft_transform_describe_passes(self._h, buf, n + 1)
        return buf.value.decode().split("\n") if n else []

    @property
    def specialised_passes(self):
        """(generic passes with an ahead-of-time specialised kernel, generic passes)."""
        total = ctypes.c_int32()
        covered = library().b200fft_transform_specialised_passes(self._h, ctypes.byref(total))
        return int(covered), int(total.value)

    @property
    def family(self):
        return Family(library().b200fft_transform_family(self._h))

    def direction(self):
        return Direction(library().b200fft_transform_direction(self._h))

    def batch_count(self):
        return int(library().b200fft_transform_batch_count(self._h))

    @property
    def real_algorithm(self):
        return RealFftAlgorithm(library().b200fft_transform_real_algorithm(self._h))

    def real_transform_len(self):
        return int(library().b200fft_transform_real_transform_len(self._h))

    @property
    def plan(self):
        return _axes_of(library().b200fft_transform_plan(self._h))

    def axis_child(self, axis):
        info = _AxisInfo()
        _check(library().b200fft_transform_axis_child_info(self._h, axis, ctypes.byref(info)))
        return AxisPlan(info)

    @property
    def input_elements(self):
        return int(library().b200fft_transform_input_elements(self._h))

    @property
    def output_elements(self):
        return int(library().b200fft_transform_output_elements(self._h))

    @property
    def input_buffer_elements(self):
        """Device input buffer size (formatted strides: batch_stride x batch)."""
        return int(library().b200fft_transform_input_buffer_elements(self._h))

    @property
    def output_buffer_elements(self):
        return int(library().b200fft_transform_output_buffer_elements(self._h))

    @property
    def input_is_real(self):
        return bool(library().b200fft_transform_input_is_real(self._h))

    @property
    def output_is_real(self):
        return bool(library().b200fft_transform_output_is_real(self._h))

    @property
    def workspace_bytes(self):
        return int(library().b200fft_transform_workspace_bytes(self._h))

    @property
    def launch_count(self):
        return int(library().b200fft_transform_launch_count(self._h))

    def input_dtype(self):
        return _np_dtype[(self.config.precision, self.input_is_real)]

    def output_dtype(self):
        return _np_dtype[(self.config.precision, self.output_is_real)]

    @property
    def input_items(self):
        """Host array items of the input (elements x words per element)."""
        return self.input_elements * _words(self.config.precision, self.input_is_real)

    @property
    def output_items(self):
        return self.output_elements * _words(self.config.precision, self.output_is_real)


class ConvolutionConjugation(enum.IntEnum):
    NONE = 0
    SEQUENCE = 1
    KERNEL = 2


class _ConvolutionApplication:
    """Common part of the convolution applications: the library object, the element
    counts and types of the input / output arrays."""

    def __init__(self, handle, config):
        self._h = handle
        self.config = config
        self.precision = config.precision
        lib = library()
        self.input_elements = int(lib.b200fft_convolution_input_elements(handle))
        self.output_elements = int(lib.b200fft_convolution_output_elements(handle))
        self.input_is_real = bool(lib.b200fft_convolution_input_is_real(handle))
        self.input_buffer_elements = int(lib.b200fft_convolution_input_buffer_elements(handle))
        self.output_buffer_elements = int(lib.b200fft_convolution_output_buffer_elements(handle))

    @classmethod
    def _build(cls, config, kernel_spectrum, device, plane_elems):
        cdt = np.complex64 if config.precision == Precision.F32 else np.complex128
        spec = np.ascontiguousarray(kernel_spectrum, dtype=cdt).ravel()
        if spec.size % plane_elems:
            raise VkFftError(Status.InputLengthMismatch,
                             f"input contains {spec.size} complex elements but kernel expects a multiple of "
                             f"{plane_elems}")
        h = ctypes.c_void_p()
        _check(library().b200fft_convolution_build(ctypes.byref(config._s), ctypes.byref(device._c()),
                                                   spec.ctypes.data, spec.size // plane_elems, ctypes.byref(h)))
        return cls(h, config)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.b200fft_convolution_destroy(h)
            self._h = None

    @property
    def workspace_bytes(self):
        return int(library().b200fft_convolution_workspace_bytes(self._h))

    @property
    def specialised_passes(self):
        """(generic passes with an ahead-of-time specialised kernel, generic passes)."""
        total = ctypes.c_int32()
        covered = library().b200fft_convolution_specialised_passes(self._h, ctypes.byref(total))
        return int(covered), int(total.value)

    def real_dtype(self):
        return np.float32 if self.precision == Precision.F32 else np.float64

    def complex_dtype(self):
        return np.complex64 if self.precision == Precision.F32 else np.complex128

    def input_dtype(self):
        return self.real_dtype() if self.input_is_real else self.complex_dtype()

    def output_dtype(self):
        return self.input_dtype()


class NdRealConvolutionIr(_ConvolutionApplication):
    """convolution_ir.rs:3867-4183 (independent coordinates): build_from_spectrum(config,
    kernel_spectrum, device).  kernel_spectrum holds K*C copies of the compact R2C spectrum
    (the reference layout) or one copy broadcast to every coordinate."""

    @classmethod
    def build_from_spectrum(cls, config, kernel_spectrum, device):
        dims = config.dimensions
        return cls._build(config, kernel_spectrum, device, int(np.prod(dims[:-1])) * (dims[-1] // 2 + 1))


class ConvolutionIr(_ConvolutionApplication):
    """convolution_ir.rs:2520-3626: 1D C2C performConvolution from a pre-transformed kernel
    spectrum (scalar, K-kernel fan-out or 2x2 / 3x3 matrix coordinates)."""

    @classmethod
    def build_from_spectrum(cls, config, kernel_spectrum, device):
        return cls._build(config, kernel_spectrum, device, int(np.prod(config.dimensions)))


class NdConvolutionIr(ConvolutionIr):
    """convolution_ir.rs:3627-3866: multidimensional C2C performConvolution."""


# ---- backend/cuda/runtime.rs --------------------------------------------------------

def probe():
    """CudaExecutionContext::probe: number of devices, or VkFftError(NativeUnavailable)."""
    n = i32()
    _check(library().b200fft_probe(ctypes.byref(n)))
    return n.value


class SlabTransform:
    """Slab-decomposed transform over `nranks` processes, one GPU each (no counterpart in
    the single-device reference).  Rank g owns planes [g D0/P, (g+1) D0/P) of axis 0;
    the forward output is the pencil layout [D0, D1/P, ...] holding axis-1 indices
    [g D1/P, (g+1) D1/P) (compact last axis for R2C); the inverse maps it back.  The
    all-to-all exchange is fused into the last FFT pass before it (peer stores over
    NVLink through CUDA IPC) and closed by a device barrier with a bounded wait."""

    def __init__(self, handle, config, direction):
        self._h = handle
        self.config = config
        self.direction = direction
        self._ctx = None
        info = _SlabInfo()
        _check(library().b200fft_slab_get_info(handle, ctypes.byref(info)))
        self.nranks, self.rank = info.nranks, info.rank
        self.planes_per_rank, self.columns_per_rank = info.planes_per_rank, info.columns_per_rank
        self.input_elements, self.output_elements = info.input_elements, info.output_elements
        self.input_is_real, self.output_is_real = bool(info.input_is_real), bool(info.output_is_real)
        self.exchange_bytes = info.exchange_bytes
        self.launch_count = info.launch_count

    @classmethod
    def build(cls, config, direction, nranks, rank, device):
        h = ctypes.c_void_p()
        _check(library().b200fft_slab_build(ctypes.byref(config._s), int(direction), int(nranks), int(rank),
                                            ctypes.byref(device._c()), ctypes.byref(h)))
        return cls(h, config, direction)

    def destroy(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.b200fft_slab_destroy(h)
            self._h = None
        if self._ctx is not None:
            self._ctx._slabs.discard(self)
            self._ctx = None

    def __del__(self):
        self.destroy()

    def set_timeout(self, seconds):
        _check(library().b200fft_slab_set_timeout(self._h, int(seconds * 1e9)))

    def set_phase_timing(self, enabled=True):
        """Record CUDA events around the phases of every execution (after attach)."""
        _check(library().b200fft_slab_set_phase_timing(self._h, int(bool(enabled))))

    def phase_times(self):
        """[local passes, exchange pass, barrier, passes after the exchange] of the last
        execution, milliseconds (waits for it)."""
        ms = (ctypes.c_float * 4)()
        _check(library().b200fft_slab_phase_times(self._h, ms))
        return [float(v) for v in ms]

    def attach(self, ctx):
        """Allocates the exchange buffers on ctx's device; returns this rank's handle."""
        buf = ctypes.create_string_buffer(SLAB_HANDLE_BYTES)
        _check(library().b200fft_slab_attach(ctx._h, self._h, buf))
        self._ctx = ctx
        ctx._slabs.add(self)
        return bytes(buf.raw)

    def connect(self, ctx, handles):
        blob = b"".join(handles)
        if len(handles) != self.nranks or len(blob) != self.nranks * SLAB_HANDLE_BYTES:
            raise VkFftError(Status.ValueOutOfRange, "connect needs one handle per rank")
        _check(library().b200fft_slab_connect(ctx._h, self._h, blob))

    def setup(self, ctx, group=None):
        """attach + all_gather_object of the handles over torch.distributed + connect."""
        import torch.distributed as dist
        mine = self.attach(ctx)
        handles = [None] * self.nranks
        dist.all_gather_object(handles, mine, group=group)
        self.connect(ctx, handles)

    def element_dtypes(self):
        real = np.float32 if self.config.precision == Precision.F32 else np.float64
        cplx = np.complex64 if self.config.precision == Precision.F32 else np.complex128
        return (real if self.input_is_real else cplx), (real if self.output_is_real else cplx)


class AsyncTransformTicket:
    """NativeAsyncTransformTicket32/64 (native_runtime.rs:372-401): wait() returns the
    output array once the submitted execution has finished."""

    def __init__(self, handle, keep, out):
        self._h = handle
        self._keep = keep  # the arrays stay alive while the execution may use them
        self._out = out

    def wait(self):
        h, self._h = self._h, None
        if h is None:
            raise VkFftError(Status.ValueOutOfRange, "ticket was already waited for")
        _check(library().b200fft_ticket_wait(h))
        self._keep = None
        return self._out

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and _lib is not None:
            _lib.b200fft_ticket_destroy(h)
            self._h = None


class CudaExecutionContext:
    """backend/cuda/runtime.rs:959-2840"""

    def __init__(self, device_index=0):
        self._h = ctypes.c_void_p()
        self._slabs = set()
        _check(library().b200fft_context_create(int(device_index), ctypes.byref(self._h)))
        self.device_index = device_index

    def close(self):
        for slab in list(getattr(self, "_slabs", ())):
            slab.destroy()  # slabs hold device memory and peer mappings of this context
        if getattr(self, "_h", None) and _lib is not None:
            _lib.b200fft_context_destroy(self._h)
            self._h = None

    def execute_slab(self, slab, input_ptr, output_ptr, workspace_ptr=0, stream=0):
        """Stream-ordered slab execution on device pointers (b200fft_execute_slab)."""
        _check(library().b200fft_execute_slab(self._h, slab._h, ctypes.c_void_p(input_ptr),
                                              ctypes.c_void_p(output_ptr), ctypes.c_void_p(workspace_ptr or None),
                                              ctypes.c_void_p(stream or None)))

    def synchronize(self, stream=0):
        """Waits for the stream and raises NativeRuntime for errors the kernels recorded."""
        _check(library().b200fft_context_synchronize(self._h, ctypes.c_void_p(stream or None)))

    def __del__(self):
        self.close()

    def device_profile(self):
        d = _Device()
        _check(library().b200fft_context_device_profile(self._h, ctypes.byref(d)))
        return DeviceProfile(d)

    def device_name(self):
        buf = ctypes.create_string_buffer(256)
        _check(library().b200fft_context_device_name(self._h, buf, 256))
        return buf.value.decode()

    def execute_transform(self, ir, data, out=None):
        """execute_transform_f32/f64 (native_runtime.rs:339-359): host array in, new array out.
        `out` optionally supplies the (e.g. pinned) destination array."""
        x = np.ascontiguousarray(data, dtype=ir.input_dtype())
        if out is None:
            out = np.empty(ir.output_items, dtype=ir.output_dtype())
        elif out.dtype != ir.output_dtype() or out.size != ir.output_items or not out.flags.c_contiguous:
            raise VkFftError(Status.InputLengthMismatch,
                             f"input contains {out.size} complex elements but kernel expects {ir.output_elements}")
        _check(library().b200fft_execute_host(self._h, ir._h, x.ctypes.data, x.nbytes,
                                              out.ctypes.data, out.nbytes))
        return out

    def submit_transform(self, ir, data, out=None):
        """submit_transform_f32_async / _f64_async (native_runtime.rs:424-451): starts the
        host execution and returns an AsyncTransformTicket at once."""
        x = np.ascontiguousarray(data, dtype=ir.input_dtype())
        if out is None:
            out = np.empty(ir.output_items, dtype=ir.output_dtype())
        h = ctypes.c_void_p()
        _check(library().b200fft_submit_host(self._h, ir._h, x.ctypes.data, x.nbytes, out.ctypes.data, out.nbytes,
                                             ctypes.byref(h)))
        return AsyncTransformTicket(h, (x, ir), out)

    # typed aliases matching the reference's two entry points
    def execute_transform_f32(self, ir, data):
        return self.execute_transform(ir, data)

    def execute_transform_f64(self, ir, data):
        return self.execute_transform(ir, data)

    def execute_transform_double_double(self, ir, data):
        """execute_transform_double_double (native_runtime.rs:971-987): float64 words,
        (re.hi, re.lo, im.hi, im.lo) per complex element, (hi, lo) per real one."""
        return self.execute_transform(ir, data)

    def execute_transform_double_double_f64_storage(self, ir, data):
        """execute_transform_double_double_f64_storage (native_runtime.rs:988-1004): f64
        host arrays, double-double compute."""
        return self.execute_transform(ir, data)

    def execute_nd_real_convolution(self, ir, data, out=None):
        """execute_nd_real_convolution_f32/f64 / execute_convolution_f32/f64 /
        execute_nd_convolution_f32/f64 (native_runtime.rs:197-337): host arrays."""
        x = np.ascontiguousarray(data, dtype=ir.input_dtype()).ravel()
        if out is None:
            out = np.empty(ir.output_elements, dtype=ir.output_dtype())
        _check(library().b200fft_execute_convolution_host(self._h, ir._h, x.ctypes.data, x.nbytes,
                                                          out.ctypes.data, out.nbytes))
        return out

    execute_convolution = execute_nd_real_convolution
    execute_nd_convolution = execute_nd_real_convolution

    def execute_nd_real_convolution_resident(self, ir, input_ptr, output_ptr, workspace_ptr=0, stream=0):
        _check(library().b200fft_execute_convolution(self._h, ir._h, ctypes.c_void_p(input_ptr),
                                                     ctypes.c_void_p(output_ptr),
                                                     ctypes.c_void_p(workspace_ptr or None),
                                                     ctypes.c_void_p(stream or None)))

    def execute_resident(self, ir, input_ptr, output_ptr, workspace_ptr=0, stream=0):
        """Stream-ordered execution on device pointers (resident chain "into" path)."""
        _check(library().b200fft_execute(self._h, ir._h, ctypes.c_void_p(input_ptr),
                                         ctypes.c_void_p(output_ptr),
                                         ctypes.c_void_p(workspace_ptr or None),
                                         ctypes.c_void_p(stream or None)))

    def execute_static_workspace(self, ir, input_ptr, output_ptr, stream=0):
        """b200fft_execute_static_workspace: resident execution that allocates no device
        memory (tables and scratch in the library's fixed per-device region of
        STATIC_WORKSPACE_BYTES; calls that overlap on the GPU race)."""
        _check(library().b200fft_execute_static_workspace(self._h, ir._h, ctypes.c_void_p(input_ptr),
                                                          ctypes.c_void_p(output_ptr),
                                                          ctypes.c_void_p(stream or None)))


STATIC_WORKSPACE_BYTES = 16 << 20


def exported_symbols():
    """Names declared in include/b200fft.h (for the symbol-export test)."""
    import re
    hdr = os.path.join(os.path.dirname(_PKG), "include", "b200fft.h")
    with open(hdr) as fh:
        text = fh.read()
    return sorted(set(re.findall(r"\b(b200fft_[a-z0-9_]+)\s*\(", text)))
