"""Planner known-answer tests, restating the reference's own planner and application
tests (vkfft-rs src/planner.rs:742-1124, src/application.rs:699-985, src/lib.rs:34-37)
against the C++ planner through the C ABI.  Host only: no GPU."""
import pytest


def kinds(plan):
    return [a.kind.name for a in plan.axes]


def test_lib_rs_doc_example(V):
    # lib.rs:34-37: [1024, 17, 65537] -> Stockham, Rader, Bluestein
    plan = V.FftPlan.build(V.FftConfig([1024, 17, 65537]))
    assert kinds(plan) == ["STOCKHAM", "RADER", "BLUESTEIN"]


def test_factorization_helpers(V):
    # planner.rs:748-752, 1098-1123
    # prime_factorization(360) = [2, 2, 2, 3, 3, 5] (ascending, with multiplicity), seen
    # through the Stockham axis plan; 47 is its own single factor (a Rader prime)
    a = V.FftPlan.build(V.FftConfig([360])).axes[0]
    assert a.kind == V.AlgorithmKind.STOCKHAM and a.radix.prime_factors == [2, 2, 2, 3, 3, 5]
    p = V.FftPlan.build(V.FftConfig([47])).axes[0]
    assert p.kind == V.AlgorithmKind.RADER and [r.prime for r in p.primes] == [47]
    assert V.next_smooth_at_least(2061) >= 2061
    v = V.next_smooth_at_least(2061)
    for c in range(2061, v):
        m = c
        for p in (2, 3, 5, 7):
            while m % p == 0:
                m //= p
        assert m != 1
    for prime in (17, 47, 59, 83):
        g = V.primitive_root(prime)
        seen, val = set(), 1
        for _ in range(prime - 1):
            seen.add(val)
            val = val * g % prime
        assert len(seen) == prime - 1


def test_stockham_lengths_stay_stockham(V):
    assert kinds(V.FftPlan.build(V.FftConfig([2 * 3 * 5 * 7 * 11 * 13]))) == ["STOCKHAM"]


def test_smooth_rader_prime_uses_fft_convolution(V):
    a = V.FftPlan.build(V.FftConfig([17])).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and a.primes[0].prime == 17
    assert a.primes[0].mode == V.RaderMode.FFT_CONVOLUTION


def test_safe_prime_uses_direct_rader_when_enabled(V):
    a = V.FftPlan.build(V.FftConfig([47])).axes[0]
    assert a.kind == V.AlgorithmKind.RADER
    assert a.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION


def test_device_scored_double_double_uses_quad_stockham_prime_set(V):
    # planner.rs:776-819
    device = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA)
    assert kinds(V.FftPlan.build_for_device(V.FftConfig([13]), device)) == ["STOCKHAM"]
    dd = V.FftConfig([13]).with_precision(V.Precision.DOUBLE_DOUBLE)
    assert kinds(V.FftPlan.build(dd)) == ["STOCKHAM"]
    a = V.FftPlan.build_for_device(dd, device).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and a.radix.prime_factors == []
    assert len(a.primes) == 1 and a.primes[0].prime == 13
    assert a.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION
    explicit = dd.with_tuning(V.PlannerTuning.portable())
    assert kinds(V.FftPlan.build_for_device(explicit, device)) == ["BLUESTEIN"]


def test_device_scored_rader_limits_follow_thread_shared_and_strided_capacity(V):
    # planner.rs:822-965
    base = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA)
    portable = V.FftPlan.build(V.FftConfig([7681])).axes[0]
    assert portable.kind == V.AlgorithmKind.RADER
    assert portable.primes[0].mode == V.RaderMode.FFT_CONVOLUTION
    assert kinds(V.FftPlan.build_for_device(V.FftConfig([7681]), base)) == ["BLUESTEIN"]
    unknown = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.OTHER, 0x1234)
    u = V.FftPlan.build_for_device(V.FftConfig([7681]), unknown).axes[0]
    assert u.kind == V.AlgorithmKind.RADER and u.primes[0].mode == V.RaderMode.FFT_CONVOLUTION
    wide = base.replace(shared_memory_bytes=64 * 1024, shared_memory_pow2_bytes=64 * 1024)
    w = V.FftPlan.build_for_device(V.FftConfig([7681]), wide).axes[0]
    assert w.kind == V.AlgorithmKind.RADER and w.primes[0].mode == V.RaderMode.FFT_CONVOLUTION
    nd = V.FftPlan.build_for_device(V.FftConfig([4001, 4001]), base)
    assert kinds(nd) == ["BLUESTEIN", "RADER"]
    child = V.FftConfig([4001])
    assert kinds(V.FftPlan.build_c2c_child_for_device(child, base, strided=False)) == ["RADER"]
    strided = V.FftPlan.build_c2c_child_for_device(child, base, strided=True).axes[0]
    assert strided.kind == V.AlgorithmKind.BLUESTEIN and strided.convolution_len == 8192
    t = V.PlannerTuning.portable()
    t.max_rader_fft_prime = 100
    pb = V.FftPlan.build(child.with_tuning(t)).axes[0]
    assert pb.kind == V.AlgorithmKind.BLUESTEIN and pb.convolution_len == 8064
    explicit = V.PlannerTuning.portable()
    explicit.max_rader_direct_prime = 1000
    thread_limited = base.replace(max_threads_per_block=128, max_workgroup_size=[128, 128, 64])
    assert kinds(V.FftPlan.build_for_device(V.FftConfig([83]).with_tuning(explicit), thread_limited)) == ["BLUESTEIN"]
    f32 = V.FftPlan.build_for_device(V.FftConfig([47]), thread_limited).axes[0]
    assert f32.kind == V.AlgorithmKind.RADER and f32.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION
    f16 = V.FftConfig([47]).with_precision(V.Precision.F16_STORAGE_F32_COMPUTE)
    assert kinds(V.FftPlan.build_for_device(f16, thread_limited)) == ["BLUESTEIN"]


def test_unsafe_direct_rader_reservation_can_push_a_later_safe_prime_to_bluestein(V):
    # planner.rs:968-1011
    length = 83 * 1009
    base = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA)
    assert kinds(V.FftPlan.build_for_device(V.FftConfig([length]), base)) == ["BLUESTEIN"]
    wider = base.replace(shared_memory_bytes=33 * 1024)
    a = V.FftPlan.build_for_device(V.FftConfig([length]), wider).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and len(a.primes) == 2
    assert a.primes[0].prime == 83 and a.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION
    assert a.primes[1].prime == 1009 and a.primes[1].mode == V.RaderMode.FFT_CONVOLUTION


def test_nested_sub_rader_prime_is_opt_in(V):
    # planner.rs:1014-1038
    assert kinds(V.FftPlan.build(V.FftConfig([107]))) == ["BLUESTEIN"]
    rec = V.PlannerTuning.portable().with_recursive_fft_rader(True)
    a = V.FftPlan.build(V.FftConfig([107]).with_tuning(rec)).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and a.primes[0].mode == V.RaderMode.FFT_CONVOLUTION
    assert a.primes[0].convolution.prime_factors == [2, 53]
    n = V.FftPlan.build(V.FftConfig([106]).with_tuning(rec)).axes[0]
    assert n.kind == V.AlgorithmKind.RADER and n.primes[0].prime == 53
    assert n.primes[0].mode == V.RaderMode.FFT_CONVOLUTION


def test_recursive_rader_eligibility_uses_precision_specific_stockham_primes(V):
    # planner.rs:1041-1062
    device = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA)
    rec = V.PlannerTuning.portable().with_recursive_fft_rader(True)
    assert kinds(V.FftPlan.build_for_device(V.FftConfig([419]).with_tuning(rec), device)) == ["RADER"]
    dd = V.FftConfig([419]).with_precision(V.Precision.DOUBLE_DOUBLE).with_tuning(rec)
    assert kinds(V.FftPlan.build_for_device(dd, device)) == ["BLUESTEIN"]


def test_unsupported_prime_uses_bluestein(V):
    a = V.FftPlan.build(V.FftConfig([65537])).axes[0]
    assert a.kind == V.AlgorithmKind.BLUESTEIN
    assert a.convolution_len >= 2 * 65537 - 1
    prod = 1
    for f in a.radix.prime_factors:
        prod *= f
    assert prod == a.convolution_len


@pytest.mark.parametrize("precision", ["F32", "F16_STORAGE_F32_COMPUTE", "F64", "F64_COMPUTE_F32_STORAGE",
                                       "DOUBLE_DOUBLE", "DOUBLE_DOUBLE_F64_STORAGE"])
def test_grouped_bluestein_across_precisions(V, precision):
    t = V.PlannerTuning.portable()
    t.max_rader_fft_prime = 100
    cfg = (V.FftConfig([103]).with_batch_count(7).with_precision(V.Precision[precision]).with_tuning(t)
           .with_grouped_batch(0, 3))
    assert kinds(V.FftPlan.build(cfg)) == ["BLUESTEIN"]


def test_plan_is_per_axis(V):
    assert kinds(V.FftPlan.build(V.FftConfig([16, 17, 1031, 65537]))) == ["STOCKHAM", "RADER", "BLUESTEIN",
                                                                         "BLUESTEIN"]


# ---- application.rs ---------------------------------------------------------------

def nvidia_vk(V, **kw):
    return V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA).replace(**kw)


def test_high_level_real_shape_follows_fixed_upstream_big_even_threshold(V):
    # application.rs:699-871
    r2c = lambda n: V.FftConfig(n).with_transform(V.TransformKind.R2C)
    roomy = nvidia_vk(V, shared_memory_bytes=64 * 1024, shared_memory_pow2_bytes=64 * 1024)
    ir = V.TransformIr.build(r2c([30]), V.Direction.FORWARD, roomy)
    assert ir.real_algorithm == V.RealFftAlgorithm.FULL_COMPLEX and ir.real_transform_len() == 30
    constrained = nvidia_vk(V, shared_memory_bytes=128, shared_memory_pow2_bytes=128)
    ir = V.TransformIr.build(r2c([30]), V.Direction.FORWARD, constrained)
    assert ir.real_algorithm == V.RealFftAlgorithm.EVEN_HALF_SIZE and ir.real_transform_len() == 15
    reserved = nvidia_vk(V, shared_memory_bytes=94 * 8, shared_memory_pow2_bytes=94 * 8)
    ir = V.TransformIr.build(r2c([94]), V.Direction.FORWARD, reserved)
    assert ir.real_algorithm == V.RealFftAlgorithm.EVEN_HALF_SIZE and ir.real_transform_len() == 47
    ir = V.TransformIr.build(r2c([8704]), V.Direction.FORWARD, roomy)
    assert ir.real_algorithm == V.RealFftAlgorithm.EVEN_HALF_SIZE and ir.real_transform_len() == 4352
    small = nvidia_vk(V, shared_memory_bytes=300 * 8, shared_memory_pow2_bytes=300 * 8)
    ir = V.TransformIr.build(r2c([206]), V.Direction.FORWARD, small)
    assert ir.real_algorithm == V.RealFftAlgorithm.EVEN_HALF_SIZE and ir.real_transform_len() == 103
    fits = nvidia_vk(V, shared_memory_bytes=512 * 8, shared_memory_pow2_bytes=512 * 8)
    ir = V.TransformIr.build(r2c([206]), V.Direction.FORWARD, fits)
    assert ir.real_algorithm == V.RealFftAlgorithm.FULL_COMPLEX and ir.real_transform_len() == 206
    generic = nvidia_vk(V, shared_memory_bytes=6000 * 8, shared_memory_pow2_bytes=6000 * 8)
    ir = V.TransformIr.build(r2c([4106]), V.Direction.FORWARD, generic)
    assert ir.real_algorithm == V.RealFftAlgorithm.EVEN_HALF_SIZE and ir.real_transform_len() == 2053
    ir = V.TransformIr.build(r2c([3, 30]), V.Direction.FORWARD, roomy)
    assert ir.family == V.Family.REAL_ND and ir.real_algorithm == V.RealFftAlgorithm.FULL_COMPLEX
    ir = V.TransformIr.build(r2c([3, 30]), V.Direction.FORWARD, constrained)
    assert ir.real_algorithm == V.RealFftAlgorithm.EVEN_HALF_SIZE and ir.real_transform_len() == 15


def test_high_level_planner_uses_device_rader_defaults_unless_tuning_is_explicit(V):
    # application.rs:873-955 (the DD / AMD entries are planned, not executed, here)
    nvidia = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA)
    intel = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.INTEL)
    a = V.FftPlan.build_for_device(V.FftConfig([47]), nvidia).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and a.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION
    assert kinds(V.FftPlan.build_for_device(V.FftConfig([47]), intel)) == ["BLUESTEIN"]
    e = V.FftPlan.build_for_device(V.FftConfig([47]).with_tuning(V.PlannerTuning.portable()), intel).axes[0]
    assert e.kind == V.AlgorithmKind.RADER and e.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION
    amd = V.DeviceProfile.generic(V.Backend.HIP, V.GpuVendor.AMD)
    a = V.FftPlan.build_for_device(V.FftConfig([19]).with_precision(V.Precision.F64), amd).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and a.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION
    dd = V.FftConfig([47]).with_precision(V.Precision.DOUBLE_DOUBLE)
    assert kinds(V.FftPlan.build_for_device(dd, nvidia)) == ["BLUESTEIN"]
    c = nvidia.replace(max_threads_per_block=128, max_workgroup_size=[128, 128, 64])
    ir = V.TransformIr.build(V.FftConfig([83]), V.Direction.FORWARD, c)
    assert ir.axis_child(0).kind == V.AlgorithmKind.BLUESTEIN
    ir = V.TransformIr.build(V.FftConfig([83]).with_precision(V.Precision.F64), V.Direction.FORWARD, c)
    a = ir.axis_child(0)
    assert a.kind == V.AlgorithmKind.RADER and a.primes[0].mode == V.RaderMode.DIRECT_MULTIPLICATION


def test_high_level_bluestein_uses_fixed_device_padding(V):
    # application.rs:957-985
    t = V.PlannerTuning.portable()
    t.max_rader_fft_prime = 100
    prof = nvidia_vk(V, shared_memory_bytes=48 * 1024, shared_memory_pow2_bytes=32 * 1024,
                     max_threads_per_block=1024, max_workgroup_size=[1024, 1024, 64])
    ir = V.TransformIr.build(V.FftConfig([4001]).with_tuning(t), V.Direction.FORWARD, prof)
    a = ir.axis_child(0)
    assert a.kind == V.AlgorithmKind.BLUESTEIN and a.convolution_len == 8192


def test_real_direction_is_checked(V, cuda_profile):
    # application.rs:49-60
    with pytest.raises(V.VkFftError) as e:
        V.TransformIr.build(V.FftConfig([8]).with_transform(V.TransformKind.R2C), V.Direction.INVERSE,
                            cuda_profile)
    assert e.value.variant == "UnsupportedKernelPath"
    with pytest.raises(V.VkFftError):
        V.TransformIr.build(V.FftConfig([8]).with_transform(V.TransformKind.C2R), V.Direction.FORWARD,
                            cuda_profile)


# ---- BASELINE configs on the B200 profile (what the executed plans are) -----------

def test_baseline_config_plans_on_b200_profile(V, cuda_profile):
    p = V.FftPlan.build_for_device(V.FftConfig([1024]).with_batch_count(8), cuda_profile)
    assert kinds(p) == ["STOCKHAM"]
    p = V.FftPlan.build_for_device(V.FftConfig([4096]).with_batch_count(65536), cuda_profile)
    assert kinds(p) == ["STOCKHAM"]
    p = V.FftPlan.build_for_device(V.FftConfig([512, 512, 512]), cuda_profile)
    assert kinds(p) == ["STOCKHAM"] * 3
    p = V.FftPlan.build_for_device(V.FftConfig([1024, 17, 65537]), cuda_profile)
    assert kinds(p) == ["STOCKHAM", "RADER", "BLUESTEIN"]
    assert p.axes[2].convolution_len == 131220
    # 4099 under default tuning: 4098 = 2*3*683 fails the safe-prime gate -> Bluestein
    a = V.FftPlan.build_for_device(V.FftConfig([4099]).with_batch_count(16384), cuda_profile).axes[0]
    assert a.kind == V.AlgorithmKind.BLUESTEIN and a.convolution_len == 8232
    rec = V.PlannerTuning.portable().with_recursive_fft_rader(True)
    a = V.FftPlan.build_for_device(V.FftConfig([4099]).with_batch_count(16384).with_tuning(rec),
                                   cuda_profile).axes[0]
    assert a.kind == V.AlgorithmKind.RADER and a.primes[0].mode == V.RaderMode.FFT_CONVOLUTION
    assert a.primes[0].convolution.prime_factors == [2, 3, 683]
    a = V.FftPlan.build_for_device(V.FftConfig([65537]).with_batch_count(2048), cuda_profile).axes[0]
    assert a.kind == V.AlgorithmKind.BLUESTEIN and a.convolution_len == 131220
    ir = V.TransformIr.build(V.FftConfig([1024, 17, 65537]), V.Direction.FORWARD, cuda_profile)
    assert [ir.axis_child(k).kind.name for k in range(3)] == ["STOCKHAM", "RADER", "BLUESTEIN"]


def test_validation_errors_match_reference(V):
    # config.rs:1036-1460 (a few representative branches) and error.rs Display texts
    with pytest.raises(V.VkFftError) as e:
        V.FftConfig([16, 0]).validate()
    assert e.value.variant == "ZeroLength" and str(e.value) == "FFT axis 1 has zero length"
    with pytest.raises(V.VkFftError) as e:
        V.FftConfig([]).validate()
    assert e.value.variant == "EmptyDimensions"
    with pytest.raises(V.VkFftError) as e:
        V.FftConfig([8]).with_batch_count(0).validate()
    assert e.value.variant == "ZeroBatchCount"
    with pytest.raises(V.VkFftError) as e:
        V.FftConfig([8, 8]).with_omit_dimension(0, True).with_omit_dimension(1, True).validate()
    assert e.value.variant == "UnsupportedKernelPath"
    with pytest.raises(V.VkFftError) as e:
        V.FftConfig([8]).with_coordinate_features(2).validate()
    assert e.value.variant == "UnsupportedKernelPath"
    t = V.PlannerTuning.portable()
    t.min_rader_direct_prime = 40
    with pytest.raises(V.VkFftError) as e:
        V.FftConfig([8]).with_tuning(t).validate()
    assert e.value.variant == "InvalidPlannerTuning"
    with pytest.raises(V.VkFftError) as e:
        V.FftPlan.build(V.FftConfig([8]).with_convolution(True))
    assert e.value.variant == "UnsupportedKernelPath"


def test_bluestein_auto_padding_matches_fixed_upstream_boundaries(V):
    """Bluestein convolution lengths chosen for device plans (scheduler.rs:11436-11500):
    the fixed upstream benchmark table where it applies, otherwise the smooth-length
    search (our entry point combines both, as upstream_bluestein_auto_padding does)."""
    P = V.Precision
    nvidia = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.NVIDIA).replace(
        shared_memory_bytes=48 * 1024, shared_memory_pow2_bytes=32 * 1024, coalesced_memory_bytes=32)
    amd = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.AMD)
    unknown = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor.OTHER, 0x1234)
    pad = V.upstream_bluestein_auto_padding
    table_hits = [(41, P.F32, nvidia, 96), (41, P.F64, nvidia, 90), (206, P.F32, nvidia, 512),
                  (256, P.F32, nvidia, 512), (257, P.F32, nvidia, 567), (4096, P.F32, nvidia, 8192),
                  (19, P.F32, amd, 42), (19, P.F64, amd, 40), (3438, P.F64, amd, 6875),
                  (3439, P.F64, amd, 8192)]
    for n, prec, dev, m in table_hits:
        assert pad(n, 1, prec, dev) == m, (n, prec, m)
    # table misses fall through to the search, which never goes below 2N - 1; a vendor
    # without a fixed upstream scheduler profile has neither (scheduler.rs:291)
    for n, prec, dev in ((66, P.DOUBLE_DOUBLE, nvidia), (4097, P.F32, nvidia)):
        assert pad(n, 1, prec, dev) >= 2 * n - 1, (n, prec)
    with pytest.raises(V.VkFftError) as e:
        pad(206, 1, P.F32, unknown)
    assert e.value.variant == "UnsupportedKernelPath" and "known GPU scheduler profile" in str(e.value)
    for prec in (P.F32, P.DOUBLE_DOUBLE, P.DOUBLE_DOUBLE_F64_STORAGE):
        assert pad(4106, 1, prec, nvidia) == 8232, prec


@pytest.mark.parametrize("vendor,other,precision,expected", [
    ("NVIDIA", 0, "F32", (17, 89, 17, 16384)),
    ("AMD", 0, "F64", (17, 89, 29, 16384)),
    ("AMD", 0, "DOUBLE_DOUBLE", (11, 29, 19, 16384)),
    ("NVIDIA", 0, "DOUBLE_DOUBLE", (11, 29, 17, 16384)),
    ("INTEL", 0, "F32", (17, 17, 17, 16384)),
    ("APPLE", 0, "F64", (17, 17, 17, 16384)),
    ("OTHER", 0x1234, "F32", (17, 17, 17, 16384)),
])
def test_device_rader_thresholds_match_fixed_upstream_initialization(V, vendor, other, precision, expected):
    # config.rs device_rader_thresholds_match_fixed_upstream_initialization: the Rader
    # prime windows (min/max direct, min/max FFT convolution) a device profile resolves to
    device = V.DeviceProfile.generic(V.Backend.VULKAN, V.GpuVendor[vendor], other)
    t = V.PlannerTuning.for_device(device, V.Precision[precision])
    got = (t.min_rader_direct_prime, t.max_rader_direct_prime, t.min_rader_fft_prime, t.max_rader_fft_prime)
    assert got == expected
