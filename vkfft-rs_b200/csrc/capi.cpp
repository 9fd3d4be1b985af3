// extern "C" boundary of the B200 FFT engine (include/b200fft.h).  Every entry point
// catches the internal FftError and returns its status; the Display text is kept in a
// thread-local buffer for b200fft_last_error_string().
#include <cstring>
#include <memory>

#include "aot.hpp"
#include "runtime.hpp"
#include "slab.hpp"

using namespace b200fft;

struct b200fft_plan {
    FftPlan plan;
};
struct b200fft_transform {
    std::unique_ptr<Transform> t;
};
struct b200fft_context {
    Context *ctx;
};
struct b200fft_convolution {
    std::unique_ptr<Convolution> c;
};
struct b200fft_slab {
    std::unique_ptr<Slab> s;
};
struct b200fft_ticket {
    std::shared_ptr<Ticket> t;
};

static thread_local std::string g_last_error;

template <typename F>
static b200fft_status guarded(F &&f) {
    try {
        f();
        return B200FFT_OK;
    } catch (const FftError &e) {
        g_last_error = e.message;
        return e.code;
    } catch (const std::bad_alloc &) {
        g_last_error = "CUDA runtime error: host allocation failed";
        return B200FFT_NATIVE_RUNTIME;
    } catch (const std::exception &e) {
        g_last_error = std::string("CUDA runtime error: ") + e.what();
        return B200FFT_NATIVE_RUNTIME;
    }
}

static void need(const void *p, const char *what) {
    if (!p) throw FftError(B200FFT_VALUE_OUT_OF_RANGE, std::string(what) + " must not be null");
}

static DeviceProfile profile_from_c(const b200fft_device_profile &c) {
    DeviceProfile d;
    if (c.backend < 0 || c.backend > 6) fail_value_range("backend");
    if (c.vendor < 0 || c.vendor > 4) fail_value_range("vendor");
    d.backend = static_cast<Backend>(c.backend);
    d.vendor = static_cast<Vendor>(c.vendor);
    d.vendor_other_id = c.vendor_other_id;
    d.supports_f64 = c.supports_f64 != 0;
    d.shared_memory_bytes = c.shared_memory_bytes;
    d.shared_memory_pow2_bytes = c.shared_memory_pow2_bytes;
    d.max_threads_per_block = c.max_threads_per_block;
    for (int i = 0; i < 3; i++) d.max_workgroup_size[i] = c.max_workgroup_size[i];
    d.coalesced_memory_bytes = c.coalesced_memory_bytes;
    d.shared_banks = c.shared_banks;
    d.subgroup.size = c.subgroup.size;
    d.subgroup.min_size = c.subgroup.min_size;
    d.subgroup.max_size = c.subgroup.max_size;
    d.subgroup.required_size_compute_supported = c.subgroup.required_size_compute_supported;
    d.subgroup.compute_supported = c.subgroup.compute_supported;
    d.subgroup.basic_supported = c.subgroup.basic_supported;
    d.subgroup.shuffle_supported = c.subgroup.shuffle_supported;
    d.subgroup.shuffle_relative_supported = c.subgroup.shuffle_relative_supported;
    d.subgroup.compute_full_subgroups = c.subgroup.compute_full_subgroups;
    return d;
}

static void profile_to_c(const DeviceProfile &d, b200fft_device_profile &c) {
    std::memset(&c, 0, sizeof(c));
    c.backend = static_cast<int32_t>(d.backend);
    c.vendor = static_cast<int32_t>(d.vendor);
    c.vendor_other_id = d.vendor_other_id;
    c.supports_f64 = d.supports_f64;
    c.shared_memory_bytes = d.shared_memory_bytes;
    c.shared_memory_pow2_bytes = d.shared_memory_pow2_bytes;
    c.max_threads_per_block = d.max_threads_per_block;
    for (int i = 0; i < 3; i++) c.max_workgroup_size[i] = d.max_workgroup_size[i];
    c.coalesced_memory_bytes = d.coalesced_memory_bytes;
    c.shared_banks = d.shared_banks;
    c.subgroup.size = d.subgroup.size;
    c.subgroup.min_size = d.subgroup.min_size;
    c.subgroup.max_size = d.subgroup.max_size;
    c.subgroup.required_size_compute_supported = d.subgroup.required_size_compute_supported;
    c.subgroup.compute_supported = d.subgroup.compute_supported;
    c.subgroup.basic_supported = d.subgroup.basic_supported;
    c.subgroup.shuffle_supported = d.subgroup.shuffle_supported;
    c.subgroup.shuffle_relative_supported = d.subgroup.shuffle_relative_supported;
    c.subgroup.compute_full_subgroups = d.subgroup.compute_full_subgroups;
}

extern "C" {

const char *b200fft_last_error_string(void) { return g_last_error.c_str(); }
uint32_t b200fft_abi_version(void) { return B200FFT_ABI_VERSION; }

b200fft_status b200fft_config_init(b200fft_config *config, uint32_t rank, const uint64_t *dimensions) {
    return guarded([&] {
        need(config, "config");
        if (rank > B200FFT_MAX_DIMS) fail_value_range("FFT rank");
        if (rank) need(dimensions, "dimensions");
        std::vector<size_t> dims(dimensions, dimensions + rank);
        FftConfig::make(dims).to_c(*config);
    });
}

b200fft_status b200fft_config_validate(const b200fft_config *config) {
    return guarded([&] {
        need(config, "config");
        FftConfig::from_c(*config).validate();
    });
}

void b200fft_planner_tuning_portable(b200fft_planner_tuning *tuning) {
    if (!tuning) return;
    std::memset(tuning, 0, sizeof(*tuning));
    PlannerTuning t = PlannerTuning::portable();
    tuning->min_rader_direct_prime = t.min_rader_direct_prime;
    tuning->max_rader_direct_prime = t.max_rader_direct_prime;
    tuning->min_rader_fft_prime = t.min_rader_fft_prime;
    tuning->max_rader_fft_prime = t.max_rader_fft_prime;
    tuning->allow_recursive_fft_rader = t.allow_recursive_fft_rader;
}

void b200fft_planner_tuning_for_device(const b200fft_device_profile *device, int32_t precision,
                                       b200fft_planner_tuning *tuning) {
    if (!device || !tuning || precision < 0 || precision > 5) return;
    PlannerTuning t = tuning_for_device(profile_from_c(*device), static_cast<Precision>(precision));
    std::memset(tuning, 0, sizeof(*tuning));
    tuning->min_rader_direct_prime = t.min_rader_direct_prime;
    tuning->max_rader_direct_prime = t.max_rader_direct_prime;
    tuning->min_rader_fft_prime = t.min_rader_fft_prime;
    tuning->max_rader_fft_prime = t.max_rader_fft_prime;
    tuning->allow_recursive_fft_rader = t.allow_recursive_fft_rader;
}

void b200fft_device_profile_generic(int32_t backend, int32_t vendor, uint32_t vendor_other_id,
                                    b200fft_device_profile *profile) {
    if (!profile || backend < 0 || backend > 6 || vendor < 0 || vendor > 4) return;
    profile_to_c(DeviceProfile::generic(static_cast<Backend>(backend), static_cast<Vendor>(vendor), vendor_other_id),
                 *profile);
}

b200fft_status b200fft_plan_build(const b200fft_config *config, b200fft_plan **plan) {
    return guarded([&] {
        need(config, "config");
        need(plan, "plan");
        *plan = new b200fft_plan{FftPlan::build(FftConfig::from_c(*config))};
    });
}

b200fft_status b200fft_plan_build_for_device(const b200fft_config *config, const b200fft_device_profile *device,
                                             b200fft_plan **plan) {
    return guarded([&] {
        need(config, "config");
        need(device, "device");
        need(plan, "plan");
        *plan = new b200fft_plan{FftPlan::build_for_device(FftConfig::from_c(*config), profile_from_c(*device))};
    });
}

b200fft_status b200fft_plan_build_c2c_child_for_device(const b200fft_config *config,
                                                       const b200fft_device_profile *device, int32_t axis_class,
                                                       b200fft_plan **plan) {
    return guarded([&] {
        need(config, "config");
        need(device, "device");
        need(plan, "plan");
        if (axis_class != 0 && axis_class != 1) fail_value_range("axis class");
        *plan = new b200fft_plan{FftPlan::build_c2c_child_for_device(
            FftConfig::from_c(*config), profile_from_c(*device), static_cast<AxisClass>(axis_class))};
    });
}

uint32_t b200fft_plan_axis_count(const b200fft_plan *plan) { return plan ? (uint32_t)plan->plan.axes.size() : 0; }

b200fft_status b200fft_plan_axis_info(const b200fft_plan *plan, uint32_t axis, b200fft_axis_info *info) {
    return guarded([&] {
        need(plan, "plan");
        need(info, "info");
        if (axis >= plan->plan.axes.size()) fail_value_range("plan axis");
        fill_axis_info(plan->plan.axes[axis], *info);
    });
}

void b200fft_plan_destroy(b200fft_plan *plan) { delete plan; }

uint64_t b200fft_next_smooth_at_least(uint64_t target) {
    try {
        return next_smooth_at_least(target, {2, 3, 5, 7});
    } catch (...) {
        return 0;
    }
}

uint64_t b200fft_primitive_root(uint64_t prime) { return primitive_root(prime); }

b200fft_status b200fft_bluestein_auto_padding(uint64_t sequence_len, uint64_t batch_count, int32_t precision,
                                              const b200fft_device_profile *device, uint64_t *padded) {
    return guarded([&] {
        need(device, "device");
        need(padded, "padded");
        if (precision < 0 || precision > 5) fail_value_range("precision");
        *padded = upstream_bluestein_auto_padding(sequence_len, batch_count, static_cast<Precision>(precision),
                                                  profile_from_c(*device));
    });
}

b200fft_status b200fft_transform_build(const b200fft_config *config, int32_t direction,
                                       const b200fft_device_profile *device, b200fft_transform **transform) {
    return guarded([&] {
        need(config, "config");
        need(device, "device");
        need(transform, "transform");
        if (direction != B200FFT_FORWARD && direction != B200FFT_INVERSE) fail_value_range("direction");
        *transform = new b200fft_transform{build_transform(FftConfig::from_c(*config), direction, profile_from_c(*device))};
    });
}

// Drops the uploaded tables of a transform and of its sub-batch and dense twins.
static void forget_transform(const Transform &t) {
    forget_program(t.id);
    for (auto &kv : t.chunks)
        if (kv.second) forget_transform(*kv.second);
    if (t.dense_twin) forget_transform(*t.dense_twin);
}

void b200fft_transform_destroy(b200fft_transform *transform) {
    if (!transform) return;
    forget_transform(*transform->t);
    delete transform;
}

int32_t b200fft_transform_family(const b200fft_transform *t) { return t ? t->t->family : -1; }
int32_t b200fft_transform_direction(const b200fft_transform *t) { return t ? t->t->direction : -1; }
uint64_t b200fft_transform_batch_count(const b200fft_transform *t) { return t ? t->t->plan.config.batch_count : 0; }
int32_t b200fft_transform_real_algorithm(const b200fft_transform *t) {
    return t ? static_cast<int32_t>(t->t->real_algorithm) : -1;
}
uint64_t b200fft_transform_real_transform_len(const b200fft_transform *t) { return t ? t->t->real_transform_len : 0; }

const b200fft_plan *b200fft_transform_plan(const b200fft_transform *t) {
    // the plan is exposed through a view object owned by the transform
    static thread_local b200fft_plan view;
    if (!t) return nullptr;
    view.plan = t->t->plan;
    return &view;
}

b200fft_status b200fft_transform_axis_child_info(const b200fft_transform *t, uint32_t axis, b200fft_axis_info *info) {
    return guarded([&] {
        need(t, "transform");
        need(info, "info");
        if (axis >= t->t->children.size()) fail_value_range("transform axis");
        if (!t->t->children[axis]) fail_unsupported("axis is omitted and has no executed child plan");
        fill_axis_info(t->t->children[axis]->axes[0], *info);
    });
}

uint64_t b200fft_transform_input_elements(const b200fft_transform *t) { return t ? t->t->logical_in_elems : 0; }
uint64_t b200fft_transform_output_elements(const b200fft_transform *t) { return t ? t->t->logical_out_elems : 0; }
uint64_t b200fft_transform_input_buffer_elements(const b200fft_transform *t) { return t ? t->t->prog.input_elems : 0; }
uint64_t b200fft_transform_output_buffer_elements(const b200fft_transform *t) {
    return t ? t->t->prog.output_elems : 0;
}
int32_t b200fft_transform_input_is_real(const b200fft_transform *t) { return t ? t->t->prog.input_real : 0; }
int32_t b200fft_transform_output_is_real(const b200fft_transform *t) { return t ? t->t->prog.output_real : 0; }
uint64_t b200fft_transform_workspace_bytes(const b200fft_transform *t) { return t ? t->t->prog.scratch_bytes() : 0; }
uint32_t b200fft_transform_launch_count(const b200fft_transform *t) {
    return t ? (uint32_t)t->t->prog.passes.size() : 0;
}

b200fft_status b200fft_probe(int32_t *device_count) {
    return guarded([&] {
        int n = probe_devices();
        if (device_count) *device_count = n;
    });
}

b200fft_status b200fft_context_create(int32_t device_ordinal, b200fft_context **context) {
    return guarded([&] {
        need(context, "context");
        *context = new b200fft_context{context_create(device_ordinal)};
    });
}

void b200fft_context_destroy(b200fft_context *context) {
    if (!context) return;
    context_destroy(context->ctx);
    delete context;
}

b200fft_status b200fft_context_device_profile(const b200fft_context *context, b200fft_device_profile *profile) {
    return guarded([&] {
        need(context, "context");
        need(profile, "profile");
        profile_to_c(context->ctx->profile, *profile);
    });
}

b200fft_status b200fft_context_device_name(const b200fft_context *context, char *name, size_t capacity) {
    return guarded([&] {
        need(context, "context");
        need(name, "name");
        if (capacity == 0) fail_value_range("name capacity");
        std::strncpy(name, context->ctx->name.c_str(), capacity - 1);
        name[capacity - 1] = 0;
    });
}

b200fft_status b200fft_execute(b200fft_context *context, b200fft_transform *transform, const void *input, void *output,
                               void *workspace, void *stream) {
    return guarded([&] {
        need(context, "context");
        need(transform, "transform");
        need(input, "input");
        need(output, "output");
        execute_program(context->ctx, transform->t->id, transform->t->prog, input, output, workspace,
                        static_cast<cudaStream_t>(stream));
    });
}

b200fft_status b200fft_execute_static_workspace(b200fft_context *context, b200fft_transform *transform,
                                                const void *input, void *output, void *stream) {
    return guarded([&] {
        need(context, "context");
        need(transform, "transform");
        need(input, "input");
        need(output, "output");
        execute_program_static(context->ctx, transform->t->id, transform->t->prog, input, output,
                               static_cast<cudaStream_t>(stream));
    });
}

b200fft_status b200fft_execute_host(b200fft_context *context, b200fft_transform *transform, const void *input,
                                    size_t input_bytes, void *output, size_t output_bytes) {
    return guarded([&] {
        need(context, "context");
        need(transform, "transform");
        need(input, "input");
        need(output, "output");
        execute_transform_host(context->ctx, *transform->t, input, input_bytes, output, output_bytes);
    });
}

b200fft_status b200fft_convolution_build(const b200fft_config *config, const b200fft_device_profile *device,
                                         const void *kernel_spectrum, uint64_t spectrum_copies,
                                         b200fft_convolution **convolution) {
    return guarded([&] {
        need(config, "config");
        need(device, "device");
        need(kernel_spectrum, "kernel spectrum");
        need(convolution, "convolution");
        *convolution = new b200fft_convolution{
            build_convolution(FftConfig::from_c(*config), profile_from_c(*device), kernel_spectrum, spectrum_copies)};
    });
}

void b200fft_convolution_destroy(b200fft_convolution *convolution) {
    if (!convolution) return;
    forget_program(convolution->c->id);
    if (convolution->c->dense_twin) forget_program(convolution->c->dense_twin->id);
    delete convolution;
}

uint64_t b200fft_convolution_workspace_bytes(const b200fft_convolution *c) { return c ? c->c->prog.scratch_bytes() : 0; }

int32_t b200fft_convolution_specialised_passes(const b200fft_convolution *c, int32_t *generic_passes) {
    if (!c) return -1;
    int total = 0;
    const int covered = aot_coverage(c->c->prog, &total);
    if (generic_passes) *generic_passes = total;
    return covered;
}

b200fft_status b200fft_execute_convolution(b200fft_context *context, b200fft_convolution *convolution,
                                           const void *input, void *output, void *workspace, void *stream) {
    return guarded([&] {
        need(context, "context");
        need(convolution, "convolution");
        need(input, "input");
        need(output, "output");
        execute_program(context->ctx, convolution->c->id, convolution->c->prog, input, output, workspace,
                        static_cast<cudaStream_t>(stream));
    });
}

b200fft_status b200fft_execute_convolution_host(b200fft_context *context, b200fft_convolution *convolution,
                                                const void *input, size_t input_bytes, void *output,
                                                size_t output_bytes) {
    return guarded([&] {
        need(context, "context");
        need(convolution, "convolution");
        need(input, "input");
        need(output, "output");
        // host arrays are logical tensors: a formatted convolution runs its dense twin
        const Convolution &cv = convolution->c->dense_twin ? *convolution->c->dense_twin : *convolution->c;
        std::lock_guard<std::mutex> host_lock(context->ctx->host_mu);  // staging buffers: one host call at a time
        execute_program_host(context->ctx, cv.id, cv.prog, input, input_bytes, output, output_bytes);
    });
}

}  // extern "C"

b200fft_status b200fft_slab_build(const b200fft_config *config, int32_t direction, uint32_t nranks, uint32_t rank,
                                  const b200fft_device_profile *device, b200fft_slab **slab) {
    return guarded([&] {
        need(config, "config");
        need(device, "device");
        need(slab, "slab");
        if (direction != B200FFT_FORWARD && direction != B200FFT_INVERSE) fail_value_range("direction");
        auto s = build_slab(FftConfig::from_c(*config), direction, (int)nranks, (int)rank, profile_from_c(*device));
        *slab = new b200fft_slab{std::move(s)};
    });
}

void b200fft_slab_destroy(b200fft_slab *slab) { delete slab; }

b200fft_status b200fft_slab_get_info(const b200fft_slab *slab, b200fft_slab_info *info) {
    return guarded([&] {
        need(slab, "slab");
        need(info, "info");
        const Slab &s = *slab->s;
        std::memset(info, 0, sizeof(*info));
        info->nranks = (uint32_t)s.nranks;
        info->rank = (uint32_t)s.rank;
        info->planes_per_rank = s.planes_per_rank;
        info->columns_per_rank = s.columns_per_rank;
        info->input_elements = s.input_elems;
        info->output_elements = s.output_elems;
        info->input_is_real = s.input_real;
        info->output_is_real = s.output_real;
        info->exchange_bytes = 256 + 2 * s.buffer_bytes();
        info->launch_count = (uint32_t)(s.pre.passes.size() + s.post.passes.size() + 1);
    });
}

b200fft_status b200fft_slab_set_timeout(b200fft_slab *slab, uint64_t timeout_ns) {
    return guarded([&] {
        need(slab, "slab");
        if (timeout_ns == 0) fail_value_range("timeout_ns");
        slab->s->timeout_ns = timeout_ns;
    });
}

b200fft_status b200fft_slab_set_phase_timing(b200fft_slab *slab, int32_t enabled) {
    return guarded([&] {
        need(slab, "slab");
        slab_set_phase_timing(slab->s.get(), enabled != 0);
    });
}

b200fft_status b200fft_slab_phase_times(b200fft_slab *slab, float *ms) {
    return guarded([&] {
        need(slab, "slab");
        need(ms, "ms");
        slab_phase_times(slab->s.get(), ms);
    });
}

b200fft_status b200fft_slab_attach(b200fft_context *context, b200fft_slab *slab, void *handle) {
    return guarded([&] {
        need(context, "context");
        need(slab, "slab");
        need(handle, "handle");
        slab_attach(context->ctx, slab->s.get(), static_cast<unsigned char *>(handle));
    });
}

b200fft_status b200fft_slab_connect(b200fft_context *context, b200fft_slab *slab, const void *handles) {
    return guarded([&] {
        need(context, "context");
        need(slab, "slab");
        need(handles, "handles");
        slab_connect(context->ctx, slab->s.get(), static_cast<const unsigned char *>(handles));
    });
}

b200fft_status b200fft_execute_slab(b200fft_context *context, b200fft_slab *slab, const void *input, void *output,
                                    void *workspace, void *stream) {
    return guarded([&] {
        need(context, "context");
        need(slab, "slab");
        need(input, "input");
        need(output, "output");
        execute_slab(context->ctx, slab->s.get(), input, output, workspace, static_cast<cudaStream_t>(stream));
    });
}

b200fft_status b200fft_context_synchronize(b200fft_context *context, void *stream) {
    return guarded([&] {
        need(context, "context");
        context_synchronize(context->ctx, static_cast<cudaStream_t>(stream));
    });
}

uint64_t b200fft_transform_describe_passes(const b200fft_transform *transform, char *buffer, uint64_t capacity) {
    if (!transform) return 0;
    std::string text;
    for (const PassPlan &pp : transform->t->prog.passes) {
        if (!text.empty()) text += '\n';
        text += pp.label;
    }
    if (buffer && capacity) {
        const size_t n = std::min<size_t>(text.size(), (size_t)capacity - 1);
        std::memcpy(buffer, text.data(), n);
        buffer[n] = '\0';
    }
    return text.size();
}

int32_t b200fft_transform_specialised_passes(const b200fft_transform *transform, int32_t *generic_passes) {
    if (!transform) return -1;
    int total = 0;
    const int covered = aot_coverage(transform->t->prog, &total);
    if (generic_passes) *generic_passes = total;
    return covered;
}

b200fft_status b200fft_submit_host(b200fft_context *context, b200fft_transform *transform, const void *input,
                                   size_t input_bytes, void *output, size_t output_bytes, b200fft_ticket **ticket) {
    return guarded([&] {
        need(context, "context");
        need(transform, "transform");
        need(input, "input");
        need(output, "output");
        need(ticket, "ticket");
        *ticket = new b200fft_ticket{
            submit_transform_host(context->ctx, *transform->t, input, input_bytes, output, output_bytes)};
    });
}

b200fft_status b200fft_ticket_wait(b200fft_ticket *ticket) {
    if (!ticket) {
        g_last_error = "ticket must not be null";
        return B200FFT_VALUE_OUT_OF_RANGE;
    }
    wait_ticket(*ticket->t);
    const b200fft_status st = static_cast<b200fft_status>(ticket->t->status);
    if (st != B200FFT_OK) g_last_error = ticket->t->message;
    delete ticket;
    return st;
}

void b200fft_ticket_destroy(b200fft_ticket *ticket) {
    if (!ticket) return;
    wait_ticket(*ticket->t);
    delete ticket;
}

uint64_t b200fft_convolution_input_elements(const b200fft_convolution *c) { return c ? c->c->logical_in_elems : 0; }
uint64_t b200fft_convolution_output_elements(const b200fft_convolution *c) { return c ? c->c->logical_out_elems : 0; }
uint64_t b200fft_convolution_input_buffer_elements(const b200fft_convolution *c) { return c ? c->c->prog.input_elems : 0; }
uint64_t b200fft_convolution_output_buffer_elements(const b200fft_convolution *c) {
    return c ? c->c->prog.output_elems : 0;
}
int32_t b200fft_convolution_input_is_real(const b200fft_convolution *c) { return c ? c->c->prog.input_real : 0; }
