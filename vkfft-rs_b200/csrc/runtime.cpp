// CUDA runtime side of the B200 FFT engine.
#include "runtime.hpp"

#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <set>

namespace b200fft {

int kernel_variant_for(int scalar_kind);
cudaError_t launch_pass(int variant, const PassParams &p, int64_t grid, int threads, size_t smem, cudaStream_t stream);
void set_kernel_smem_limits();
void set_reg_kernel_smem_limits();
cudaError_t launch_reg(int variant, const RegParams &rp, cudaStream_t stream);
cudaError_t launch_boundary_copy(const BoundaryCopy &b, cudaStream_t stream);
cudaError_t launch_conv_multiply(const ConvMultiply &m, int kind, cudaStream_t stream);
cudaError_t launch_r2r(const R2rPass &r, int kind, cudaStream_t stream);

// ---- host-side fault injection (no GPU fault is ever provoked) ------------------
// B200FFT_FAULT=alloc:<n> or launch:<n> makes the n-th device allocation or kernel
// launch of the process fail on the host with a NativeRuntime error.
static std::atomic<long> g_alloc_count{0}, g_launch_count{0};
static bool injected(const char *what, std::atomic<long> &counter) {
    const char *env = std::getenv("B200FFT_FAULT");
    long n = ++counter;
    if (!env) return false;
    size_t wl = std::strlen(what);
    if (std::strncmp(env, what, wl) != 0 || env[wl] != ':') return false;
    return std::atol(env + wl + 1) == n;
}

static void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) fail_runtime(std::string(what) + " failed: " + cudaGetErrorString(e));
}

static void *device_alloc(size_t bytes, const char *what) {
    if (injected("alloc", g_alloc_count)) fail_runtime(std::string(what) + " failed: injected allocation fault");
    void *p = nullptr;
    check(cudaMalloc(&p, std::max<size_t>(bytes, 256)), what);
    return p;
}

static std::mutex g_ctx_mu;
static std::set<Context *> g_contexts;

int probe_devices() {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail_unavailable(cudaGetErrorString(e));
    }
    if (n <= 0) fail_unavailable("no CUDA device is present");
    return n;
}

Context *context_create(int device) {
    int n = probe_devices();
    if (device < 0 || device >= n) fail_unavailable("CUDA device ordinal " + std::to_string(device) + " is out of range");
    check(cudaSetDevice(device), "cudaSetDevice");
    auto *ctx = new Context();
    ctx->device = device;
    try {
        check(cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking), "cudaStreamCreate");
        ctx->d_err = static_cast<int *>(device_alloc(sizeof(int), "error word allocation"));
        check(cudaMemset(ctx->d_err, 0, sizeof(int)), "cudaMemset");
        // the memset runs on the legacy stream, which the context's non-blocking streams
        // do not wait for
        check(cudaStreamSynchronize(cudaStreamLegacy), "stream synchronize");
        cudaDeviceProp prop;
        check(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
        ctx->name = prop.name;
        ctx->sm_count = prop.multiProcessorCount;
        // The profile the reference derives from the same attributes
        // (backend/cuda/runtime.rs:1204-1225).
        DeviceProfile d = cuda_device_profile(prop.sharedMemPerBlock, prop.maxThreadsPerBlock, prop.maxThreadsDim[0],
                                              prop.maxThreadsDim[1], prop.maxThreadsDim[2],
                                              prop.major > 1 || (prop.major == 1 && prop.minor >= 3));
        ctx->profile = d;
        set_kernel_smem_limits();
        set_reg_kernel_smem_limits();
    } catch (...) {
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        if (ctx->d_err) cudaFree(ctx->d_err);
        delete ctx;
        throw;
    }
    std::lock_guard<std::mutex> g(g_ctx_mu);
    g_contexts.insert(ctx);
    return ctx;
}

void context_destroy(Context *ctx) {
    if (!ctx) return;
    {
        std::lock_guard<std::mutex> g(g_ctx_mu);
        g_contexts.erase(ctx);
    }
    if (ctx->worker.joinable()) {  // finish every submitted job first
        {
            std::lock_guard<std::mutex> l(ctx->job_mu);
            ctx->stopping = true;
        }
        ctx->job_cv.notify_all();
        ctx->worker.join();
    }
    ctx->staging.reset();  // joins its copy threads, frees the pinned rings
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (auto &kv : ctx->tables) cudaFree(kv.second.base);
    cudaFree(ctx->scratch);
    cudaFree(ctx->stage_in);
    cudaFree(ctx->stage_out);
    for (cudaStream_t s : ctx->pipe)
        if (s) {
            cudaStreamSynchronize(s);
            cudaStreamDestroy(s);
        }
    cudaFree(ctx->pipe_buf);
    cudaFree(ctx->d_err);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
}

void forget_program(uint64_t id) {
    std::lock_guard<std::mutex> g(g_ctx_mu);
    for (Context *ctx : g_contexts) {
        std::lock_guard<std::mutex> l(ctx->mu);
        auto it = ctx->tables.find(id);
        if (it != ctx->tables.end()) {
            cudaSetDevice(ctx->device);
            cudaStreamSynchronize(ctx->stream);
            cudaFree(it->second.base);
            ctx->tables.erase(it);
        }
    }
}

// Upload (once per context) every table of the program, rounded to the pass precision.
static DeviceTables &ensure_tables(Context *ctx, uint64_t id, const Program &prog) {
    auto it = ctx->tables.find(id);
    if (it != ctx->tables.end()) return it->second;
    std::vector<size_t> offs;
    size_t total = 0;
    for (auto &t : prog.tables) {
        offs.push_back(total);
        total += (t.bytes(prog.cbytes()) + 255) & ~size_t(255);
    }
    DeviceTables dt;
    std::vector<unsigned char> host(std::max<size_t>(total, 256));
    for (size_t k = 0; k < prog.tables.size(); k++) {
        pack_table(prog.tables[k], prog, host.data() + offs[k]);
    }
    dt.base = device_alloc(host.size(), "table upload allocation");
    // A copy from pageable memory may return before its DMA has reached device memory, and
    // the kernels that read the tables run on non-blocking streams: wait for the legacy
    // stream that carries the copy.
    cudaError_t e = cudaMemcpy(dt.base, host.data(), host.size(), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) {
        cudaFree(dt.base);
        check(e, "table upload");
    }
    for (size_t k = 0; k < prog.tables.size(); k++)
        dt.ptrs.push_back(static_cast<unsigned char *>(dt.base) + offs[k]);
    try {
        dt.spec = aot_kernels_for(prog, ctx->device);
    } catch (...) {
        cudaFree(dt.base);
        throw;
    }
    return ctx->tables.emplace(id, std::move(dt)).first->second;
}

static void *ensure_buffer(void *&buf, size_t &have, size_t need, const char *what) {
    if (need > have) {
        cudaFree(buf);
        buf = nullptr;
        have = 0;
        buf = device_alloc(need, what);
        have = need;
    }
    return buf;
}

void execute_program(Context *ctx, uint64_t id, const Program &prog, const void *in, void *out, void *workspace,
                     cudaStream_t stream, const PeerStore *peer, cudaEvent_t before_last) {
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    std::lock_guard<std::mutex> l(ctx->mu);
    if (!stream) stream = ctx->stream;
    DeviceTables &dt = ensure_tables(ctx, id, prog);
    const size_t esz = (size_t)prog.cbytes();
    unsigned char *scr = static_cast<unsigned char *>(workspace);
    if (!scr && prog.scratch_bytes() > 0)
        scr = static_cast<unsigned char *>(
            ensure_buffer(ctx->scratch, ctx->scratch_bytes, prog.scratch_bytes(), "scratch allocation"));
    void *bufs[2 + kScratchBuffers] = {const_cast<void *>(in), out};
    for (int k = 0; k < kScratchBuffers; k++) bufs[2 + k] = scr ? scr + prog.scratch_offset(k) : nullptr;
    const int variant = kernel_variant_for(prog.scalar_kind());
    for (size_t pi = 0; pi < prog.passes.size(); pi++) {
        const PassPlan &pp = prog.passes[pi];
        if (before_last && pi + 1 == prog.passes.size()) check(cudaEventRecord(before_last, stream), "cudaEventRecord");
        if (pp.kernel == KERNEL_R2R) {
            R2rPass rr = pp.rr;
            rr.src = bufs[pp.src_buf];
            rr.dst = bufs[pp.dst_buf];
            rr.tb = pp.reg_table2 >= 0 ? dt.ptrs[pp.reg_table2] : nullptr;
            check(launch_r2r(rr, prog.scalar_kind(), stream), "kernel launch");
            continue;
        }
        if (pp.kernel == KERNEL_CMUL) {
            ConvMultiply cm = pp.cm;
            cm.src = bufs[pp.src_buf];
            cm.dst = bufs[pp.dst_buf];
            cm.ker = dt.ptrs[pp.reg_table];
            check(launch_conv_multiply(cm, prog.scalar_kind(), stream), "kernel launch");
            continue;
        }
        if (pp.kernel == KERNEL_COPY) {
            BoundaryCopy bc = pp.bc;
            bc.src = bufs[pp.src_buf];
            bc.dst = bufs[pp.dst_buf];
            check(launch_boundary_copy(bc, stream), "kernel launch");
            continue;
        }
        if (pp.kernel == KERNEL_REG) {
            RegParams rp = pp.rp;
            rp.in = static_cast<const unsigned char *>(bufs[pp.src_buf]) + pp.src_off * (pp.reg_in_real ? esz / 2 : esz);
            rp.out = static_cast<unsigned char *>(bufs[pp.dst_buf]) + pp.dst_off * (pp.reg_out_real ? esz / 2 : esz);
            rp.tw = dt.ptrs[pp.reg_table];
            rp.tw2 = pp.reg_table2 >= 0 ? dt.ptrs[pp.reg_table2] : nullptr;
            rp.tw3 = pp.reg_table3 >= 0 ? dt.ptrs[pp.reg_table3] : nullptr;
            rp.err = ctx->d_err;
            int rv = pp.reg_variant;
            if (pp.reg_variant_plain >= 0 && (reinterpret_cast<uintptr_t>(rp.in) & 15)) rv = pp.reg_variant_plain;
            if (pp.peer_scatter) {
                if (!peer) fail_runtime("slab exchange pass launched without the ranks' buffers");
                rp.peer = *peer;
                rp.peer.sub = peer->chunk * pp.peer_es;
            }
            if (injected("launch", g_launch_count)) fail_runtime("kernel launch failed: injected launch fault");
            check(launch_reg(rv, rp, stream), "kernel launch");
            continue;
        }
        PassParams p = pp.p;
        for (int k = 0; k < p.nops; k++) {
            const void **slots[3] = {&p.ops[k].lut, &p.ops[k].lut2, &p.ops[k].lut3};
            for (int s = 0; s < 3; s++) *slots[s] = pp.op_tables[k][s] >= 0 ? dt.ptrs[pp.op_tables[k][s]] : nullptr;
        }
        const size_t in_sz = p.in.real ? esz / 2 : esz, out_sz = p.out.real ? esz / 2 : esz;
        p.src = static_cast<const unsigned char *>(bufs[pp.src_buf]) + pp.src_off * in_sz;
        p.dst = static_cast<unsigned char *>(bufs[pp.dst_buf]) + pp.dst_off * out_sz;
        p.err = ctx->d_err;
        if (pp.peer_scatter) {
            if (!peer) fail_runtime("slab exchange pass launched without the ranks' buffers");
            p.peer = *peer;
            p.peer.sub = peer->chunk * pp.peer_es;
        }
        if (injected("launch", g_launch_count)) fail_runtime("kernel launch failed: injected launch fault");
        if (pi < dt.spec.size() && dt.spec[pi]) {
            void *args[] = {&p};
            check(cudaLaunchKernel(dt.spec[pi], dim3((unsigned)pp.grid), dim3(pp.threads), args, pp.smem, stream),
                  "kernel launch");
        } else {
            check(launch_pass(variant, p, pp.grid, pp.threads, pp.smem, stream), "kernel launch");
        }
    }
}

static HostStaging &staging_of(Context *ctx) {  // the caller holds ctx->host_mu
    if (!ctx->staging) ctx->staging = std::make_unique<HostStaging>(ctx->device);
    return *ctx->staging;
}

// Host -> device copy of one host call's input: pinned arrays go straight to the copy
// engine, large pageable ones through the context's pinned staging, small pageable ones
// through the driver's own pageable path.
static void host_upload(Context *ctx, void *dst, const void *src, size_t bytes, bool pageable, cudaStream_t s) {
    if (pageable && bytes >= StagingTuning().min_staged_upload)
        staging_of(ctx).upload(dst, src, bytes, s);
    else
        check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s), "input upload");
}

// Device -> host copy of a host call's output; a staged copy returns when the bytes are
// in `dst`, a direct one is queued on `s`.
static void host_download(Context *ctx, void *dst, const void *src, size_t bytes, bool pageable, cudaStream_t s) {
    if (pageable && bytes >= StagingTuning().min_staged_download)
        staging_of(ctx).download(dst, src, bytes, s);
    else
        check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s), "output download");
}

void execute_program_host(Context *ctx, uint64_t id, const Program &prog, const void *in, size_t in_bytes, void *out,
                          size_t out_bytes) {
    const size_t in_need = prog.input_bytes(), out_need = prog.output_bytes();
    const size_t in_el = in_need / std::max<size_t>(prog.input_elems, 1), out_el = out_need / std::max<size_t>(prog.output_elems, 1);
    if (in_bytes != in_need) fail_input_length(prog.input_elems, in_bytes / std::max<size_t>(in_el, 1));
    if (out_bytes != out_need) fail_input_length(prog.output_elems, out_bytes / std::max<size_t>(out_el, 1));
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    void *din, *dout;
    {
        std::lock_guard<std::mutex> l(ctx->mu);
        din = ensure_buffer(ctx->stage_in, ctx->stage_in_bytes, in_need, "input staging allocation");
        dout = ensure_buffer(ctx->stage_out, ctx->stage_out_bytes, out_need, "output staging allocation");
    }
    host_upload(ctx, din, in, in_need, host_is_pageable(in), ctx->stream);
    execute_program(ctx, id, prog, din, dout, nullptr, ctx->stream);
    int local_err = 0;
    int *err = ctx->staging ? ctx->staging->pinned_word() : &local_err;
    *err = 0;
    check(cudaMemcpyAsync(err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream), "error word read");
    host_download(ctx, out, dout, out_need, host_is_pageable(out), ctx->stream);
    check(cudaStreamSynchronize(ctx->stream), "stream synchronize");
    if (*err) {
        const int e = *err;
        cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream);
        cudaStreamSynchronize(ctx->stream);
        fail_runtime("B200 FFT kernel reported error word " + std::to_string(e));
    }
}

static std::string describe_error_word(int err) {
    std::string m = "B200 FFT kernel reported error word " + std::to_string(err);
    if (err & 32) m += " (slab exchange barrier timed out: a peer rank did not arrive)";
    if (err & ~32) m += " (invalid pass program)";
    return m;
}

void context_synchronize(Context *ctx, cudaStream_t stream) {
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!stream) stream = ctx->stream;
    check(cudaStreamSynchronize(stream), "stream synchronize");
    int err = 0;
    check(cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost), "error word read");
    if (err) {
        check(cudaMemset(ctx->d_err, 0, sizeof(int)), "error word reset");
        check(cudaStreamSynchronize(cudaStreamLegacy), "stream synchronize");
        fail_runtime(describe_error_word(err));
    }
}

// ---- pipelined host execution ------------------------------------------------------

// The executed algorithm of two programs is the same when every pass runs the same
// kernel on the same op sequence (only line counts, grids and scratch sizes differ).
static bool same_algorithm(const Program &a, const Program &b) {
    if (a.passes.size() != b.passes.size() || a.tables.size() != b.tables.size()) return false;
    for (size_t i = 0; i < a.passes.size(); i++) {
        const PassPlan &x = a.passes[i], &y = b.passes[i];
        if (x.kernel != y.kernel || x.reg_variant != y.reg_variant || x.p.nops != y.p.nops) return false;
        for (int k = 0; k < x.p.nops; k++) {
            const Op &u = x.p.ops[k], &v = y.p.ops[k];
            if (u.type != v.type || u.radix != v.radix || u.len != v.len || u.flags != v.flags || u.mul != v.mul)
                return false;
        }
    }
    for (size_t i = 0; i < a.tables.size(); i++)
        if (a.tables[i].bytes(a.cbytes()) != b.tables[i].bytes(b.cbytes())) return false;
    return true;
}

static Transform *chunk_transform(Transform &t, size_t batch) {
    std::lock_guard<std::mutex> g(t.chunk_mu);
    auto it = t.chunks.find(batch);
    if (it != t.chunks.end()) return it->second.get();
    std::unique_ptr<Transform> c;
    try {
        FftConfig cfg = t.config;
        cfg.batch_count = batch;
        c = build_transform(cfg, t.direction, t.device);
        if (!same_algorithm(t.prog, c->prog)) c.reset();
    } catch (const FftError &) {
        c.reset();
    }
    return t.chunks.emplace(batch, std::move(c)).first->second.get();
}

// Mixed precision through the host API: the arrays are of the API type (f32 for F16
// storage, f64 for F64 compute / F32 storage, as execute_transform_f32 / _f64 take them);
// they are converted to and from the storage type around the execution.
static void execute_mixed_host(Context *ctx, Transform &t, const void *in, size_t in_bytes, void *out,
                               size_t out_bytes) {
    const Program &prog = t.prog;
    const size_t api = t.config.precision == Precision::F16StorageF32Compute ? 4 : 8;
    const size_t sb = prog.io_scalar_bytes();
    const size_t n_in = prog.input_elems * (prog.input_real ? 1 : 2), n_out = prog.output_elems * (prog.output_real ? 1 : 2);
    if (in_bytes != n_in * api) fail_input_length(prog.input_elems, in_bytes / (api * (prog.input_real ? 1 : 2)));
    if (out_bytes != n_out * api) fail_input_length(prog.output_elems, out_bytes / (api * (prog.output_real ? 1 : 2)));
    if (api == sb) {  // double-double with f64 storage: the host arrays are the storage type
        execute_program_host(ctx, t.id, prog, in, in_bytes, out, out_bytes);
        return;
    }
    std::vector<unsigned char> si(n_in * sb), so(n_out * sb);
    for (size_t k = 0; k < n_in; k++) {
        const double v = api == 8 ? static_cast<const double *>(in)[k] : static_cast<const float *>(in)[k];
        if (sb == 2)
            reinterpret_cast<__half *>(si.data())[k] = __float2half_rn((float)v);
        else
            reinterpret_cast<float *>(si.data())[k] = (float)v;
    }
    execute_program_host(ctx, t.id, prog, si.data(), si.size(), so.data(), so.size());
    for (size_t k = 0; k < n_out; k++) {
        const double v = sb == 2 ? (double)__half2float(reinterpret_cast<const __half *>(so.data())[k])
                                 : (double)reinterpret_cast<const float *>(so.data())[k];
        if (api == 8)
            static_cast<double *>(out)[k] = v;
        else
            static_cast<float *>(out)[k] = (float)v;
    }
}

// Host arrays are logical tensors (the reference packs formatted layouts internally,
// nd_real_ir.rs:715-750): a transform with formatted buffer strides runs its dense twin.
static Transform &host_view(Transform &t) {
    if (!t.formatted) return t;
    std::lock_guard<std::mutex> g(t.chunk_mu);
    if (!t.dense_twin) {
        FftConfig cfg = t.config;
        for (auto &v : cfg.input_buffer_axis_strides) v.reset();
        for (auto &v : cfg.output_buffer_axis_strides) v.reset();
        cfg.input_buffer_batch_stride.reset();
        cfg.output_buffer_batch_stride.reset();
        t.dense_twin = build_transform(cfg, t.direction, t.device);
    }
    return *t.dense_twin;
}

void execute_transform_host(Context *ctx, Transform &t_in, const void *in, size_t in_bytes, void *out,
                            size_t out_bytes) {
    std::lock_guard<std::mutex> host_lock(ctx->host_mu);  // the worker thread may run one too
    Transform &t = host_view(t_in);
    const Program &prog = t.prog;
    if (prog.storage_scalar_bytes) {
        execute_mixed_host(ctx, t, in, in_bytes, out, out_bytes);
        return;
    }
    const size_t in_need = prog.input_bytes(), out_need = prog.output_bytes();
    const size_t batch = t.plan.config.kernel_preparation_system_count();
    // input bytes per sub-batch: small enough that the unoverlapped first upload and last
    // download of a call stay short, large enough that each copy runs at full PCIe rate
    // (B200FFT_HOST_CHUNK_MB overrides the 32 MiB default)
    static const size_t kChunkBytes = [] {
        const char *e = std::getenv("B200FFT_HOST_CHUNK_MB");
        const long mb = e ? std::atol(e) : 32;
        return size_t(mb > 0 ? mb : 32) << 20;
    }();
    const size_t in_per = batch ? in_need / batch : 0, out_per = batch ? out_need / batch : 0;
    const size_t chunk = in_per ? std::max<size_t>(1, kChunkBytes / in_per) : 0;
    Transform *ct = nullptr, *rt = nullptr;
    const size_t nfull = chunk ? batch / chunk : 0, rem = chunk ? batch % chunk : 0;
    if (in_bytes == in_need && out_bytes == out_need && in_per * batch == in_need && out_per * batch == out_need &&
        nfull >= 3) {
        ct = chunk_transform(t, chunk);
        if (ct && rem) rt = chunk_transform(t, rem);
    }
    if (!ct || (rem && !rt)) {
        execute_program_host(ctx, t.id, prog, in, in_bytes, out, out_bytes);
        return;
    }
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    const size_t scr = std::max(ct->prog.scratch_bytes(), rt ? rt->prog.scratch_bytes() : 0);
    const size_t cin = (chunk * in_per + 255) & ~size_t(255), cout = (chunk * out_per + 255) & ~size_t(255);
    const size_t slot_bytes = cin + cout + ((scr + 255) & ~size_t(255));
    unsigned char *base;
    {
        std::lock_guard<std::mutex> l(ctx->mu);
        for (cudaStream_t &s : ctx->pipe)
            if (!s) check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
        base = static_cast<unsigned char *>(
            ensure_buffer(ctx->pipe_buf, ctx->pipe_bytes, Context::kPipeSlots * slot_bytes, "pipeline staging allocation"));
    }
    const size_t nchunks = nfull + (rem ? 1 : 0);
    // large pageable arrays go through the pinned staging sub-batch by sub-batch (a staged
    // download returns once its bytes are on the host); pinned ones overlap on the streams
    const bool page_in = host_is_pageable(in), page_out = host_is_pageable(out);
    for (size_t i = 0; i < nchunks; i++) {
        const int slot = (int)(i % Context::kPipeSlots);
        cudaStream_t s = ctx->pipe[slot];
        Transform *tt = i < nfull ? ct : rt;
        const size_t nb = i < nfull ? chunk : rem;
        unsigned char *din = base + slot * slot_bytes, *dout = din + cin, *dscr = dout + cout;
        host_upload(ctx, din, static_cast<const unsigned char *>(in) + i * chunk * in_per, nb * in_per, page_in, s);
        execute_program(ctx, tt->id, tt->prog, din, dout, scr ? dscr : nullptr, s);
        host_download(ctx, static_cast<unsigned char *>(out) + i * chunk * out_per, dout, nb * out_per, page_out, s);
    }
    for (cudaStream_t s : ctx->pipe) check(cudaStreamSynchronize(s), "stream synchronize");
    int err = 0;
    check(cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost), "error word read");
    if (err) {
        check(cudaMemset(ctx->d_err, 0, sizeof(int)), "error word reset");
        check(cudaStreamSynchronize(cudaStreamLegacy), "stream synchronize");
        fail_runtime(describe_error_word(err));
    }
}

// ---- asynchronous submissions ----------------------------------------------------------

static void worker_loop(Context *ctx) {
    for (;;) {
        std::function<void()> job;
        {
            std::unique_lock<std::mutex> l(ctx->job_mu);
            ctx->job_cv.wait(l, [&] { return ctx->stopping || !ctx->jobs.empty(); });
            if (ctx->jobs.empty()) return;  // stopping and drained
            job = std::move(ctx->jobs.front());
            ctx->jobs.pop_front();
        }
        job();
    }
}

std::shared_ptr<Ticket> submit_transform_host(Context *ctx, Transform &t, const void *in, size_t in_bytes, void *out,
                                              size_t out_bytes) {
    auto ticket = std::make_shared<Ticket>();
    auto job = [ctx, &t, in, in_bytes, out, out_bytes, ticket] {
        int status = 0;
        std::string message;
        try {
            execute_transform_host(ctx, t, in, in_bytes, out, out_bytes);
        } catch (const FftError &e) {
            status = e.code;
            message = e.message;
        } catch (const std::exception &e) {
            status = B200FFT_NATIVE_RUNTIME;
            message = std::string("CUDA runtime error: ") + e.what();
        }
        std::lock_guard<std::mutex> l(ticket->mu);
        ticket->status = status;
        ticket->message = std::move(message);
        ticket->done = true;
        ticket->cv.notify_all();
    };
    {
        std::lock_guard<std::mutex> l(ctx->job_mu);
        if (!ctx->worker.joinable()) ctx->worker = std::thread(worker_loop, ctx);
        ctx->jobs.push_back(std::move(job));
    }
    ctx->job_cv.notify_one();
    return ticket;
}

void wait_ticket(Ticket &t) {
    std::unique_lock<std::mutex> l(t.mu);
    t.cv.wait(l, [&] { return t.done; });
}

}  // namespace b200fft
