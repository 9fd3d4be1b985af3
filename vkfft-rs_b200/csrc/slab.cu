// Slab-decomposed multi-GPU transforms: one process per GPU, the planes of axis 0 split
// evenly over the ranks, one exchange step (the all-to-all transpose) between the local
// FFTs of the higher axes and the FFT of axis 0.
//
// Forward, rank g of P, global dims [D0, D1, ...] (compact last axis for R2C):
//   input  [D0/P, D1, H]   planes g*D0/P .. of axis 0           (H = product of the rest)
//   local FFTs of the last axes; the axis-1 FFT pass stores every element straight into
//   the exchange buffer of its owner rank r = k1 / (D1/P) over NVLink (peer pointers
//   from CUDA IPC) in pencil layout [D0, D1/P, H];
//   barrier (epoch flags written into every peer, bounded wait);
//   axis-0 FFT exchange -> output [D0, D1/P, H] (axis-1 indices g*D1/P ..).
// Inverse is the mirror image: the axis-0 FFT pass scatters into the ranks' slabs
// [D0/P, D1, H], then the higher axes run locally.
//
// The exchange is therefore fused into the FFT pass that produces the data: no pack
// kernel, no staging copy, no library collective.  Exchange buffers are double-buffered
// by call parity, so one barrier per call orders both the arrival of this call's data
// and the peers' reads of the buffer from the call before.
#include <cuda_runtime.h>

#include <cstring>

#include "runtime.hpp"
#include "slab.hpp"

namespace b200fft {

namespace {

constexpr size_t kFlagBytes = 256;  // epoch flags, one uint32 per rank, at the start of the exchange allocation

struct BarrierParams {
    unsigned *flags[kMaxPeers];  // rank r's flag array (peer mapping, own one at [rank])
    int rank, n;
    unsigned epoch;
    int *err;
    unsigned long long timeout_ns;
};

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Thread r tells rank r that this rank's data has landed (release, system scope), then
// waits for rank r's word in this rank's own flags (acquire).  The wait gives up after
// timeout_ns, records error bit 32 in the context's error word and returns.
__global__ void slab_barrier_kernel(const __grid_constant__ BarrierParams bp) {
    const int r = threadIdx.x;
    if (r < bp.n) {
        __threadfence_system();
        unsigned *dst = bp.flags[r] + bp.rank;
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(dst), "r"(bp.epoch) : "memory");
    }
    __syncthreads();
    if (r < bp.n) {
        const unsigned *src = bp.flags[bp.rank] + r;
        const unsigned long long t0 = global_ns();
        for (;;) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(src) : "memory");
            if ((int)(v - bp.epoch) >= 0) break;
            if (global_ns() - t0 > bp.timeout_ns) {
                atomicOr(bp.err, 32);
                break;
            }
            __nanosleep(256);
        }
        __threadfence_system();
    }
}

void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) fail_runtime(std::string(what) + " failed: " + cudaGetErrorString(e));
}

}  // namespace

void release_slab_device(Slab *s) {
    forget_program(s->id_pre);
    forget_program(s->id_post);
    if (s->ctx) {
        cudaSetDevice(s->ctx->device);
        cudaStreamSynchronize(s->ctx->stream);
        for (void *&e : s->events)
            if (e) {
                cudaEventSynchronize(static_cast<cudaEvent_t>(e));
                cudaEventDestroy(static_cast<cudaEvent_t>(e));
                e = nullptr;
            }
        for (int r = 0; r < s->nranks; r++)
            if (r != s->rank && s->peer_ptr[r]) cudaIpcCloseMemHandle(s->peer_ptr[r]);
        if (s->local) cudaFree(s->local);
    }
}

void slab_attach(Context *ctx, Slab *s, unsigned char *handle_out) {
    if (s->ctx && s->ctx != ctx) fail_unsupported("slab transform is attached to another context");
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!s->local) {
        void *p = nullptr;
        check(cudaMalloc(&p, kFlagBytes + 2 * s->buffer_bytes()), "slab exchange allocation");
        cudaError_t e = cudaMemset(p, 0, kFlagBytes);
        if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);  // before any peer or barrier
        if (e != cudaSuccess) {
            cudaFree(p);
            check(e, "cudaMemset");
        }
        s->local = p;
        s->ctx = ctx;
    }
    cudaIpcMemHandle_t h;
    check(cudaIpcGetMemHandle(&h, s->local), "cudaIpcGetMemHandle");
    std::memset(handle_out, 0, B200FFT_SLAB_HANDLE_BYTES);
    static_assert(sizeof(cudaIpcMemHandle_t) <= 64, "IPC handle size");
    std::memcpy(handle_out, &h, sizeof(h));
    check(cudaDeviceGetPCIBusId(reinterpret_cast<char *>(handle_out) + 64, 32, ctx->device), "cudaDeviceGetPCIBusId");
}

void slab_connect(Context *ctx, Slab *s, const unsigned char *handles) {
    if (s->ctx != ctx || !s->local) fail_unsupported("attach the slab transform to this context first");
    if (s->connected) fail_unsupported("slab transform is already connected");
    const int P = s->nranks;
    for (int a = 0; a < P; a++)
        for (int b = a + 1; b < P; b++)
            if (std::strncmp(reinterpret_cast<const char *>(handles) + a * B200FFT_SLAB_HANDLE_BYTES + 64,
                             reinterpret_cast<const char *>(handles) + b * B200FFT_SLAB_HANDLE_BYTES + 64, 32) == 0)
                throw FftError(B200FFT_UNSUPPORTED_KERNEL_PATH, "slab ranks " + std::to_string(a) + " and " +
                                                                    std::to_string(b) +
                                                                    " share one GPU; every rank needs its own device");
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    for (int r = 0; r < P; r++) {
        if (r == s->rank) {
            s->peer_ptr[r] = s->local;
            continue;
        }
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handles + r * B200FFT_SLAB_HANDLE_BYTES, sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; q++)
                if (q != s->rank && s->peer_ptr[q]) {
                    cudaIpcCloseMemHandle(s->peer_ptr[q]);
                    s->peer_ptr[q] = nullptr;
                }
            check(e, "cudaIpcOpenMemHandle of a peer's exchange buffer");
        }
        s->peer_ptr[r] = p;
    }
    s->connected = true;
}

void slab_set_phase_timing(Slab *s, bool enabled) {
    if (enabled && !s->ctx) fail_unsupported("attach the slab transform to a context before enabling phase timing");
    if (enabled && !s->events[0]) {
        check(cudaSetDevice(s->ctx->device), "cudaSetDevice");
        for (void *&e : s->events) {
            cudaEvent_t ev;
            check(cudaEventCreate(&ev), "cudaEventCreate");
            e = ev;
        }
    }
    s->timing = enabled;
}

void slab_phase_times(Slab *s, float ms[4]) {
    if (!s->timing || !s->events[0]) fail_unsupported("phase timing is not enabled on this slab transform");
    check(cudaSetDevice(s->ctx->device), "cudaSetDevice");
    check(cudaEventSynchronize(static_cast<cudaEvent_t>(s->events[4])), "cudaEventSynchronize");
    for (int k = 0; k < 4; k++)
        check(cudaEventElapsedTime(&ms[k], static_cast<cudaEvent_t>(s->events[k]),
                                   static_cast<cudaEvent_t>(s->events[k + 1])),
              "cudaEventElapsedTime");
}

void execute_slab(Context *ctx, Slab *s, const void *in, void *out, void *workspace, CUstream_st *stream) {
    if (s->ctx != ctx || !s->connected) fail_unsupported("slab transform is not connected on this context");
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!stream) stream = ctx->stream;
    const unsigned epoch = ++s->epoch;
    const size_t buf_off = kFlagBytes + (epoch & 1) * s->buffer_bytes();
    PeerStore ps = s->peer;
    for (int r = 0; r < s->nranks; r++) ps.ptr[r] = static_cast<unsigned char *>(s->peer_ptr[r]) + buf_off;
    auto ev = [&](int k) { return s->timing ? static_cast<cudaEvent_t>(s->events[k]) : nullptr; };
    if (s->timing) check(cudaEventRecord(ev(0), stream), "cudaEventRecord");
    execute_program(ctx, s->id_pre, s->pre, in, out, workspace, stream, &ps, ev(1));
    if (s->timing) check(cudaEventRecord(ev(2), stream), "cudaEventRecord");
    BarrierParams bp{};
    for (int r = 0; r < s->nranks; r++) bp.flags[r] = static_cast<unsigned *>(s->peer_ptr[r]);
    bp.rank = s->rank;
    bp.n = s->nranks;
    bp.epoch = epoch;
    bp.err = ctx->d_err;
    bp.timeout_ns = s->timeout_ns;
    slab_barrier_kernel<<<1, 32, 0, stream>>>(bp);
    check(cudaGetLastError(), "slab barrier launch");
    if (s->timing) check(cudaEventRecord(ev(3), stream), "cudaEventRecord");
    execute_program(ctx, s->id_post, s->post, static_cast<unsigned char *>(s->local) + buf_off, out, workspace, stream);
    if (s->timing) check(cudaEventRecord(ev(4), stream), "cudaEventRecord");
}

}  // namespace b200fft
