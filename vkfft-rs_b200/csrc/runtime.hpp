// CUDA execution context: the B200 counterpart of the reference's
// CudaExecutionContext (backend/cuda/runtime.rs:959-2840).  Owns a stream, a device
// error word, lazily uploaded per-transform tables and a growable scratch arena.
#pragma once

#include <cuda_runtime.h>

#include <condition_variable>
#include <deque>
#include <functional>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>

#include "aot.hpp"
#include "host_staging.hpp"
#include "transform.hpp"

namespace b200fft {

struct DeviceTables {
    void *base = nullptr;
    std::vector<const void *> ptrs;
    std::vector<const void *> spec;  // per pass: ahead-of-time specialised kernel (aot.hpp) or null
};

struct Context {
    int device = 0;
    cudaStream_t stream = nullptr;
    int *d_err = nullptr;
    DeviceProfile profile;
    std::string name;
    int sm_count = 0;
    std::mutex mu;
    std::unordered_map<uint64_t, DeviceTables> tables;  // by Program owner id
    void *scratch = nullptr;
    size_t scratch_bytes = 0;
    void *stage_in = nullptr, *stage_out = nullptr;
    size_t stage_in_bytes = 0, stage_out_bytes = 0;
    std::mutex host_mu;  // host executions (staging buffers, pipeline streams) one at a time
    // pinned staging of large pageable host arrays (created by the first host call needing it)
    std::unique_ptr<HostStaging> staging;
    // asynchronous submissions: one worker thread runs them in submission order
    std::mutex job_mu;
    std::condition_variable job_cv;
    std::deque<std::function<void()>> jobs;
    std::thread worker;
    bool stopping = false;
    // pipelined host execution: streams and per-slot staging (input, output, scratch)
    static constexpr int kPipeSlots = 4;
    cudaStream_t pipe[kPipeSlots] = {};
    void *pipe_buf = nullptr;
    size_t pipe_bytes = 0;
};

int probe_devices();
Context *context_create(int device);
void context_destroy(Context *ctx);
void forget_program(uint64_t id);  // drop uploaded tables of a destroyed transform from every context

// Stream-ordered execution of a program on device pointers.  peer: the exchange
// buffers of the ranks for passes marked peer_scatter (slab transforms only).
// before_last: an event recorded on the stream just before the last pass is launched
// (the slab's phase timing), or null.
void execute_program(Context *ctx, uint64_t id, const Program &prog, const void *in, void *out, void *workspace,
                     cudaStream_t stream, const PeerStore *peer = nullptr, cudaEvent_t before_last = nullptr);
// Stream-ordered execution out of the library's static device region (allocates nothing).
void execute_program_static(Context *ctx, uint64_t id, const Program &prog, const void *in, void *out,
                            cudaStream_t stream);
// Result of an asynchronous submission (NativeAsyncRuntime tickets, native_runtime.rs:362-451).
struct Ticket {
    std::mutex mu;
    std::condition_variable cv;
    bool done = false;
    int status = 0;
    std::string message;
};
// Queues a host execution (copy semantics) on the context's worker; the arrays must
// stay valid until the ticket is waited for.
std::shared_ptr<Ticket> submit_transform_host(Context *ctx, Transform &t, const void *in, size_t in_bytes, void *out,
                                              size_t out_bytes);
void wait_ticket(Ticket &t);

// Waits for the stream (null: the context's) and turns a recorded kernel error into
// a NativeRuntime error (clearing it).
void context_synchronize(Context *ctx, cudaStream_t stream);
// Host-buffer execution of a transform with copy semantics: large batched transforms are
// split into sub-batches whose upload, transform and download overlap on three streams.
void execute_transform_host(Context *ctx, Transform &t, const void *in, size_t in_bytes, void *out,
                            size_t out_bytes);
// Synchronous host-buffer execution with copy semantics.
void execute_program_host(Context *ctx, uint64_t id, const Program &prog, const void *in, size_t in_bytes, void *out,
                          size_t out_bytes);

}  // namespace b200fft
