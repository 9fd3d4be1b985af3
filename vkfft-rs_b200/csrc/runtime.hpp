// CUDA execution context: the B200 counterpart of the reference's
// CudaExecutionContext (backend/cuda/runtime.rs:959-2840).  Owns a stream, a device
// error word, lazily uploaded per-transform tables and a growable scratch arena.
#pragma once

#include <cuda_runtime.h>

#include <mutex>
#include <string>
#include <unordered_map>

#include "transform.hpp"

namespace b200fft {

struct DeviceTables {
    void *base = nullptr;
    std::vector<const void *> ptrs;
    std::vector<const void *> jit;  // per pass: specialised kernel (jit.cpp) or null
};

bool jit_enabled();
std::vector<const void *> jit_kernels_for(const Program &prog, int device);
int jit_compile_check(const Program &prog, std::string &log);

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
    // pipelined host execution: streams and per-slot staging (input, output, scratch)
    static constexpr int kPipeSlots = 3;
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
void execute_program(Context *ctx, uint64_t id, const Program &prog, const void *in, void *out, void *workspace,
                     cudaStream_t stream, const PeerStore *peer = nullptr);
// Stream-ordered execution out of the library's static device region (allocates nothing).
void execute_program_static(Context *ctx, uint64_t id, const Program &prog, const void *in, void *out,
                            cudaStream_t stream);
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
