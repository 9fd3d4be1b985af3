// Slab-decomposed multi-GPU transform (one process per GPU): plans in slab_plan.cpp,
// exchange and execution in slab.cu.
#pragma once

#include <memory>
#include <optional>

#include "transform.hpp"

struct CUstream_st;

namespace b200fft {

struct Context;

struct Slab {
    uint64_t id_pre = 0, id_post = 0;  // program ids (table cache keys)
    FftConfig config;
    int direction = 0;
    int nranks = 1, rank = 0;
    DeviceProfile device;
    size_t planes_per_rank = 0, columns_per_rank = 0;
    size_t exchange_elems = 0;  // complex elements of one exchange buffer
    size_t input_elems = 0, output_elems = 0;
    bool input_real = false, output_real = false;
    RealAlgorithm real_algorithm = RealAlgorithm::FullComplex;
    std::vector<std::optional<FftPlan>> children;  // executed 1D child plan per axis
    Program pre;   // local FFTs ending in the exchange pass
    Program post;  // FFTs after the exchange
    PeerStore peer{};  // chunk / offset of the exchange pass (pointers set per call)
    // attachment to one context (device)
    Context *ctx = nullptr;
    void *local = nullptr;  // [epoch flags | exchange buffer 0 | exchange buffer 1]
    void *peer_ptr[kMaxPeers] = {};
    bool connected = false;
    unsigned epoch = 0;
    unsigned long long timeout_ns = 20ull * 1000000000ull;
    // phase timing (b200fft_slab_set_phase_timing): events bracketing the local passes,
    // the exchange pass, the barrier and the passes after it, recorded by every call
    bool timing = false;
    void *events[5] = {};  // cudaEvent_t, created on the attached context's device

    size_t buffer_bytes() const;
    ~Slab();
};

std::unique_ptr<Slab> build_slab(const FftConfig &config, int direction, int nranks, int rank,
                                 const DeviceProfile &device);
void slab_attach(Context *ctx, Slab *s, unsigned char *handle_out);
void slab_connect(Context *ctx, Slab *s, const unsigned char *handles);
void execute_slab(Context *ctx, Slab *s, const void *in, void *out, void *workspace, CUstream_st *stream);
void release_slab_device(Slab *s);  // frees the exchange buffers and peer mappings (slab.cu)
void slab_set_phase_timing(Slab *s, bool enabled);
// Milliseconds of the last call's phases: [local passes, exchange pass, barrier, passes
// after the exchange]; waits for that call to finish.
void slab_phase_times(Slab *s, float ms[4]);

}  // namespace b200fft
