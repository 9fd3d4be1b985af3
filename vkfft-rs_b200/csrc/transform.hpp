// TransformIr analogue: device-scored plan + executed child plans + B200 program.
#pragma once

#include <map>
#include <memory>
#include <mutex>
#include <optional>

#include "lower.hpp"

namespace b200fft {

struct Transform {
    uint64_t id = 0;
    FftConfig config;  // with device-resolved tuning
    int direction = 0;
    DeviceProfile device;
    FftPlan plan;  // FftPlan::build_for_device
    int family = B200FFT_FAMILY_COMPLEX_1D;
    RealAlgorithm real_algorithm = RealAlgorithm::FullComplex;
    size_t real_transform_len = 0;
    // executed 1D child plan per tensor axis (empty for omitted axes)
    std::vector<std::optional<FftPlan>> children;
    Program prog;
    // same transform over a sub-batch, for pipelined host execution (runtime.cpp);
    // null when planning the sub-batch changes the executed algorithm
    std::mutex chunk_mu;
    std::map<size_t, std::unique_ptr<Transform>> chunks;
    // logical (host-API) element counts; prog.input_elems / output_elems are the device
    // buffers', which differ with formatted strides
    size_t logical_in_elems = 0, logical_out_elems = 0;
    bool formatted = false;
    std::unique_ptr<Transform> dense_twin;  // same transform on dense buffers (host API)
};

std::unique_ptr<Transform> build_transform(const FftConfig &config, int direction, const DeviceProfile &device);

// Convolution application (convolution_ir.rs:3867-4250, ND real, independent coordinates).
struct Convolution {
    uint64_t id = 0;
    FftConfig config;
    DeviceProfile device;
    std::unique_ptr<Transform> forward;  // R2C over the image, batch = coordinates
    std::unique_ptr<Transform> inverse;  // normalised C2R
    Program prog;                        // forward + multiply + inverse, one launch list
    size_t spectrum_elems = 0;           // complex elements of one spectrum copy
    // logical (host-API) element counts; prog.input_elems / output_elems are the device
    // buffers', which differ with formatted strides
    size_t logical_in_elems = 0, logical_out_elems = 0;
    std::unique_ptr<Convolution> dense_twin;  // same convolution on dense buffers (host API)
};

std::unique_ptr<Convolution> build_convolution(const FftConfig &config, const DeviceProfile &device,
                                               const void *spectrum, uint64_t copies);

const char *precision_name(Precision p);

}  // namespace b200fft
