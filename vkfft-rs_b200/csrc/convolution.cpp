// FFT convolution application (convolution_ir.rs): placeholder until the fused
// multiply passes land.
#include "transform.hpp"

namespace b200fft {

std::unique_ptr<Convolution> build_convolution(const FftConfig &, const DeviceProfile &, const void *, uint64_t) {
    fail_unsupported("B200 engine: FFT convolution is not implemented yet");
}

}  // namespace b200fft
