// backend_b200.h -- vvllm::Backend adapter that runs the quantized-linear hot path on a B200.
//
// Drop-in for vvllm's `Backend::linear_q8` / `linear_q8_add`
// (include/vvllm/backend/backend.h:62-65, :75-78).  Built against the
// reference's own headers; the reference is not modified.
//
// BackendB200Host keeps the reference CPU backend (src/backend/backend_naive.h)
// for every non-hot op and sends only linear_q8 / linear_q8_add to the GPU
// through libb200q8's C ABI: host activations are copied to the device, the
// int8 weights are uploaded once and cached by host address (as
// backend_cuda.cc:51-59 does), and the result is copied back.  It lets the
// reference's unchanged transformer_forward run with the B200 kernels behind
// the interface.  A production engine keeps activations on the device and
// subclasses the CUDA backend instead (same two overrides, no copies).
//
// Failures are fail-stop, like the reference (src/backend/cuda_kernels.cu:11-21):
// a non-zero status prints the library's message and aborts.
#pragma once

#include <cstddef>
#include <cstdint>

#include "src/backend/backend_naive.h"

struct b200q8_backend;

namespace vvllm_b200 {

class BackendB200Host : public vvllm::BackendCPU {
public:
    explicit BackendB200Host(int device = 0);
    ~BackendB200Host() override;
    BackendB200Host(const BackendB200Host&) = delete;
    BackendB200Host& operator=(const BackendB200Host&) = delete;

    void linear_q8(float* out, const float* inp, const int8_t* weight, const float* scales, const float* bias,
                   std::size_t M, std::size_t N, std::size_t K) override;
    void linear_q8_add(float* out, const float* inp, const int8_t* weight, const float* scales, const float* bias,
                       const float* residual, std::size_t M, std::size_t N, std::size_t K) override;

    std::size_t gpu_calls() const { return calls_; }

private:
    float* device_buffer(int which, std::size_t floats);

    b200q8_backend* be_ = nullptr;
    float* buf_[3] = {nullptr, nullptr, nullptr};  // inp, out, residual
    std::size_t cap_[3] = {0, 0, 0};
    std::size_t calls_ = 0;
};

}  // namespace vvllm_b200
