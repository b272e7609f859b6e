// backend_b200_cuda.h -- device-resident vvllm::Backend adapter: the reference's CUDA backend with
// the quantized-linear hot path replaced by the B200 kernels.
//
// BackendB200 derives from vvllm::BackendCUDA (src/backend/backend_cuda.h) and overrides only
// Backend::linear_q8 and Backend::linear_q8_add (include/vvllm/backend/backend.h:62-65, :75-78).
// Everything else -- embedding, RMSNorm, RoPE, attention, the fp32 lm_head `linear`, fp16
// conversions, the KV cache -- stays the reference's GPU code, so transformer_forward
// (include/vvllm/model/transformer.h:64-213) runs unchanged with device tensors.
//
// Conventions are BackendCUDA's (src/backend/backend_cuda.cc:188-275): out / inp / residual are
// device pointers, fp16 data behind float* when the backend was built with fp16 = true
// (transformer.h:82, :93); weight / scales / bias are host pointers owned by the model, uploaded
// on first use and cached by host address.  The difference is what is cached: the int8 weight
// stays int8 on the device (1 byte per weight read per call), where BackendCUDA builds an fp16
// dequantized copy and reads 2 bytes per weight through cuBLAS.  Work goes to the legacy default
// stream, the stream BackendCUDA's kernels and cuBLAS handle use, so the order of the forward
// pass is kept.
//
// Failures are fail-stop, as in the reference (src/backend/cuda_kernels.cu:11-21): a non-zero
// status prints the library's message and aborts.
#pragma once

#include <cstddef>
#include <cstdint>

#include "src/backend/backend_cuda.h"

struct b200q8_backend;

namespace vvllm_b200 {

class BackendB200 : public vvllm::BackendCUDA {
public:
    explicit BackendB200(bool fp16 = false, int device = 0);
    ~BackendB200() override;
    BackendB200(const BackendB200&) = delete;
    BackendB200& operator=(const BackendB200&) = delete;

    void linear_q8(float* out, const float* inp, const int8_t* weight, const float* scales, const float* bias,
                   std::size_t M, std::size_t N, std::size_t K) override;
    void linear_q8_add(float* out, const float* inp, const int8_t* weight, const float* scales, const float* bias,
                       const float* residual, std::size_t M, std::size_t N, std::size_t K) override;

    std::size_t b200_calls() const { return calls_; }
    std::size_t cached_bytes() const;

private:
    b200q8_backend* be_ = nullptr;
    std::size_t calls_ = 0;
};

}  // namespace vvllm_b200
