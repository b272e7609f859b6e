// backend_b200.cc -- see backend_b200.h.
#include "backend_b200.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "b200q8.h"

namespace vvllm_b200 {
namespace {

void check_status(int st, const char* what)
{
    if (st != B200Q8_OK) {
        std::fprintf(stderr, "BackendB200Host: %s failed (status %d): %s\n", what, st, b200q8_last_error());
        std::abort();
    }
}

void check_cuda(cudaError_t e, const char* what)
{
    if (e != cudaSuccess) {
        std::fprintf(stderr, "BackendB200Host: %s failed: %s\n", what, cudaGetErrorString(e));
        std::abort();
    }
}

}  // namespace

BackendB200Host::BackendB200Host(int device)
{
    check_status(b200q8_backend_create(device, /*fp16=*/0, &be_), "b200q8_backend_create");
}

BackendB200Host::~BackendB200Host()
{
    for (float* p : buf_)
        if (p) cudaFree(p);
    if (be_) b200q8_backend_destroy(be_);
}

float* BackendB200Host::device_buffer(int which, std::size_t floats)
{
    if (cap_[which] < floats) {
        if (buf_[which]) cudaFree(buf_[which]);
        buf_[which] = nullptr;
        check_cuda(cudaMalloc(&buf_[which], floats * sizeof(float)), "cudaMalloc");
        cap_[which] = floats;
    }
    return buf_[which];
}

void BackendB200Host::linear_q8(float* out, const float* inp, const int8_t* weight, const float* scales,
                                const float* bias, std::size_t M, std::size_t N, std::size_t K)
{
    if (M == 0 || N == 0) return;
    float* d_in = device_buffer(0, M * K);
    float* d_out = device_buffer(1, M * N);
    check_cuda(cudaMemcpy(d_in, inp, M * K * sizeof(float), cudaMemcpyHostToDevice), "H2D input");
    check_status(b200q8_backend_linear_q8(be_, d_out, d_in, weight, scales, bias, M, N, K), "linear_q8");
    check_cuda(cudaMemcpy(out, d_out, M * N * sizeof(float), cudaMemcpyDeviceToHost), "D2H output");
    calls_++;
}

void BackendB200Host::linear_q8_add(float* out, const float* inp, const int8_t* weight, const float* scales,
                                    const float* bias, const float* residual, std::size_t M, std::size_t N,
                                    std::size_t K)
{
    if (M == 0 || N == 0) return;
    float* d_in = device_buffer(0, M * K);
    float* d_out = device_buffer(1, M * N);
    float* d_res = device_buffer(2, M * N);
    check_cuda(cudaMemcpy(d_in, inp, M * K * sizeof(float), cudaMemcpyHostToDevice), "H2D input");
    // out may alias residual (transformer.h:165-166, :187-188): read it before anything is written
    check_cuda(cudaMemcpy(d_res, residual, M * N * sizeof(float), cudaMemcpyHostToDevice), "H2D residual");
    check_status(b200q8_backend_linear_q8_add(be_, d_out, d_in, weight, scales, bias, d_res, M, N, K),
                 "linear_q8_add");
    check_cuda(cudaMemcpy(out, d_out, M * N * sizeof(float), cudaMemcpyDeviceToHost), "D2H output");
    calls_++;
}

}  // namespace vvllm_b200
