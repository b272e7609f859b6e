// backend_b200_cuda.cc -- see backend_b200_cuda.h.
#include "backend_b200_cuda.h"

#include <cstdio>
#include <cstdlib>

#include "b200q8.h"

namespace vvllm_b200 {
namespace {

void check_status(int st, const char* what)
{
    if (st != B200Q8_OK) {
        std::fprintf(stderr, "BackendB200: %s failed (status %d): %s\n", what, st, b200q8_last_error());
        std::abort();
    }
}

}  // namespace

BackendB200::BackendB200(bool fp16, int device) : vvllm::BackendCUDA(fp16)
{
    check_status(b200q8_backend_create(device, fp16 ? 1 : 0, &be_), "b200q8_backend_create");
}

BackendB200::~BackendB200()
{
    if (be_) b200q8_backend_destroy(be_);
}

std::size_t BackendB200::cached_bytes() const
{
    std::size_t n = 0;
    check_status(b200q8_backend_cached_bytes(be_, &n), "b200q8_backend_cached_bytes");
    return n;
}

void BackendB200::linear_q8(float* out, const float* inp, const int8_t* weight, const float* scales,
                            const float* bias, std::size_t M, std::size_t N, std::size_t K)
{
    check_status(b200q8_backend_linear_q8(be_, out, inp, weight, scales, bias, M, N, K), "linear_q8");
    calls_++;
}

// out may be residual itself (transformer.h:165-166, :187-188): the library reads each residual
// element before it writes that output element.
void BackendB200::linear_q8_add(float* out, const float* inp, const int8_t* weight, const float* scales,
                                const float* bias, const float* residual, std::size_t M, std::size_t N,
                                std::size_t K)
{
    check_status(b200q8_backend_linear_q8_add(be_, out, inp, weight, scales, bias, residual, M, N, K),
                 "linear_q8_add");
    calls_++;
}

}  // namespace vvllm_b200
