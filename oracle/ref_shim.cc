// ref_shim.cc -- extern "C" entry points into the reference's own CPU code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference sources where they lie (src/backend/backend_naive.cc and
// src/quantize/quantize.cc of hoobean1996/vvllm, flags as in its
// src/backend/BUILD.bazel:5-8 and .bazelrc:2) into oracle/_ref/libvvllm_ref.so.
// Nothing of the reference is copied here; this file only forwards to
//   vvllm::quantize_per_channel   (include/vvllm/quantize/quantize.h:18)
//   vvllm::BackendCPU::linear_q8  (src/backend/backend_naive.h:30-31)
//   vvllm::BackendCPU::linear_q8_add (src/backend/backend_naive.h:35-37)
//   vvllm::BackendCPU::rms_norm, silu_mul (src/backend/backend_naive.cc:67-75, :293-300),
//     applied per token the way src/model/transformer.cc:40-50 and
//     include/vvllm/model/transformer.h:175-180 apply them
// It is used to pin oracle/q8_oracle.c bit-for-bit, to make the golden
// fixtures under tests/golden/, and as the timed CPU baseline of bench.py.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "src/backend/backend_naive.h"
#include "vvllm/quantize/quantize.h"

extern "C" {

int vref_quantize_per_channel(const float* w, size_t N, size_t K, int8_t* q, float* scales)
{
    vvllm::QuantizedWeight qw = vvllm::quantize_per_channel(w, N, K);
    std::memcpy(q, qw.data.data(), N * K);
    std::memcpy(scales, qw.scales.data(), N * sizeof(float));
    return 0;
}

int vref_linear_q8(float* out, const float* inp, const int8_t* weight, const float* scales,
                   const float* bias, size_t M, size_t N, size_t K)
{
    vvllm::BackendCPU be;
    be.linear_q8(out, inp, weight, scales, bias, M, N, K);
    return 0;
}

int vref_linear_q8_add(float* out, const float* inp, const int8_t* weight, const float* scales,
                       const float* bias, const float* residual, size_t M, size_t N, size_t K)
{
    vvllm::BackendCPU be;
    be.linear_q8_add(out, inp, weight, scales, bias, residual, M, N, K);
    return 0;
}

int vref_rms_norm(float* out, const float* x, const float* w, size_t M, size_t K, float eps)
{
    vvllm::BackendCPU be;
    for (size_t m = 0; m < M; m++) be.rms_norm(out + m * K, x + m * K, w, K, eps);
    return 0;
}

int vref_silu_mul(float* out, const float* gate_up, size_t M, size_t K)
{
    vvllm::BackendCPU be;
    for (size_t m = 0; m < M; m++) be.silu_mul(out + m * K, gate_up + m * 2 * K, gate_up + m * 2 * K + K, K);
    return 0;
}

// The reference is single-threaded.  This harness-level parallel variant gives
// each of nthreads host threads a disjoint slice of output channels and calls
// the unmodified BackendCPU::linear_q8 on it; every output element is computed
// by the same code as in the single-threaded call, so results are identical.
int vref_linear_q8_mt(float* out, const float* inp, const int8_t* weight, const float* scales,
                      const float* bias, size_t M, size_t N, size_t K, int nthreads)
{
    if (nthreads < 1) nthreads = 1;
    if (static_cast<size_t>(nthreads) > N) nthreads = static_cast<int>(N ? N : 1);
    std::vector<std::thread> pool;
    pool.reserve(nthreads);
    for (int t = 0; t < nthreads; t++) {
        size_t j0 = N * t / nthreads, j1 = N * (t + 1) / nthreads;
        pool.emplace_back([=]() {
            vvllm::BackendCPU be;
            size_t n = j1 - j0;
            if (n == 0) return;
            if (M == 1) {
                be.linear_q8(out + j0, inp, weight + j0 * K, scales + j0, bias ? bias + j0 : nullptr,
                             1, n, K);
                return;
            }
            std::vector<float> tmp(M * n);
            be.linear_q8(tmp.data(), inp, weight + j0 * K, scales + j0, bias ? bias + j0 : nullptr, M,
                         n, K);
            for (size_t i = 0; i < M; i++)
                std::memcpy(out + i * N + j0, tmp.data() + i * n, n * sizeof(float));
        });
    }
    for (auto& th : pool) th.join();
    return 0;
}

}  // extern "C"
