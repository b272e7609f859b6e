// refgpu_driver.cc -- the reference's own GPU code path, as a checker and a timed baseline
// (test infrastructure only, never the product path).
//
// oracle/Makefile compiles this file with the reference's CUDA backend where it lies
// (src/backend/backend_cuda.cc and src/backend/cuda_kernels.cu for sm_100a, linked with
// cuBLAS), its Qwen2 forward pass (src/model/qwen2/model.cc, transformer_forward in
// include/vvllm/model/transformer.h:64-213), its CUDA KV cache (src/kv_cache/kv_cache_cuda.cc)
// and the device-resident adapter vvllm_b200/adapter/backend_b200_cuda.cc, into
// oracle/_ref/libvvllm_refgpu.so.  Nothing of the reference is copied here.
//
// vvllm_refgpu_logits: the logits of a prompt and a few decode steps of the seeded synthetic
//   Qwen2.5-0.5B-shaped model (oracle/e2e_model.h) with quantized projections, run on
//     0 = the reference CPU backend (fp32, CPU tensors),
//     1 = the reference CUDA backend (vvllm::BackendCUDA: cuBLAS GemmEx on an fp16 dequantized
//         copy of every int8 weight, src/backend/backend_cuda.cc:188-275),
//     2 = vvllm_b200::BackendB200 (the same CUDA backend with linear_q8 / linear_q8_add on the
//         B200 int8 kernels),
//   with fp32 or fp16 activations (backends 1 and 2; the CPU backend is fp32 only).
// vref_gpu_*: BackendCUDA::linear_q8 itself on caller device buffers, for the bench's timing of
//   the reference's GPU path.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "backend_b200_cuda.h"
#include "e2e_model.h"
#include "src/backend/backend_cuda.h"
#include "src/backend/backend_naive.h"
#include "src/kv_cache/kv_cache_cpu.h"
#include "src/kv_cache/kv_cache_cuda.h"
#include "vvllm/model/qwen2/model.h"

#define REFGPU_API extern "C" __attribute__((visibility("default")))

// logits: (1 + n_decode) x vocab floats (host).  tokens: n_prompt prompt ids, then n_decode
// decode ids.  b200_calls: linear_q8 / linear_q8_add calls the adapter served (backend 2).
REFGPU_API int vvllm_refgpu_logits(int backend, int fp16, int layers, const int* tokens, int n_prompt, int n_decode,
                                   float* logits, long long* b200_calls)
{
    if (backend < 0 || backend > 2 || (backend == 0 && fp16)) return -1;
    const vvllm::ModelConfig cfg = e2e::qwen05_config(layers);
    const std::unordered_map<std::string, vvllm::Tensor> w = e2e::make_weights(cfg);
    std::unique_ptr<vvllm::Backend> be;
    vvllm_b200::BackendB200* b200 = nullptr;
    if (backend == 0) {
        be = std::make_unique<vvllm::BackendCPU>();
    } else if (backend == 1) {
        be = std::make_unique<vvllm::BackendCUDA>(fp16 != 0);
    } else {
        b200 = new vvllm_b200::BackendB200(fp16 != 0, 0);
        be.reset(b200);
    }
    std::unique_ptr<vvllm::KVCache> kvc;
    if (backend == 0)
        kvc = std::make_unique<vvllm::KVCacheCPU>();
    else
        kvc = std::make_unique<vvllm::KVCacheCUDA>(fp16 != 0);
    const std::size_t V = cfg.vocab_size;
    auto take = [&](const vvllm::Tensor& t, float* dst) {
        if (backend == 0) {
            std::memcpy(dst, t.data<float>(), V * sizeof(float));
            return cudaSuccess;
        }
        return cudaMemcpy(dst, t.data<float>(), V * sizeof(float), cudaMemcpyDeviceToHost);
    };
    int rc = 0;
    {
        vvllm::Qwen2Model model(cfg, *be);
        model.load_weights(w, /*quantize=*/true);
        std::vector<int> prompt(tokens, tokens + n_prompt);
        vvllm::Tensor out = model.forward(prompt, 0, *kvc);
        if (take(out, logits) != cudaSuccess) rc = -2;
        for (int d = 0; d < n_decode && rc == 0; d++) {
            std::vector<int> one{tokens[n_prompt + d]};
            vvllm::Tensor o = model.forward(one, (std::size_t)(n_prompt + d), *kvc);
            if (take(o, logits + (std::size_t)(d + 1) * V) != cudaSuccess) rc = -2;
        }
    }
    if (b200_calls) *b200_calls = b200 ? (long long)b200->b200_calls() : 0;
    kvc.reset();
    be.reset();
    return rc;
}

// The reference's GPU linear_q8 on caller buffers: out / inp device pointers (fp16 behind the
// pointers when fp16 = 1), weight / scales / bias host pointers cached by the backend on first
// use (int8 upload, then the fp16 dequantized copy cuBLAS reads).
REFGPU_API void* vref_gpu_create(int fp16) { return new vvllm::BackendCUDA(fp16 != 0); }

REFGPU_API int vref_gpu_linear_q8(void* be, void* out, const void* inp, const int8_t* weight, const float* scales,
                                  const float* bias, size_t M, size_t N, size_t K)
{
    static_cast<vvllm::BackendCUDA*>(be)->linear_q8(static_cast<float*>(out), static_cast<const float*>(inp), weight,
                                                    scales, bias, M, N, K);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

REFGPU_API void vref_gpu_destroy(void* be) { delete static_cast<vvllm::BackendCUDA*>(be); }
