// e2e_driver.cc -- forward-pass checker (test infrastructure only, never the product path).
//
// Runs the reference's own Qwen2 forward pass (src/model/qwen2/model.cc and
// transformer_forward, include/vvllm/model/transformer.h:64-213), compiled from
// the reference sources where they lie, on a seeded synthetic Qwen2.5-0.5B-shaped
// model with quantized projections, once with the reference CPU backend and once
// with vvllm_b200::BackendB200Host (the hot path on the GPU behind the unchanged
// Backend interface).  Returns the logits of every forward call.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "backend_b200.h"
#include "e2e_model.h"
#include "src/backend/backend_naive.h"
#include "src/kv_cache/kv_cache_cpu.h"
#include "vvllm/model/qwen2/model.h"

// The reference's tensor.cc links CUDA memory helpers for device tensors (tensor.cc:11-17);
// this checker makes CPU tensors only, so they are never reached.
extern "C" {
void* cuda_malloc(size_t) { std::fprintf(stderr, "e2e_driver: unexpected device tensor\n"); std::abort(); }
void cuda_free(void*) { std::abort(); }
void cuda_memcpy_h2d(void*, const void*, size_t) { std::abort(); }
void cuda_memcpy_d2h(void*, const void*, size_t) { std::abort(); }
void cuda_memcpy_d2d(void*, const void*, size_t) { std::abort(); }
}


// logits: (1 + n_decode) x vocab floats.  tokens: n_prompt prompt ids, then n_decode decode ids.
extern "C" __attribute__((visibility("default"))) int vvllm_e2e_logits(int use_b200, int layers, const int* tokens,
                                                                      int n_prompt, int n_decode, float* logits,
                                                                      long long* gpu_calls)
{
    const vvllm::ModelConfig cfg = e2e::qwen05_config(layers);
    const std::unordered_map<std::string, vvllm::Tensor> w = e2e::make_weights(cfg);
    vvllm::BackendCPU cpu;
    vvllm_b200::BackendB200Host* b200 = use_b200 ? new vvllm_b200::BackendB200Host(0) : nullptr;
    vvllm::Backend& be = use_b200 ? static_cast<vvllm::Backend&>(*b200) : static_cast<vvllm::Backend&>(cpu);
    {
        vvllm::Qwen2Model model(cfg, be);
        model.load_weights(w, /*quantize=*/true);
        vvllm::KVCacheCPU kvc;
        std::vector<int> prompt(tokens, tokens + n_prompt);
        vvllm::Tensor out = model.forward(prompt, 0, kvc);
        std::memcpy(logits, out.data<float>(), cfg.vocab_size * sizeof(float));
        for (int d = 0; d < n_decode; d++) {
            std::vector<int> one{tokens[n_prompt + d]};
            vvllm::Tensor o = model.forward(one, (std::size_t)(n_prompt + d), kvc);
            std::memcpy(logits + (std::size_t)(d + 1) * cfg.vocab_size, o.data<float>(),
                        cfg.vocab_size * sizeof(float));
        }
    }
    if (gpu_calls) *gpu_calls = b200 ? (long long)b200->gpu_calls() : 0;
    delete b200;
    return 0;
}
