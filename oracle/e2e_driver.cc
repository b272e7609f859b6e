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
#include <functional>
#include <random>
#include <string>
#include <unordered_map>
#include <vector>

#include "backend_b200.h"
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

namespace {

vvllm::ModelConfig qwen05_config(int layers)
{
    vvllm::ModelConfig c;
    c.model_type = "qwen2";
    c.vocab_size = 151936;
    c.hidden_size = 896;
    c.intermediate_size = 4864;
    c.num_hidden_layers = (std::size_t)layers;
    c.num_attention_heads = 14;
    c.num_key_value_heads = 2;
    c.max_position_embeddings = 32768;
    c.rms_norm_eps = 1e-6;
    c.rope_theta = 1000000.0;
    c.bos_token_id = 151643;
    c.eos_token_ids = {151645};
    c.tie_word_embeddings = true;
    return c;
}

// N(mean, std) weights, seeded per tensor name (std::mt19937 + std::normal_distribution).
void add_tensor(std::unordered_map<std::string, vvllm::Tensor>& w, const std::string& name, std::size_t n,
                float mean, float stddev)
{
    vvllm::Tensor t({n}, vvllm::DType::Float32, vvllm::Device::CPU);
    std::mt19937 rng((unsigned)std::hash<std::string>{}(name) ^ 0x5eedu);
    std::normal_distribution<float> d(mean, stddev);
    float* p = t.data<float>();
    for (std::size_t i = 0; i < n; i++) p[i] = d(rng);
    w.emplace(name, std::move(t));
}

}  // namespace

// logits: (1 + n_decode) x vocab floats.  tokens: n_prompt prompt ids, then n_decode decode ids.
extern "C" __attribute__((visibility("default"))) int vvllm_e2e_logits(int use_b200, int layers, const int* tokens,
                                                                      int n_prompt, int n_decode, float* logits,
                                                                      long long* gpu_calls)
{
    const vvllm::ModelConfig cfg = qwen05_config(layers);
    const std::size_t H = cfg.hidden_size, I = cfg.intermediate_size;
    const std::size_t hd = H / cfg.num_attention_heads, kv = cfg.num_key_value_heads * hd;
    std::unordered_map<std::string, vvllm::Tensor> w;
    add_tensor(w, "model.embed_tokens.weight", cfg.vocab_size * H, 0.0f, 0.02f);
    add_tensor(w, "model.norm.weight", H, 1.0f, 0.02f);
    for (int l = 0; l < layers; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        add_tensor(w, p + "input_layernorm.weight", H, 1.0f, 0.02f);
        add_tensor(w, p + "post_attention_layernorm.weight", H, 1.0f, 0.02f);
        add_tensor(w, p + "self_attn.q_proj.weight", H * H, 0.0f, 0.02f);
        add_tensor(w, p + "self_attn.q_proj.bias", H, 0.0f, 0.02f);
        add_tensor(w, p + "self_attn.k_proj.weight", kv * H, 0.0f, 0.02f);
        add_tensor(w, p + "self_attn.k_proj.bias", kv, 0.0f, 0.02f);
        add_tensor(w, p + "self_attn.v_proj.weight", kv * H, 0.0f, 0.02f);
        add_tensor(w, p + "self_attn.v_proj.bias", kv, 0.0f, 0.02f);
        add_tensor(w, p + "self_attn.o_proj.weight", H * H, 0.0f, 0.02f);
        add_tensor(w, p + "mlp.gate_proj.weight", I * H, 0.0f, 0.02f);
        add_tensor(w, p + "mlp.up_proj.weight", I * H, 0.0f, 0.02f);
        add_tensor(w, p + "mlp.down_proj.weight", H * I, 0.0f, 0.02f);
    }
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
