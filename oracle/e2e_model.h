// e2e_model.h -- the seeded synthetic model both forward-pass checkers build (test
// infrastructure only): a Qwen2.5-0.5B-shaped config with `layers` layers and every weight
// N(mean, std) from std::mt19937 seeded by the tensor's name.
#pragma once

#include <cstddef>
#include <functional>
#include <random>
#include <string>
#include <unordered_map>

#include "vvllm/model/qwen2/model.h"

namespace e2e {

inline vvllm::ModelConfig qwen05_config(int layers)
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
inline void add_tensor(std::unordered_map<std::string, vvllm::Tensor>& w, const std::string& name, std::size_t n,
                       float mean, float stddev)
{
    vvllm::Tensor t({n}, vvllm::DType::Float32, vvllm::Device::CPU);
    std::mt19937 rng((unsigned)std::hash<std::string>{}(name) ^ 0x5eedu);
    std::normal_distribution<float> d(mean, stddev);
    float* p = t.data<float>();
    for (std::size_t i = 0; i < n; i++) p[i] = d(rng);
    w.emplace(name, std::move(t));
}

// Every tensor Qwen2Model::load_weights reads (src/model/qwen2/model.cc), host fp32.
inline std::unordered_map<std::string, vvllm::Tensor> make_weights(const vvllm::ModelConfig& cfg)
{
    const std::size_t H = cfg.hidden_size, I = cfg.intermediate_size;
    const std::size_t hd = H / cfg.num_attention_heads, kv = cfg.num_key_value_heads * hd;
    std::unordered_map<std::string, vvllm::Tensor> w;
    add_tensor(w, "model.embed_tokens.weight", cfg.vocab_size * H, 0.0f, 0.02f);
    add_tensor(w, "model.norm.weight", H, 1.0f, 0.02f);
    for (std::size_t l = 0; l < cfg.num_hidden_layers; l++) {
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
    return w;
}

}  // namespace e2e
