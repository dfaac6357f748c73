// Test infrastructure only: a Python binding around the UNMODIFIED mLLM
// reference runtime headers (src/core/runtime/*.h of the reference tree),
// compiled from the reference sources where they lie by oracle/build_ref.py.
// Nothing here is product code; the product never links this file.
//
// Each function forwards to the reference symbol named beside it, so the
// checker and the CPU baseline run the reference's own LibTorch code path.
#include <torch/extension.h>

#include "core/runtime/TransformerBlock.h"  // Attention.h, RoPE.h, KVCache.h, RMSNorm.h, MLP.h, Linear.h
#include "core/runtime/Sampler.h"

#include <tuple>

namespace {

using torch::Tensor;

// RoPE::BuildCosSin  (src/core/runtime/RoPE.h:29-59)
std::tuple<Tensor, Tensor> rope_build_cos_sin(const Tensor& positions, int64_t head_dim, double theta) {
    auto cs = mllm::RoPE::BuildCosSin(positions, static_cast<int>(head_dim), theta);
    return {cs.first, cs.second};
}

// RoPE::Apply  (src/core/runtime/RoPE.h:68-89)
Tensor rope_apply(const Tensor& x, const Tensor& cos, const Tensor& sin) {
    return mllm::RoPE::Apply(x, cos, sin);
}

// RMSNorm::Forward  (src/core/runtime/RMSNorm.h:27-64)
Tensor rms_norm(const Tensor& x, const Tensor& w, double eps) {
    return mllm::RMSNorm::Forward(x, w, eps);
}

// Linear::Forward  (src/core/runtime/Linear.h:33-68)
Tensor linear(const Tensor& x, const Tensor& w) {
    return mllm::Linear::Forward(x, w);
}

// KVCache (src/core/runtime/KVCache.h:9-28) marshalled as an optional
// (key, value) pair: undefined tensors mean "not initialised".
mllm::KVCache make_cache(const c10::optional<Tensor>& key, const c10::optional<Tensor>& value) {
    mllm::KVCache c;
    if (key.has_value() && value.has_value()) {
        c.key = *key;
        c.value = *value;
    }
    return c;
}

// Attention::Forward  (src/core/runtime/Attention.h:29-86)
std::tuple<Tensor, Tensor, Tensor> attention_forward(
    const Tensor& hidden, const Tensor& w_q, const Tensor& w_k, const Tensor& w_v, const Tensor& w_o,
    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, double rope_theta,
    const Tensor& position_ids, const c10::optional<Tensor>& cache_key,
    const c10::optional<Tensor>& cache_value, bool use_cache) {
    mllm::KVCache cache = make_cache(cache_key, cache_value);
    Tensor out = mllm::Attention::Forward(hidden, w_q, w_k, w_v, w_o, (int)num_heads, (int)num_kv_heads,
                                          (int)head_dim, rope_theta, position_ids,
                                          use_cache ? &cache : nullptr);
    return {out, cache.key, cache.value};
}

// Attention::ForwardProjected  (src/core/runtime/Attention.h:100-326)
std::tuple<Tensor, Tensor, Tensor> attention_forward_projected(
    const Tensor& q, const Tensor& k, const Tensor& v, const Tensor& w_o,
    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, double rope_theta,
    const Tensor& position_ids, const c10::optional<Tensor>& cache_key,
    const c10::optional<Tensor>& cache_value, bool use_cache) {
    mllm::KVCache cache = make_cache(cache_key, cache_value);
    Tensor out = mllm::Attention::ForwardProjected(q, k, v, w_o, (int)num_heads, (int)num_kv_heads,
                                                   (int)head_dim, rope_theta, position_ids,
                                                   use_cache ? &cache : nullptr);
    return {out, cache.key, cache.value};
}

// TransformerBlock::Forward  (src/core/runtime/TransformerBlock.h:51-220)
std::tuple<Tensor, Tensor, Tensor> transformer_block_forward(
    const Tensor& hidden, const std::map<std::string, Tensor>& w,
    int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, double rope_theta, double eps,
    bool use_qk_norm, const Tensor& position_ids, const c10::optional<Tensor>& cache_key,
    const c10::optional<Tensor>& cache_value, bool use_cache) {
    mllm::LayerWeights lw;
    auto get = [&](const char* n) -> Tensor {
        auto it = w.find(n);
        return it == w.end() ? Tensor() : it->second;
    };
    lw.input_layernorm = get("input_layernorm");
    lw.post_attention_layernorm = get("post_attention_layernorm");
    lw.w_q = get("w_q");
    lw.w_k = get("w_k");
    lw.w_v = get("w_v");
    lw.w_o = get("w_o");
    lw.w_q_norm = get("w_q_norm");
    lw.w_k_norm = get("w_k_norm");
    lw.w_gate = get("w_gate");
    lw.w_up = get("w_up");
    lw.w_down = get("w_down");
    mllm::KVCache cache = make_cache(cache_key, cache_value);
    Tensor out = mllm::TransformerBlock::Forward(hidden, lw, (int)num_heads, (int)num_kv_heads,
                                                 (int)head_dim, rope_theta, eps, use_qk_norm,
                                                 position_ids, use_cache ? &cache : nullptr);
    return {out, cache.key, cache.value};
}

// Sampler::Sample (Sampler.cpp:49-232) on a copy of `logits`; returns the token and the copy,
// which the reference's repetition penalty modifies in place.
std::tuple<int64_t, Tensor> sample(Tensor logits, double temperature, int64_t top_k, double top_p, bool use_greedy,
                                   std::vector<int64_t> previous_tokens, double repetition_penalty) {
    Tensor x = logits.clone();
    const int64_t tok = mllm::Sampler::Sample(x, (float)temperature, (int)top_k, (float)top_p, use_greedy,
                                              previous_tokens, (float)repetition_penalty);
    return {tok, x};
}

void set_num_threads(int64_t n) { at::set_num_threads((int)n); }
int64_t get_num_threads() { return at::get_num_threads(); }

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "mLLM reference runtime (src/core/runtime) compiled as the parity oracle; test use only";
    m.def("rope_build_cos_sin", &rope_build_cos_sin);
    m.def("rope_apply", &rope_apply);
    m.def("rms_norm", &rms_norm);
    m.def("linear", &linear);
    m.def("attention_forward", &attention_forward);
    m.def("attention_forward_projected", &attention_forward_projected);
    m.def("transformer_block_forward", &transformer_block_forward);
    m.def("sample", &sample);
    m.def("set_num_threads", &set_num_threads);
    m.def("get_num_threads", &get_num_threads);
}
