// Python binding of the mLLM model runners, compiled two ways (mllm_b200/dropin/build_facade.py):
//
//   * "reference": against the reference tree's own runtime headers -> oracle/_ref/mllm_ref_runner
//   * "dropin":    with mllm_b200/dropin ahead on the include path  -> tests/facade/mllm_dropin_runner
//
// The runner sources (QwenRunner.cpp, LlamaRunner.cpp, Sampler.cpp, tokenizers) are the
// reference's, unchanged, in both builds; only the core/runtime headers they include differ.
// That is what makes the drop-in claim testable: the same runner code, the same weights, the
// same input ids, with and without the B200 attention path.  Test infrastructure only.
#include <torch/extension.h>

#include "core/runtime/TransformerBlock.h"
#include "models/base/ModelRunnerFactory.h"

#include <memory>
#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

namespace {

using torch::Tensor;

class Runner {
public:
    explicit Runner(const std::string& path) {
        bundle_ = mllm::ModelRunnerFactory::Create(path);
        if (!bundle_.runner->Load(path)) throw std::runtime_error("runner Load failed for " + path);
    }
    // IModelRunner::Forward: prefill when S > 1 or the cache is empty, decode otherwise
    // (QwenRunner.cpp:301-324 decides; nothing here changes that).
    Tensor forward(const Tensor& ids) { return bundle_.runner->Forward(ids, Tensor()); }
    void reset_cache() { bundle_.runner->InitKVCache(0, 0); }
    std::string model_type() const { return bundle_.runner->GetModelType(); }
    // IModelRunner::Generate with greedy sampling (batch 1, the reference's own loop).
    std::vector<int64_t> generate(const std::vector<int64_t>& ids, int max_new_tokens, float repetition_penalty) {
        mllm::GenerateOptions o;
        o.max_new_tokens = max_new_tokens;
        o.use_greedy = true;
        o.repetition_penalty = repetition_penalty;
        o.eos_token_id = -1;   // random weights: never stop early
        return bundle_.runner->Generate(ids, o).tokens;
    }

private:
    mllm::ModelBundle bundle_;
};

// A KVCache held across calls, for driving TransformerBlock::Forward step by step.
struct Cache {
    mllm::KVCache c;
    Tensor key() const { return c.key; }
    Tensor value() const { return c.value; }
    bool initialized() const { return c.IsInitialized(); }
    void clear() { c.Clear(); }
};

Tensor block_forward(const Tensor& hidden, const std::map<std::string, Tensor>& w, int64_t H, int64_t Hkv,
                     int64_t D, double theta, double eps, bool qk_norm, const Tensor& pos, Cache* cache) {
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
    return mllm::TransformerBlock::Forward(hidden, lw, (int)H, (int)Hkv, (int)D, theta, eps, qk_norm, pos,
                                           cache ? &cache->c : nullptr);
}

#ifdef MLLM_DROPIN
// The drop-in's tensor-parallel mode: `comm` is an mllm_comm_t made by mllm_comm_init (passed as
// an integer address); world 1 turns it off.
void set_tensor_parallel(int64_t comm, int rank, int world) {
    mllm::b200::SetTensorParallel(reinterpret_cast<mllm_comm_t>(comm), rank, world);
}
#endif

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
#ifdef MLLM_DROPIN
    m.def("set_tensor_parallel", &set_tensor_parallel, pybind11::arg("comm"), pybind11::arg("rank"),
          pybind11::arg("world"));
#endif
    pybind11::class_<Runner>(m, "Runner")
        .def(pybind11::init<const std::string&>())
        .def("forward", &Runner::forward)
        .def("reset_cache", &Runner::reset_cache)
        .def("model_type", &Runner::model_type)
        .def("generate", &Runner::generate, pybind11::arg("ids"), pybind11::arg("max_new_tokens"),
             pybind11::arg("repetition_penalty") = 1.0f);
    pybind11::class_<Cache>(m, "Cache")
        .def(pybind11::init<>())
        .def("key", &Cache::key)
        .def("value", &Cache::value)
        .def("initialized", &Cache::initialized)
        .def("clear", &Cache::clear);
    m.def("block_forward", &block_forward, pybind11::arg("hidden"), pybind11::arg("weights"), pybind11::arg("H"),
          pybind11::arg("Hkv"), pybind11::arg("D"), pybind11::arg("theta"), pybind11::arg("eps"),
          pybind11::arg("qk_norm"), pybind11::arg("pos"), pybind11::arg("cache") = nullptr);
}
