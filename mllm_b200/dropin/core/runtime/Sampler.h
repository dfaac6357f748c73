// Drop-in replacement for the mLLM reference's src/core/runtime/Sampler.h (+ Sampler.cpp).
//
// Same class and static entry point, Sampler::Sample(logits, temperature, top_k, top_p,
// use_greedy, previous_tokens, repetition_penalty), with the reference's argument checks and
// messages (Sampler.cpp:59-81).  The work runs on the device in one launch (mllm_sample): the
// repetition penalty is applied in place as the reference does (Sampler.cpp:12-46) but without
// its device sync per previous token, then the greedy argmax or the top-k / top-p draw.  Per
// call that is one copy of the history to the device and one read of the token back.
// Host logits are copied to the current CUDA device and sampled there.
// Header-only: link it instead of the reference's Sampler.cpp.
#pragma once

#include <torch/torch.h>

#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <vector>

#include "core/runtime/B200Device.h"

namespace mllm
{
    class Sampler
    {
    public:
        static int64_t Sample(
            torch::Tensor logits,
            float temperature,
            int top_k,
            float top_p,
            bool use_greedy,
            const std::vector<int64_t>& previous_tokens,
            float repetition_penalty)
        {
            if (logits.dim() != 1)
            {
                throw std::runtime_error("Sampler expects 1D logits tensor.");
            }
            if (logits.size(0) <= 0)
            {
                throw std::runtime_error("Sampler received empty logits.");
            }
            if (!std::isfinite(temperature))
            {
                throw std::runtime_error("Sampler temperature must be finite.");
            }
            if (!std::isfinite(top_p) || top_p <= 0.0f)
            {
                throw std::runtime_error("Sampler top_p must be in (0, 1].");
            }
            if (!logits.is_cuda())
            {
                // host logits (LlamaRunner keeps its lm_head on the host): sampled on the device;
                // the repetition penalty's in-place writes are copied back, as the reference
                // leaves them in its argument (Sampler.cpp:12-46)
                const torch::Device dev = b200::ComputeDevice("Sampler");
                torch::Tensor d = logits.to(dev).contiguous();
                const int64_t token =
                    Sample(d, temperature, top_k, top_p, use_greedy, previous_tokens, repetition_penalty);
                if (repetition_penalty > 1.0f && !previous_tokens.empty())
                {
                    logits.copy_(d);
                }
                return token;
            }
            if (logits.scalar_type() != torch::kBFloat16 && logits.scalar_type() != torch::kFloat32)
            {
                throw std::runtime_error("Sampler: logits must be bf16 or fp32.");
            }
            if (logits.stride(0) != 1)
            {
                throw std::runtime_error("Sampler: logits must be contiguous.");
            }
            const int64_t V = logits.size(0);
            const auto dev = logits.device();
            torch::Tensor prev, counts;
            if (repetition_penalty > 1.0f && !previous_tokens.empty())
            {
                prev = torch::tensor(previous_tokens, torch::kInt64).to(dev, /*non_blocking=*/true);
                counts = torch::tensor({(int32_t)previous_tokens.size()}, torch::kInt32).to(dev, true);
            }
            // the draw's stream: a seed from LibTorch's default generator (so torch::manual_seed
            // makes runs repeatable) and a per-process call counter
            static uint64_t calls = 0;
            const uint64_t seed = (uint64_t)torch::randint(INT64_MAX, {1}, torch::kInt64).item<int64_t>();
            auto out = torch::empty({1}, torch::TensorOptions().dtype(torch::kInt64).device(dev));
            const size_t bytes = mllm_sample_workspace_size(1, (int)V);
            auto ws = b200::SamplerWorkspace(bytes, dev);
            b200::Check(mllm_sample(logits.data_ptr(), logits.scalar_type() == torch::kBFloat16, V, 1, (int)V,
                                    prev.defined() ? prev.data_ptr<int64_t>() : nullptr, 0,
                                    counts.defined() ? counts.data_ptr<int32_t>() : nullptr, temperature, top_k,
                                    top_p, use_greedy, repetition_penalty, seed, calls++, out.data_ptr<int64_t>(),
                                    ws.data_ptr(), (size_t)ws.numel(), b200::CurrentStream()),
                        "Sampler");
            return out.item<int64_t>();
        }
    };
}
