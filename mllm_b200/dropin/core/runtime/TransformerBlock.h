// Drop-in replacement for the mLLM reference's src/core/runtime/TransformerBlock.h.
//
// `LayerWeights` keeps the reference's exact member list (TransformerBlock.h:13-46), because
// the unchanged runners fill it field by field (QwenRunner.cpp, LlamaRunner.cpp).
// `TransformerBlock::Forward` keeps the reference's signature (TransformerBlock.h:51-62) and
// its sequence of steps: pre-norm (RMSNorm), attention, residual add, post-norm, SwiGLU MLP,
// residual add.  The only change is inside the Qwen3 branch (use_qk_norm): the per-head q/k
// RMSNorm (TransformerBlock.h:103-107,130-134) moves into the fused QKV epilogue kernel, so
// the projections go straight from the q/k/v GEMMs into Attention::ForwardProjectedNormed, and up
// to 256 tokens the three GEMMs are one mllm_linear_bf16 launch (b200::ProjectQKV).
// RMSNorm, Linear and MLP are the reference's own headers, unchanged.
#pragma once

#include <torch/torch.h>

#include "core/runtime/Attention.h"
#include "core/runtime/KVCache.h"
#include "core/runtime/Linear.h"
#include "core/runtime/MLP.h"
#include "core/runtime/RMSNorm.h"

namespace mllm
{
    struct LayerWeights
    {
        torch::Tensor input_layernorm;
        torch::Tensor post_attention_layernorm;

        torch::Tensor w_q;
        torch::Tensor w_k;
        torch::Tensor w_v;
        torch::Tensor w_o;

        // Qwen3 per-head QK-norm weights (undefined for Llama)
        torch::Tensor w_q_norm;
        torch::Tensor w_k_norm;

        torch::Tensor w_gate;
        torch::Tensor w_up;
        torch::Tensor w_down;

        // FP8 block scales (undefined for FP16/BF16 models)
        torch::Tensor w_q_scale;
        torch::Tensor w_k_scale;
        torch::Tensor w_v_scale;
        torch::Tensor w_o_scale;
        torch::Tensor w_gate_scale;
        torch::Tensor w_up_scale;
        torch::Tensor w_down_scale;
    };

    class TransformerBlock
    {
    public:
        static torch::Tensor Forward(
            const torch::Tensor& hidden,
            const LayerWeights& lw,
            int num_heads,
            int num_kv_heads,
            int head_dim,
            double rope_theta,
            double rms_norm_eps,
            bool use_qk_norm,
            const torch::Tensor& position_ids,
            KVCache* kv_cache)
        {
            torch::Tensor attn_in = RMSNorm::Forward(hidden, lw.input_layernorm, rms_norm_eps);
            torch::Tensor attn_out;
            if (use_qk_norm)
            {
                const auto B = attn_in.size(0);
                const auto S = attn_in.size(1);
                torch::Tensor q, k, v;
                if (!b200::ProjectQKV(attn_in, lw.w_q, lw.w_k, lw.w_v, num_heads, num_kv_heads, head_dim, &q, &k,
                                      &v))
                {
                    q = Linear::Forward(attn_in, lw.w_q).view({B, S, num_heads, head_dim}).transpose(1, 2);
                    k = Linear::Forward(attn_in, lw.w_k).view({B, S, num_kv_heads, head_dim}).transpose(1, 2);
                    v = Linear::Forward(attn_in, lw.w_v).view({B, S, num_kv_heads, head_dim}).transpose(1, 2);
                }
                attn_out = Attention::ForwardProjectedNormed(q, k, v, lw.w_o, num_heads, num_kv_heads, head_dim,
                                                             rope_theta, position_ids, kv_cache, lw.w_q_norm,
                                                             lw.w_k_norm, rms_norm_eps);
            }
            else
            {
                attn_out = Attention::Forward(attn_in, lw.w_q, lw.w_k, lw.w_v, lw.w_o, num_heads, num_kv_heads,
                                              head_dim, rope_theta, position_ids, kv_cache);
            }
            torch::Tensor h = hidden + attn_out;
            torch::Tensor mlp_in = RMSNorm::Forward(h, lw.post_attention_layernorm, rms_norm_eps);
            return h + MLP::Forward(mlp_in, lw.w_gate, lw.w_up, lw.w_down);
        }
    };
}
