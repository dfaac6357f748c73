// Drop-in replacement for the mLLM reference's src/core/runtime/Attention.h.
//
// Same class, same static entry points and signatures:
//   Attention::Forward          (Attention.h:29-86)   project q/k/v, then ForwardProjected
//   Attention::ForwardProjected (Attention.h:100-326) RoPE, KV append, GQA attention, o_proj
// and the same argument checks and messages (Attention.h:42-47, 129-144).  Behind them the
// LibTorch chain (RoPE ops, torch::cat, repeat_interleave, fp32 score matrix, mask, softmax,
// two matmuls, merge) becomes B200 kernels reached through the C ABI (mllm_attn.h):
//   S > 1:  mllm_qkv_epilogue_bf16 (RoPE + optional per-head QK-RMSNorm + in-place KV append),
//           then mllm_prefill_attention_bf16 (causal GQA attention on tcgen05 tensor cores)
//   S == 1: mllm_decode_step_bf16 (the same epilogue for the new token fused into split-K
//           flash-decode over the cache, one launch)
// The projections stay LibTorch GEMMs (Linear::Forward), as in the reference, except that up to
// 256 tokens q/k/v come from one mllm_linear_bf16 launch (b200::ProjectQKV).
//
// Host tensors (a runner that keeps its weights on the host, as LlamaRunner does) are staged on
// the current CUDA device -- weights once, activations per call -- and the result returns to the
// host; the computation itself is the same device path.
//
// ForwardProjectedNormed is the one addition: it takes the per-head q/k RMSNorm weights that
// the reference applies in TransformerBlock.h:103-134 and fuses that norm into the epilogue.
#pragma once

#include <torch/torch.h>

#include <cmath>
#include <stdexcept>

#include "core/runtime/B200Device.h"
#include "core/runtime/KVCache.h"
#include "core/runtime/Linear.h"
#include "core/runtime/RoPE.h"

namespace mllm
{
    class Attention
    {
    public:
        static torch::Tensor Forward(
            const torch::Tensor& hidden,
            const torch::Tensor& w_q,
            const torch::Tensor& w_k,
            const torch::Tensor& w_v,
            const torch::Tensor& w_o,
            int num_heads,
            int num_kv_heads,
            int head_dim,
            double rope_theta,
            const torch::Tensor& position_ids,
            KVCache* kv_cache)
        {
            if (hidden.dim() != 3)
            {
                throw std::runtime_error("Attention: hidden must be [B, S, H].");
            }
            if (!hidden.is_cuda())
            {
                // host tensors (a runner that keeps its weights on the host): computed on the
                // device, returned on the host
                const torch::Device dev = b200::ComputeDevice("Attention");
                return Forward(b200::StageActivation(hidden, dev), b200::StageWeight(w_q, dev),
                               b200::StageWeight(w_k, dev), b200::StageWeight(w_v, dev), b200::StageWeight(w_o, dev),
                               num_heads, num_kv_heads, head_dim, rope_theta, position_ids.to(dev), kv_cache)
                    .to(hidden.device(), hidden.scalar_type());
            }
            const auto B = hidden.size(0);
            const auto S = hidden.size(1);
            // [B, S, h*D] -> [B, h, S, D] views; the epilogue reads them through their strides.
            torch::Tensor q, k, v;
            if (!b200::ProjectQKV(hidden, w_q, w_k, w_v, num_heads, num_kv_heads, head_dim, &q, &k, &v))
            {
                q = Linear::Forward(hidden, w_q).view({B, S, num_heads, head_dim}).transpose(1, 2);
                k = Linear::Forward(hidden, w_k).view({B, S, num_kv_heads, head_dim}).transpose(1, 2);
                v = Linear::Forward(hidden, w_v).view({B, S, num_kv_heads, head_dim}).transpose(1, 2);
            }
            return ForwardProjected(q, k, v, w_o, num_heads, num_kv_heads, head_dim, rope_theta,
                                    position_ids, kv_cache);
        }

        static torch::Tensor ForwardProjected(
            torch::Tensor q,
            torch::Tensor k,
            torch::Tensor v,
            const torch::Tensor& w_o,
            int num_heads,
            int num_kv_heads,
            int head_dim,
            double rope_theta,
            const torch::Tensor& position_ids,
            KVCache* kv_cache)
        {
            if (q.defined() && !q.is_cuda())
            {
                const torch::Device dev = b200::ComputeDevice("Attention");
                return ForwardProjectedNormed(b200::StageActivation(q, dev), b200::StageActivation(k, dev),
                                              b200::StageActivation(v, dev), b200::StageWeight(w_o, dev), num_heads,
                                              num_kv_heads, head_dim, rope_theta, position_ids.to(dev), kv_cache,
                                              torch::Tensor(), torch::Tensor(), 0.0)
                    .to(q.device(), q.scalar_type());
            }
            return ForwardProjectedNormed(q, k, v, w_o, num_heads, num_kv_heads, head_dim, rope_theta,
                                          position_ids, kv_cache, torch::Tensor(), torch::Tensor(), 0.0);
        }

        // q [B, H, S, D], k/v [B, Hkv, S, D]: projections before the per-head norm when the
        // norm weights are given (Qwen3), otherwise exactly the reference's ForwardProjected input.
        static torch::Tensor ForwardProjectedNormed(
            const torch::Tensor& q,
            const torch::Tensor& k,
            const torch::Tensor& v,
            const torch::Tensor& w_o,
            int num_heads,
            int num_kv_heads,
            int head_dim,
            double rope_theta,
            const torch::Tensor& position_ids,
            KVCache* kv_cache,
            const torch::Tensor& q_norm_weight,
            const torch::Tensor& k_norm_weight,
            double rms_norm_eps)
        {
            if (q.dim() != 4 || k.dim() != 4 || v.dim() != 4)
            {
                throw std::runtime_error("Attention::ForwardProjected: q/k/v must be rank-4 tensors.");
            }
            if (num_heads % num_kv_heads != 0)
            {
                throw std::runtime_error("Attention: num_heads must be divisible by num_kv_heads.");
            }
            b200::RequireCudaBf16(q, "Attention");
            b200::RequireCudaBf16(k, "Attention");
            b200::RequireCudaBf16(v, "Attention");
            const int64_t B = q.size(0);
            const int64_t S = q.size(2);
            if (q.size(1) != num_heads || k.size(1) != num_kv_heads || v.size(1) != num_kv_heads ||
                q.size(3) != head_dim || k.size(3) != head_dim || v.size(3) != head_dim ||
                k.size(0) != B || v.size(0) != B || k.size(2) != S || v.size(2) != S)
            {
                throw std::runtime_error("Attention: q/k/v shapes do not match the head geometry.");
            }
            if (position_ids.numel() != S)
            {
                throw std::runtime_error("Attention: position_ids must hold one position per new token.");
            }

            KVCache scratch;  // kv_cache == nullptr: attend over this call's rows only
            KVCache* cache = (kv_cache != nullptr) ? kv_cache : &scratch;
            cache->Reserve(B, num_kv_heads, head_dim, cache->length + S, q.options());
            const int64_t start = cache->length;
            const auto& ks = cache->key_storage;
            const auto& vs = cache->value_storage;

            auto pos = position_ids.to(q.device(), torch::kInt64).contiguous();
            torch::Tensor qn, kn;
            if (q_norm_weight.defined() != k_norm_weight.defined())
            {
                throw std::runtime_error("Attention: give both q/k norm weights or neither.");
            }
            if (q_norm_weight.defined())
            {
                qn = q_norm_weight.to(q.device(), torch::kBFloat16).contiguous();
                kn = k_norm_weight.to(q.device(), torch::kBFloat16).contiguous();
                if (qn.numel() != head_dim || kn.numel() != head_dim)
                {
                    throw std::runtime_error("RMSNorm: last dim of x must match weight length.");
                }
            }
            const mllm_stream_t stream = b200::CurrentStream();
            const float scale = (float)(1.0 / std::sqrt((double)head_dim));
            auto out = torch::empty({B, S, (int64_t)num_heads * head_dim}, q.options());
            if (S == 1)
            {
                // decode: the new token's epilogue (QK-norm, RoPE, append at row `start`) and the
                // attention over all start + 1 rows in one fused launch.  While a CUDA graph of the
                // layer is recorded, the lengths come from the device (row lens[b] - 1 is appended)
                // and the plan covers the cache's capacity, so that every replay is valid.
                b200::DecodeGraphContext* graph = b200::ActiveDecodeGraph();
                const int64_t L = start + 1;
                const int64_t plan_len = graph ? graph->plan_len : L;
                const size_t bytes =
                    mllm_decode_attention_workspace_size((int)B, num_heads, num_kv_heads, head_dim, (int)plan_len);
                auto ws = b200::DecodeWorkspace(bytes, q.device());
                b200::Check(
                    mllm_decode_step_bf16(
                        q.data_ptr(), q.stride(0), q.stride(1), k.data_ptr(), k.stride(0), k.stride(1),
                        v.data_ptr(), v.stride(0), v.stride(1), pos.data_ptr<int64_t>(), 0, rope_theta,
                        nullptr, nullptr, 0, qn.defined() ? qn.data_ptr() : nullptr,
                        kn.defined() ? kn.data_ptr() : nullptr, rms_norm_eps, ks.data_ptr(), vs.data_ptr(),
                        ks.stride(0), ks.stride(1), ks.stride(2), graph ? graph->lens.data_ptr<int32_t>() : nullptr,
                        (int)B, num_heads, num_kv_heads, head_dim, (int)plan_len, scale, out.data_ptr(),
                        ws.data_ptr(), (size_t)ws.numel(), stream),
                    "Attention (decode step)");
                if (graph == nullptr)
                {
                    cache->SetLength(L);
                }
            }
            else
            {
                auto q_rot = torch::empty({B, num_heads, S, head_dim}, q.options());
                b200::Check(
                    mllm_qkv_epilogue_bf16(
                        q.data_ptr(), q.stride(0), q.stride(2), q.stride(1),
                        k.data_ptr(), k.stride(0), k.stride(2), k.stride(1),
                        v.data_ptr(), v.stride(0), v.stride(2), v.stride(1),
                        (int)B, (int)S, num_heads, num_kv_heads, head_dim,
                        pos.data_ptr<int64_t>(), 0, pos.stride(0), rope_theta,
                        nullptr, nullptr, 0, 0,
                        qn.defined() ? qn.data_ptr() : nullptr, kn.defined() ? kn.data_ptr() : nullptr,
                        rms_norm_eps, q_rot.data_ptr(),
                        ks.data_ptr(), vs.data_ptr(), ks.stride(0), ks.stride(1), ks.stride(2), cache->Capacity(),
                        nullptr, start, stream),
                    "Attention (QKV epilogue)");
                cache->SetLength(start + S);
                const int64_t L = cache->length;
                b200::Check(mllm_prefill_attention_bf16(q_rot.data_ptr(), ks.data_ptr(), vs.data_ptr(), ks.stride(0),
                                                        ks.stride(1), ks.stride(2), (int)B, num_heads, num_kv_heads,
                                                        head_dim, (int)S, (int)L, scale, out.data_ptr(), stream),
                            "Attention (prefill)");
            }
            return Linear::Forward(out, w_o);
        }
    };
}
