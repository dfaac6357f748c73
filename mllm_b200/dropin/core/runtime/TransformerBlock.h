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
//
// A runner that keeps its weights on the host (LlamaRunner) is served on the GPU all the same:
// the layer's weights are staged on the device once and the hidden state per call (FromHost).
//
// With b200::SetTensorParallel (one process per GPU, a communicator from mllm_comm_init), each
// rank runs its KV-head group of the attention and the o_proj partials are all-reduced
// (HeadSharded); the unchanged runners drive it exactly as they drive one GPU.
//
// With MLLM_B200_DECODE_GRAPHS=1, decode steps (one new token per sequence over an initialized
// cache) replay a CUDA graph of the whole layer once its inputs are stable: the runners launch
// every layer's few dozen kernels from the host each step (QwenRunner.cpp:349-375).  A layer is
// recorded on the second decode call that sees the same cache storage, weights, shapes and
// workspaces as the call before; any change runs the layer eagerly and records it again later.
// Generate's Clear() keeps the caches' storage, so the graphs survive from one generation to the
// next; InitKVCache() replaces the caches, and every layer is recorded again.
#pragma once

#include <ATen/cuda/CUDAEvent.h>
#include <ATen/cuda/CUDAGraph.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/torch.h>

#include <cstring>
#include <memory>
#include <unordered_map>
#include <vector>

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
            if (!hidden.is_cuda())
            {
                return FromHost(hidden, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps, use_qk_norm,
                                position_ids, kv_cache);
            }
            const b200::TensorParallel& tp = b200::ActiveTensorParallel();
            if (tp.world > 1)
            {
                return HeadSharded(hidden, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps,
                                   use_qk_norm, position_ids, kv_cache, tp);
            }
            if (kv_cache != nullptr && kv_cache->IsInitialized() && hidden.dim() == 3 && hidden.size(1) == 1 &&
                hidden.is_cuda() && position_ids.is_cuda() && b200::DecodeGraphsEnabled() &&
                b200::ActiveDecodeGraph() == nullptr)
            {
                return DecodeGraphed(hidden, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps,
                                     use_qk_norm, position_ids, kv_cache);
            }
            return Layer(hidden, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps, use_qk_norm,
                         position_ids, kv_cache);
        }

    private:
        // A runner whose weights and hidden states live on the host (LlamaRunner): the whole layer
        // runs on the current CUDA device -- weights staged once (b200::StageWeight), the hidden
        // state and positions copied per call, the KV cache kept on the device -- and the output
        // comes back on the host in the hidden state's dtype.
        static torch::Tensor FromHost(
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
            const torch::Device dev = b200::ComputeDevice("TransformerBlock");
            LayerWeights g;
            g.input_layernorm = b200::StageWeight(lw.input_layernorm, dev);
            g.post_attention_layernorm = b200::StageWeight(lw.post_attention_layernorm, dev);
            g.w_q = b200::StageWeight(lw.w_q, dev);
            g.w_k = b200::StageWeight(lw.w_k, dev);
            g.w_v = b200::StageWeight(lw.w_v, dev);
            g.w_o = b200::StageWeight(lw.w_o, dev);
            g.w_q_norm = b200::StageWeight(lw.w_q_norm, dev);
            g.w_k_norm = b200::StageWeight(lw.w_k_norm, dev);
            g.w_gate = b200::StageWeight(lw.w_gate, dev);
            g.w_up = b200::StageWeight(lw.w_up, dev);
            g.w_down = b200::StageWeight(lw.w_down, dev);
            const torch::Tensor h = b200::StageActivation(hidden, dev);
            const torch::Tensor pos = position_ids.to(dev);
            torch::Tensor out = Forward(h, g, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps, use_qk_norm,
                                        pos, kv_cache);
            return out.to(hidden.device(), hidden.scalar_type());
        }

        // Tensor parallel (b200::SetTensorParallel): this rank's KV-head group of the layer, then
        // the sum of the ranks' o_proj partials.  The layer is the reference's step sequence with
        // the head counts of one group and the weight slices of its heads; the partial o_proj
        // output is all-reduced before the residual add (decode graphs included: the collective
        // is recorded with the layer).
        static torch::Tensor HeadSharded(
            const torch::Tensor& hidden,
            const LayerWeights& lw,
            int num_heads,
            int num_kv_heads,
            int head_dim,
            double rope_theta,
            double rms_norm_eps,
            bool use_qk_norm,
            const torch::Tensor& position_ids,
            KVCache* kv_cache,
            const b200::TensorParallel& tp)
        {
            if (num_heads % num_kv_heads != 0)
            {
                throw std::runtime_error("Attention: num_heads must be divisible by num_kv_heads.");
            }
            if (num_kv_heads % tp.world != 0)
            {
                throw std::runtime_error("TensorParallel: the kv heads do not split evenly over the ranks");
            }
            const int n_rep = num_heads / num_kv_heads;
            const int kv_local = num_kv_heads / tp.world;
            const int q_local = kv_local * n_rep;
            const int64_t q0 = (int64_t)tp.rank * q_local * head_dim, q1 = q0 + (int64_t)q_local * head_dim;
            const int64_t k0 = (int64_t)tp.rank * kv_local * head_dim, k1 = k0 + (int64_t)kv_local * head_dim;
            LayerWeights s = lw;
            s.w_q = b200::ShardWeight(lw.w_q, 0, q0, q1);
            s.w_k = b200::ShardWeight(lw.w_k, 0, k0, k1);
            s.w_v = b200::ShardWeight(lw.w_v, 0, k0, k1);
            s.w_o = b200::ShardWeight(lw.w_o, 1, q0, q1);
            torch::Tensor attn_in = RMSNorm::Forward(hidden, lw.input_layernorm, rms_norm_eps);
            torch::Tensor attn_out;
            if (use_qk_norm)
            {
                const auto B = attn_in.size(0);
                const auto S = attn_in.size(1);
                torch::Tensor q, k, v;
                if (!b200::ProjectQKV(attn_in, s.w_q, s.w_k, s.w_v, q_local, kv_local, head_dim, &q, &k, &v))
                {
                    q = Linear::Forward(attn_in, s.w_q).view({B, S, q_local, head_dim}).transpose(1, 2);
                    k = Linear::Forward(attn_in, s.w_k).view({B, S, kv_local, head_dim}).transpose(1, 2);
                    v = Linear::Forward(attn_in, s.w_v).view({B, S, kv_local, head_dim}).transpose(1, 2);
                }
                attn_out = Attention::ForwardProjectedNormed(q, k, v, s.w_o, q_local, kv_local, head_dim, rope_theta,
                                                             position_ids, kv_cache, lw.w_q_norm, lw.w_k_norm,
                                                             rms_norm_eps);
            }
            else
            {
                attn_out = Attention::Forward(attn_in, s.w_q, s.w_k, s.w_v, s.w_o, q_local, kv_local, head_dim,
                                              rope_theta, position_ids, kv_cache);
            }
            attn_out = attn_out.contiguous();
            b200::RequireCudaBf16(attn_out, "TensorParallel");
            b200::Check(mllm_comm_all_reduce_bf16(tp.comm, attn_out.data_ptr(), attn_out.data_ptr(),
                                                  (size_t)attn_out.numel(), b200::CurrentStream()),
                        "TensorParallel (o_proj all-reduce)");
            torch::Tensor h = hidden + attn_out;
            torch::Tensor mlp_in = RMSNorm::Forward(h, lw.post_attention_layernorm, rms_norm_eps);
            return h + MLP::Forward(mlp_in, lw.w_gate, lw.w_up, lw.w_down);
        }

        // The reference's step sequence (TransformerBlock.h:77-195), run kernel by kernel.
        static torch::Tensor Layer(
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

        // One decode layer recorded as a CUDA graph.  `in` and `pos` are the buffers it reads (the
        // caller's tensors are copied in unless they are those buffers, as the previous layer's
        // `out` is), `lens` the cache rows including the new token, `out` what it writes.
        struct DecodeGraph
        {
            std::unique_ptr<at::cuda::CUDAGraph> graph;
            torch::Tensor in, pos, lens, out;
            std::vector<uint64_t> identity;   // everything the recording depends on
        };

        static std::unordered_map<const KVCache*, DecodeGraph>& Graphs()
        {
            // never destroyed: the graphs must not outlive the CUDA context at process exit
            thread_local auto* graphs = new std::unordered_map<const KVCache*, DecodeGraph>();
            return *graphs;
        }

        static std::vector<uint64_t> Identity(const torch::Tensor& hidden, const LayerWeights& lw, int num_heads,
                                              int num_kv_heads, int head_dim, double rope_theta,
                                              double rms_norm_eps, bool use_qk_norm,
                                              const torch::Tensor& position_ids, const KVCache* kv_cache)
        {
            auto ptr = [](const torch::Tensor& t) {
                return t.defined() ? (uint64_t)reinterpret_cast<uintptr_t>(t.data_ptr()) : 0u;
            };
            auto bits = [](double x) {
                uint64_t u;
                std::memcpy(&u, &x, sizeof u);
                return u;
            };
            return {ptr(kv_cache->key_storage), ptr(kv_cache->value_storage), (uint64_t)kv_cache->Capacity(),
                    (uint64_t)hidden.size(0), (uint64_t)hidden.size(2), (uint64_t)hidden.scalar_type(),
                    (uint64_t)hidden.device().index(), (uint64_t)position_ids.numel(),
                    (uint64_t)position_ids.scalar_type(), ptr(lw.input_layernorm), ptr(lw.post_attention_layernorm),
                    ptr(lw.w_q), ptr(lw.w_k), ptr(lw.w_v), ptr(lw.w_o), ptr(lw.w_q_norm), ptr(lw.w_k_norm),
                    ptr(lw.w_gate), ptr(lw.w_up), ptr(lw.w_down), (uint64_t)num_heads, (uint64_t)num_kv_heads,
                    (uint64_t)head_dim, bits(rope_theta), bits(rms_norm_eps), (uint64_t)use_qk_norm,
                    b200::WorkspaceGeneration()};
        }

        static torch::Tensor Replay(DecodeGraph& g, const torch::Tensor& hidden, const torch::Tensor& position_ids,
                                    KVCache* kv_cache, int64_t length)
        {
            if (hidden.data_ptr() != g.in.data_ptr() || hidden.strides() != g.in.strides())
            {
                g.in.copy_(hidden);
            }
            g.pos.copy_(position_ids.reshape(g.pos.sizes()));
            g.lens.fill_(length + 1);
            g.graph->replay();
            kv_cache->SetLength(length + 1);
            return g.out;
        }

        static torch::Tensor DecodeGraphed(const torch::Tensor& hidden, const LayerWeights& lw, int num_heads,
                                           int num_kv_heads, int head_dim, double rope_theta, double rms_norm_eps,
                                           bool use_qk_norm, const torch::Tensor& position_ids, KVCache* kv_cache)
        {
            const int64_t B = hidden.size(0);
            const int64_t length = kv_cache->length;
            // room for the new row now, so that a recorded step never reallocates the cache
            kv_cache->Reserve(B, num_kv_heads, head_dim, length + 1, hidden.options());
            auto id = [&] {
                return Identity(hidden, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps, use_qk_norm,
                                position_ids, kv_cache);
            };
            auto eager = [&] {
                return Layer(hidden, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps, use_qk_norm,
                             position_ids, kv_cache);
            };
            DecodeGraph& g = Graphs()[kv_cache];
            const std::vector<uint64_t> now = id();
            if (g.graph && g.identity == now)
            {
                return Replay(g, hidden, position_ids, kv_cache, length);
            }
            if (g.graph || g.identity != now)
            {
                // new or changed since the last call: run it as is, record it next time if it holds
                g = DecodeGraph{};
                torch::Tensor out = eager();
                g.identity = id();   // after the call: it may have grown a workspace
                return out;
            }

            // The same inputs as the last call: record the layer, then replay it for this step.
            // The workspaces take their recorded sizes first, so that nothing is allocated while
            // recording (a buffer allocated then would belong to the graph's private pool).
            const int64_t cap = kv_cache->Capacity();
            b200::DecodeWorkspace(
                mllm_decode_attention_workspace_size((int)B, num_heads, num_kv_heads, head_dim, (int)cap),
                hidden.device());
            const uint64_t generation = b200::WorkspaceGeneration();
            g.in = hidden;
            g.pos = position_ids.to(torch::kInt64).clone();
            g.lens = torch::full({B}, length + 1, torch::TensorOptions().dtype(torch::kInt32).device(hidden.device()));
            auto graph = std::make_unique<at::cuda::CUDAGraph>();
            const at::cuda::CUDAStream cur = at::cuda::getCurrentCUDAStream();
            const at::cuda::CUDAStream side = at::cuda::getStreamFromPool(false, hidden.device().index());
            at::cuda::CUDAEvent ready;
            ready.record(cur);
            ready.block(side);
            torch::Tensor out;
            {
                c10::cuda::CUDAStreamGuard guard(side);
                b200::DecodeGraphContext ctx{g.lens, cap};
                b200::ActiveDecodeGraph() = &ctx;
                graph->capture_begin();
                try
                {
                    out = Layer(g.in, lw, num_heads, num_kv_heads, head_dim, rope_theta, rms_norm_eps, use_qk_norm,
                                g.pos, kv_cache);
                }
                catch (...)
                {
                    b200::ActiveDecodeGraph() = nullptr;
                    try
                    {
                        graph->capture_end();
                    }
                    catch (...)
                    {
                    }
                    g = DecodeGraph{};
                    throw;
                }
                graph->capture_end();
                b200::ActiveDecodeGraph() = nullptr;
            }
            at::cuda::CUDAEvent done;
            done.record(side);
            done.block(cur);
            if (b200::WorkspaceGeneration() != generation)
            {
                // a workspace was reallocated while recording: the graph may point at freed memory
                g = DecodeGraph{};
                torch::Tensor o = eager();
                g.identity = id();
                return o;
            }
            g.graph = std::move(graph);
            g.out = out;
            g.identity = id();
            return Replay(g, hidden, position_ids, kv_cache, length);
        }
    };
}
