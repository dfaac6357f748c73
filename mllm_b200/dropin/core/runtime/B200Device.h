// Host glue shared by the drop-in runtime headers: argument checks in the reference's error
// style, the current CUDA stream, status -> std::runtime_error, and the decode workspace.
// (No counterpart in the reference: this is the bridge from LibTorch tensors to the C ABI.)
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <torch/torch.h>

#include <c10/cuda/CUDAFunctions.h>

#include <cstdint>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <functional>
#include <unordered_map>

#include "mllm_attn.h"

namespace mllm
{
    namespace b200
    {
        inline mllm_stream_t CurrentStream()
        {
            return reinterpret_cast<mllm_stream_t>(at::cuda::getCurrentCUDAStream().stream());
        }

        // Bumped whenever a shared workspace below is reallocated: a CUDA graph recorded with the
        // old buffer must not be replayed after that.
        inline uint64_t& WorkspaceGeneration()
        {
            thread_local uint64_t generation = 0;
            return generation;
        }

        // Set while a decode layer is recorded as a CUDA graph: the decode step then reads each
        // sequence's length (including the new token) from `lens` on the device, sizes its plan
        // for `plan_len` rows, and leaves the host-side cache length to the recorder.
        struct DecodeGraphContext
        {
            torch::Tensor lens;   // int32 [B]
            int64_t plan_len;
        };

        inline DecodeGraphContext*& ActiveDecodeGraph()
        {
            thread_local DecodeGraphContext* ctx = nullptr;
            return ctx;
        }

        // Decode layers replay CUDA graphs when MLLM_B200_DECODE_GRAPHS=1 (read at every call).
        inline bool DecodeGraphsEnabled()
        {
            const char* v = std::getenv("MLLM_B200_DECODE_GRAPHS");
            return v != nullptr && v[0] == '1' && v[1] == '\0';
        }

        // ---- Host tensors ----
        // A runner may keep its weights and activations on the host: the reference's LlamaRunner
        // never moves them to CUDA (LlamaRunner.cpp:111-187, 189-281).  The drop-in then stages
        // them on the current CUDA device -- each weight once, the activations per call -- runs
        // the layer there, and hands the result back on the host.  The work itself never runs on
        // the CPU.

        // The current CUDA device; there is no CPU path to fall back to.
        inline torch::Device ComputeDevice(const char* who)
        {
            if (!torch::cuda::is_available())
            {
                throw std::runtime_error(std::string(who) + ": the B200 attention path needs a CUDA device.");
            }
            return torch::Device(torch::kCUDA, c10::cuda::current_device());
        }

        // Device copy (bf16, contiguous) of a host weight, made on first use and kept while the
        // weight lives unchanged.  The cache holds a reference to the host tensor, so its address
        // cannot be reused by another tensor while it is cached, and re-stages the weight when its
        // version counter has moved (an in-place write since).  CUDA tensors pass through.
        inline torch::Tensor StageWeight(const torch::Tensor& w, const torch::Device& dev)
        {
            if (!w.defined() || w.is_cuda())
            {
                return w;
            }
            struct Entry
            {
                torch::Tensor host;
                int64_t version;
                torch::Tensor device;
            };
            thread_local std::unordered_map<const void*, Entry> cache;
            const void* key = w.unsafeGetTensorImpl();
            auto it = cache.find(key);
            if (it != cache.end() && it->second.version == (int64_t)w._version() && it->second.device.device() == dev)
            {
                return it->second.device;
            }
            torch::Tensor d = w.to(dev, torch::kBFloat16).contiguous();
            cache[key] = Entry{w, (int64_t)w._version(), d};
            return d;
        }

        // An activation on the compute device in bf16 (a copy when it lives on the host).
        inline torch::Tensor StageActivation(const torch::Tensor& x, const torch::Device& dev)
        {
            if (!x.defined() || (x.is_cuda() && x.scalar_type() == torch::kBFloat16))
            {
                return x;
            }
            return x.to(dev, torch::kBFloat16);
        }

        // ---- Tensor parallelism (no counterpart in the reference, which runs on one device) ----
        // With a communicator set, TransformerBlock::Forward runs only this rank's KV-head group:
        // kv heads [rank*Hkv/world, (rank+1)*Hkv/world) and their query heads, with the row slices
        // of w_q/w_k/w_v and the column slice of w_o (cut once per weight and cached), a KV cache
        // that holds those kv heads only, and the o_proj partial summed over the ranks by
        // mllm_comm_all_reduce_bf16 on the current stream.  Every rank runs the same runner on the
        // same inputs (one process per GPU); norms, MLP, embeddings and lm_head are replicated.
        // The caller owns the communicator (mllm_comm_init) and clears the setting before it
        // destroys it.
        struct TensorParallel
        {
            mllm_comm_t comm = nullptr;
            int rank = 0;
            int world = 1;
        };

        inline TensorParallel& ActiveTensorParallel()
        {
            static TensorParallel tp;
            return tp;
        }

        // world == 1 (or comm == nullptr) turns tensor parallelism off.
        inline void SetTensorParallel(mllm_comm_t comm, int rank, int world)
        {
            if (world < 1 || rank < 0 || rank >= world || (world > 1 && comm == nullptr))
            {
                throw std::runtime_error("TensorParallel: bad rank / world / communicator");
            }
            ActiveTensorParallel() = world > 1 ? TensorParallel{comm, rank, world} : TensorParallel{};
        }

        // Rows [r0, r1) (dim 0) or columns (dim 1) of a weight, contiguous, cut once and cached
        // (the cache holds the source, so its address stays unique while cached).
        inline torch::Tensor ShardWeight(const torch::Tensor& w, int dim, int64_t r0, int64_t r1)
        {
            if (!w.defined())
            {
                return w;
            }
            struct Key
            {
                const void* impl;
                int dim;
                int64_t r0, r1;
                bool operator==(const Key& o) const { return impl == o.impl && dim == o.dim && r0 == o.r0 && r1 == o.r1; }
            };
            struct KeyHash
            {
                size_t operator()(const Key& k) const
                {
                    return std::hash<const void*>()(k.impl) ^ (std::hash<int64_t>()(k.r0 * 31 + k.r1) << 1) ^ k.dim;
                }
            };
            struct Entry
            {
                torch::Tensor source;
                int64_t version;
                torch::Tensor shard;
            };
            thread_local std::unordered_map<Key, Entry, KeyHash> cache;
            const Key key{w.unsafeGetTensorImpl(), dim, r0, r1};
            auto it = cache.find(key);
            if (it != cache.end() && it->second.version == (int64_t)w._version())
            {
                return it->second.shard;
            }
            torch::Tensor s = w.narrow(dim, r0, r1 - r0).contiguous();
            cache[key] = Entry{w, (int64_t)w._version(), s};
            return s;
        }

        // Converts a nonzero mllm_status into std::runtime_error, the reference's convention.
        inline void Check(int status, const char* what)
        {
            if (status != MLLM_OK)
            {
                throw std::runtime_error(std::string(what) + ": " + mllm_attn_status_string(status) +
                                         " (" + mllm_attn_last_error() + ")");
            }
        }

        // The B200 path has no CPU fallback: CUDA bf16 tensors with a contiguous last dim.
        inline void RequireCudaBf16(const torch::Tensor& t, const char* who)
        {
            if (!t.defined() || !t.is_cuda())
            {
                throw std::runtime_error(std::string(who) + ": the B200 attention path needs CUDA tensors.");
            }
            if (t.scalar_type() != torch::kBFloat16)
            {
                throw std::runtime_error(std::string(who) + ": the B200 attention path computes in bfloat16.");
            }
            if (t.stride(-1) != 1)
            {
                throw std::runtime_error(std::string(who) + ": head_dim must be the contiguous dimension.");
            }
        }

        // Grow-only, zero-filled scratch for mllm_linear_bf16's split partials and tile counters
        // (every call leaves the counters at zero, so the buffer is reused as is).
        inline torch::Tensor LinearWorkspace(size_t bytes, const torch::Device& dev)
        {
            thread_local torch::Tensor ws;
            if (!ws.defined() || (size_t)ws.numel() < bytes || ws.device() != dev)
            {
                ws = torch::zeros({(int64_t)std::max<size_t>(bytes, (size_t)1 << 20)},
                                  torch::TensorOptions().dtype(torch::kUInt8).device(dev));
                ++WorkspaceGeneration();
            }
            return ws;
        }

        // The attention step's q/k/v projections (Linear.h:33-68, three F::linear calls in
        // TransformerBlock.h:82-96 / Attention.h:52-54) as ONE mllm_linear_bf16 launch when the
        // shapes allow it (bf16 CUDA, at most 256 tokens, hidden a multiple of 64, projection rows
        // multiples of 128): q|k|v side by side in one [B, S, (H + 2 Hkv) D] tensor, returned as
        // the same [B, h, S, D] views the three GEMMs would give.  Returns false (and touches
        // nothing) when the shapes do not fit; the caller then runs the three GEMMs.
        inline bool ProjectQKV(const torch::Tensor& x, const torch::Tensor& w_q, const torch::Tensor& w_k,
                               const torch::Tensor& w_v, int64_t num_heads, int64_t num_kv_heads,
                               int64_t head_dim, torch::Tensor* q, torch::Tensor* k, torch::Tensor* v)
        {
            if (x.dim() != 3 || !x.is_cuda() || x.scalar_type() != torch::kBFloat16)
                return false;
            const int64_t B = x.size(0), S = x.size(1), K = x.size(2);
            if (B * S > 256 || B * S == 0 || K % 64 != 0)
                return false;
            const torch::Tensor* ws_[3] = {&w_q, &w_k, &w_v};
            for (const torch::Tensor* w : ws_)
            {
                if (!w->defined() || !w->is_cuda() || w->scalar_type() != torch::kBFloat16 || w->dim() != 2 ||
                    w->size(1) != K || w->stride(1) != 1 || w->size(0) % 128 != 0 || w->stride(0) % 8 != 0 ||
                    reinterpret_cast<uintptr_t>(w->data_ptr()) % 16 != 0)
                    return false;
            }
            const int64_t hq = num_heads * head_dim, hk = num_kv_heads * head_dim;
            if (w_q.size(0) != hq || w_k.size(0) != hk || w_v.size(0) != hk)
                return false;
            torch::Tensor x2 = x.reshape({B * S, K});
            if (x2.stride(1) != 1 || x2.stride(0) % 8 != 0 || reinterpret_cast<uintptr_t>(x2.data_ptr()) % 16 != 0)
                x2 = x2.contiguous();
            auto qkv = torch::empty({B * S, hq + 2 * hk}, x.options());
            const void* wp[3] = {w_q.data_ptr(), w_k.data_ptr(), w_v.data_ptr()};
            const int64_t wst[3] = {w_q.stride(0), w_k.stride(0), w_v.stride(0)};
            const int64_t nf[3] = {hq, hk, hk};
            const size_t bytes = mllm_linear_workspace_size((int)(B * S), 3, nf, K);
            torch::Tensor ws;
            if (bytes > 0)
                ws = LinearWorkspace(bytes, x.device());
            Check(mllm_linear_bf16(x2.data_ptr(), x2.stride(0), (int)(B * S), K, 3, wp, wst, nf, qkv.data_ptr(),
                                   qkv.stride(0), bytes > 0 ? ws.data_ptr() : nullptr,
                                   bytes > 0 ? (size_t)ws.numel() : 0, CurrentStream()),
                  "Linear");
            auto q3 = qkv.view({B, S, hq + 2 * hk});
            *q = q3.narrow(2, 0, hq).view({B, S, num_heads, head_dim}).transpose(1, 2);
            *k = q3.narrow(2, hq, hk).view({B, S, num_kv_heads, head_dim}).transpose(1, 2);
            *v = q3.narrow(2, hq + hk, hk).view({B, S, num_kv_heads, head_dim}).transpose(1, 2);
            return true;
        }

        // Grow-only, zero-filled scratch for the split-K decode partials (the C ABI never
        // allocates); its 256-byte header starts at zero and every call leaves it zero.
        inline torch::Tensor DecodeWorkspace(size_t bytes, const torch::Device& dev)
        {
            thread_local torch::Tensor ws;
            if (!ws.defined() || (size_t)ws.numel() < bytes || ws.device() != dev)
            {
                ws = torch::zeros({(int64_t)std::max<size_t>(bytes, 256)},
                                  torch::TensorOptions().dtype(torch::kUInt8).device(dev));
                ++WorkspaceGeneration();
            }
            return ws;
        }

        // Grow-only scratch for the device sampler (token counts, sort buffers). Kept apart from
        // the decode workspace so that nothing the sampler leaves behind can reach the decode
        // work-item counter.
        inline torch::Tensor SamplerWorkspace(size_t bytes, const torch::Device& dev)
        {
            thread_local torch::Tensor ws;
            if (!ws.defined() || (size_t)ws.numel() < bytes || ws.device() != dev)
            {
                ws = torch::zeros({(int64_t)std::max<size_t>(bytes, 256)},
                                  torch::TensorOptions().dtype(torch::kUInt8).device(dev));
            }
            return ws;
        }
    }
}
