// Host glue shared by the drop-in runtime headers: argument checks in the reference's error
// style, the current CUDA stream, status -> std::runtime_error, and the decode workspace.
// (No counterpart in the reference: this is the bridge from LibTorch tensors to the C ABI.)
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <torch/torch.h>

#include <stdexcept>
#include <string>

#include "mllm_attn.h"

namespace mllm
{
    namespace b200
    {
        inline mllm_stream_t CurrentStream()
        {
            return reinterpret_cast<mllm_stream_t>(at::cuda::getCurrentCUDAStream().stream());
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

        // Grow-only scratch for the split-K decode partials (the C ABI never allocates).
        inline torch::Tensor DecodeWorkspace(size_t bytes, const torch::Device& dev)
        {
            thread_local torch::Tensor ws;
            if (!ws.defined() || (size_t)ws.numel() < bytes || ws.device() != dev)
            {
                ws = torch::empty({(int64_t)std::max<size_t>(bytes, 256)},
                                  torch::TensorOptions().dtype(torch::kUInt8).device(dev));
            }
            return ws;
        }
    }
}
