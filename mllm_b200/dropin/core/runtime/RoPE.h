// Drop-in replacement for the mLLM reference's src/core/runtime/RoPE.h.
//
// Same class and signatures (RoPE::BuildCosSin, RoPE.h:29-59; RoPE::Apply, RoPE.h:68-89) and
// the same fp32 step order (NeoX rotate-half, cos/sin duplicated over both halves), computed by
// the B200 kernels through the C ABI.  Inside the attention path RoPE is fused into the QKV
// epilogue; these entry points serve callers that use RoPE on its own.
#pragma once

#include <torch/torch.h>

#include <stdexcept>
#include <utility>

#include "core/runtime/B200Device.h"

namespace mllm
{
    class RoPE
    {
    public:
        // positions: [S] integer tensor on a CUDA device.  Returns (cos, sin), fp32 [S, D].
        static std::pair<torch::Tensor, torch::Tensor> BuildCosSin(
            const torch::Tensor& positions,
            int head_dim,
            double rope_theta)
        {
            if (head_dim % 2 != 0)
            {
                throw std::runtime_error("RoPE: head_dim must be even.");
            }
            if (!positions.is_cuda())
            {
                throw std::runtime_error("RoPE: the B200 path needs CUDA positions.");
            }
            auto pos = positions.to(torch::kInt64).contiguous();
            auto fopts = torch::TensorOptions().dtype(torch::kFloat32).device(pos.device());
            auto cos = torch::empty({pos.numel(), head_dim}, fopts);
            auto sin = torch::empty({pos.numel(), head_dim}, fopts);
            b200::Check(mllm_rope_build_cos_sin(pos.data_ptr<int64_t>(), pos.numel(), head_dim, rope_theta,
                                                cos.data_ptr<float>(), sin.data_ptr<float>(),
                                                b200::CurrentStream()),
                        "RoPE::BuildCosSin");
            return { cos, sin };
        }

        // x: [B, H, S, D] bf16 on CUDA (any strides, D contiguous); cos/sin: [S, D] fp32.
        static torch::Tensor Apply(
            const torch::Tensor& x,
            const torch::Tensor& cos,
            const torch::Tensor& sin)
        {
            b200::RequireCudaBf16(x, "RoPE::Apply");
            if (x.dim() != 4)
            {
                throw std::runtime_error("RoPE::Apply: x must be [B, H, S, D].");
            }
            auto c = cos.to(torch::kFloat32).contiguous();
            auto s = sin.to(torch::kFloat32).contiguous();
            if (c.size(0) != x.size(2) || c.size(1) != x.size(3))
            {
                throw std::runtime_error("RoPE::Apply: cos/sin must be [S, D].");
            }
            auto out = torch::empty(x.sizes(), x.options().memory_format(torch::MemoryFormat::Contiguous));
            b200::Check(mllm_rope_apply_bf16(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2), (int)x.size(0),
                                             (int)x.size(1), (int)x.size(2), (int)x.size(3), c.data_ptr<float>(),
                                             s.data_ptr<float>(), out.data_ptr(), b200::CurrentStream()),
                        "RoPE::Apply");
            return out;
        }
    };
}
