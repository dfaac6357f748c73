// Drop-in replacement for the mLLM reference's src/core/runtime/KVCache.h (KVCache.h:9-28).
//
// Same public members and methods -- `key`, `value`, `IsInitialized()`, `Clear()` -- so the
// unchanged runners keep working: they read `kv_caches_[0].key.size(2)` as the decode position
// (QwenRunner.cpp:301-310, LlamaRunner.cpp:204-232), test IsInitialized() and Clear() the
// caches at the start of Generate.
//
// Storage is different: instead of a tensor re-allocated by torch::cat on every step
// (Attention.h:189-203), the rows live in preallocated bf16 buffers [B, Hkv, capacity, D]
// that grow geometrically; the fused QKV epilogue kernel writes new rows in place and `key` /
// `value` are narrow views of the valid rows [B, Hkv, length, D].
#pragma once

#include <torch/torch.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>

namespace mllm
{
    struct KVCache
    {
        // Valid rows, [batch, num_kv_heads, length, head_dim] (views of the storage below).
        torch::Tensor key;
        torch::Tensor value;

        bool IsInitialized() const
        {
            return key.defined() && value.defined();
        }

        // Forgets the rows; the storage is kept for the next sequence.
        void Clear()
        {
            key = torch::Tensor();
            value = torch::Tensor();
            length = 0;
        }

        // ---- B200 storage (no counterpart in the reference) ----
        torch::Tensor key_storage;    // [B, Hkv, capacity, D] bf16
        torch::Tensor value_storage;
        int64_t length = 0;

        int64_t Capacity() const
        {
            return key_storage.defined() ? key_storage.size(2) : 0;
        }

        // Makes room for `rows` rows of a [B, Hkv, *, D] cache with the given options,
        // preserving the valid rows.  A cache whose key/value were assigned from outside
        // (not views of the storage) is adopted by copying it in.
        void Reserve(int64_t B, int64_t Hkv, int64_t D, int64_t rows, const torch::TensorOptions& opt)
        {
            const bool shape_ok = key_storage.defined() && key_storage.size(0) == B &&
                                  key_storage.size(1) == Hkv && key_storage.size(3) == D &&
                                  key_storage.device() == opt.device();
            const bool adopted = IsInitialized() &&
                                 (!key_storage.defined() || key.data_ptr() != key_storage.data_ptr());
            if (adopted)
            {
                if (key.size(0) != B || key.size(1) != Hkv || key.size(3) != D)
                {
                    throw std::runtime_error("KVCache: cached rows do not match the attention geometry.");
                }
                length = key.size(2);
            }
            else if (!shape_ok)
            {
                if (length != 0)
                {
                    throw std::runtime_error("KVCache: batch or head geometry changed while initialized.");
                }
            }
            if (shape_ok && !adopted && rows <= Capacity())
            {
                return;
            }
            int64_t cap = std::max<int64_t>(rows, shape_ok ? 2 * Capacity() : 0);
            cap = std::max<int64_t>(cap, 256);
            cap = (cap + 255) / 256 * 256;
            auto o = opt.dtype(torch::kBFloat16);
            torch::Tensor ks = torch::empty({B, Hkv, cap, D}, o);
            torch::Tensor vs = torch::empty({B, Hkv, cap, D}, o);
            if (length > 0)
            {
                const torch::Tensor& src_k = adopted ? key : key_storage.narrow(2, 0, length);
                const torch::Tensor& src_v = adopted ? value : value_storage.narrow(2, 0, length);
                ks.narrow(2, 0, length).copy_(src_k);
                vs.narrow(2, 0, length).copy_(src_v);
            }
            key_storage = ks;
            value_storage = vs;
            SetLength(length);
        }

        // Publishes `n` valid rows through `key` / `value`.
        void SetLength(int64_t n)
        {
            length = n;
            if (n > 0)
            {
                key = key_storage.narrow(2, 0, n);
                value = value_storage.narrow(2, 0, n);
            }
            else
            {
                key = torch::Tensor();
                value = torch::Tensor();
            }
        }
    };
}
