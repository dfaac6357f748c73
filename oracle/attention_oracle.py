"""CPU restatement of mLLM's attention path, in numpy (fp32 with explicit bf16 rounding).

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg may import this module, and only as the checker.  The product (mllm_b200) never calls it.

Parity is pinned: tests/test_oracle_golden.py checks every function here against golden
vectors produced by the reference's own LibTorch code (oracle/_ref, built from the reference
sources by oracle/build_ref.py; fixtures made by tests/golden/make_golden.py).

Every function cites the reference file:line whose algorithm it restates.  Rounding points
follow the reference exactly: where the reference casts to the input dtype (bf16 on the GPU
path), the restatement rounds to bf16 with round-to-nearest-even at the same step.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

F32 = np.float32


# ----------------------------------------------------------------------------------------
# bf16 helpers (numpy has no bf16: carry bf16 values as fp32 arrays + uint16 bit patterns)
# ----------------------------------------------------------------------------------------

def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern (uint16), round-to-nearest-even (what `.to(kBFloat16)` does)."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=F32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to the nearest bf16 value, returned as fp32."""
    return bf16_to_f32(bf16_bits(x))


def _cast(x: np.ndarray, dtype: str) -> np.ndarray:
    return round_bf16(x) if dtype == "bf16" else np.asarray(x, dtype=F32)


# ----------------------------------------------------------------------------------------
# RoPE  (src/core/runtime/RoPE.h)
# ----------------------------------------------------------------------------------------

def rope_inv_freq(head_dim: int, rope_theta: float) -> np.ndarray:
    """inv_freq = exp(-(idx/D) * ln(theta)), idx = 0,2,..,D-2 (RoPE.h:43-50).  The argument is
    formed in fp32 with the reference's two roundings; exp itself is evaluated correctly
    rounded (float64, then one rounding to fp32).  LibTorch's vectorised fp32 exp is a
    1-ulp approximation of the same value, so the two agree except where it misrounds."""
    idx = np.arange(0, head_dim, 2, dtype=F32)
    log_theta = F32(math.log(rope_theta))
    arg = (-((idx / F32(head_dim)) * log_theta)).astype(F32)
    return np.exp(arg.astype(np.float64)).astype(F32)


def rope_build_cos_sin(positions: np.ndarray, head_dim: int, rope_theta: float):
    """RoPE::BuildCosSin (RoPE.h:29-59): cos/sin [S, D] fp32, table = cat(freqs, freqs)."""
    if head_dim % 2 != 0:
        raise RuntimeError("RoPE: head_dim must be even.")
    inv_freq = rope_inv_freq(head_dim, rope_theta)
    pos = np.asarray(positions).astype(F32)
    freqs = (pos[:, None] * inv_freq[None, :]).astype(F32)      # RoPE.h:54
    emb = np.concatenate([freqs, freqs], axis=-1).astype(np.float64)   # RoPE.h:56
    # cos/sin of the fp32 argument, correctly rounded to fp32 (RoPE.h:58)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def rope_apply(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """RoPE::Apply (RoPE.h:68-89): out = x*cos + cat(-x2, x1)*sin in fp32, three separate
    roundings (mul, mul, add; no fused multiply-add), then cast to the input dtype."""
    x = np.asarray(x, dtype=F32)
    half = x.shape[-1] // 2
    rotated = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    a = (x * cos).astype(F32)
    b = (rotated * sin).astype(F32)
    return _cast((a + b).astype(F32), dtype)


# ----------------------------------------------------------------------------------------
# RMSNorm  (src/core/runtime/RMSNorm.h)  -- the per-head QK-norm use
# ----------------------------------------------------------------------------------------

def libtorch_cpu_row_sum(x: np.ndarray) -> np.ndarray:
    """fp32 sum over the last (contiguous) axis in the summation order of the reference's CPU
    LibTorch reduction (cascade row sum, 8-wide vectors, 4 interleaved vector accumulators):
      P_k[j] = sum_i x[(4i + k)*8 + j]        (sequential in i)
      acc[j] = ((P_0[j] + P_1[j]) + P_2[j]) + P_3[j]
      total  = sum_j acc[j]                    (sequential in j, from 0)
    Valid when the length is a multiple of 32 (head_dim 64 and 128).  This is the order the
    pinned fixtures were produced with (checked bit for bit by the golden tests); other lengths
    fall back to numpy's sum."""
    n = x.shape[-1]
    if n % 32 != 0:
        return np.sum(x, axis=-1, dtype=F32)
    v = x.reshape(x.shape[:-1] + (n // 32, 4, 8))          # [..., i, k, j]
    p = np.zeros(x.shape[:-1] + (4, 8), dtype=F32)
    for i in range(n // 32):
        p = (p + v[..., i, :, :]).astype(F32)
    acc = p[..., 0, :]
    for k in range(1, 4):
        acc = (acc + p[..., k, :]).astype(F32)
    tot = np.zeros(x.shape[:-1], dtype=F32)
    for j in range(8):
        tot = (tot + acc[..., j]).astype(F32)
    return tot


def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, dtype: str = "f32") -> np.ndarray:
    """RMSNorm::Forward (RMSNorm.h:27-64): fp32 mean of squares (the squares of bf16 values are
    exact; the sum follows the reference's reduction order, then / D), plus eps, rsqrt as
    1/sqrt (two roundings, as LibTorch's CPU rsqrt), x * r, then times the weight (a separate
    rounding), cast back to the input dtype."""
    x = np.asarray(x, dtype=F32)
    var = (libtorch_cpu_row_sum((x * x).astype(F32)) / F32(x.shape[-1])).astype(F32)[..., None]
    r = (F32(1.0) / np.sqrt((var + F32(eps)).astype(F32))).astype(F32)
    xn = (x * r).astype(F32)
    return _cast((xn * np.asarray(weight, dtype=F32)).astype(F32), dtype)


# ----------------------------------------------------------------------------------------
# Linear  (src/core/runtime/Linear.h:33-68)
# ----------------------------------------------------------------------------------------

def linear(x: np.ndarray, w: np.ndarray, dtype: str = "f32") -> np.ndarray:
    """y = x @ w.T in the input dtype (fp32 accumulate, one rounding to bf16 for bf16)."""
    return _cast(np.matmul(np.asarray(x, F32), np.asarray(w, F32).T).astype(F32), dtype)


# ----------------------------------------------------------------------------------------
# KVCache  (src/core/runtime/KVCache.h:9-28)
# ----------------------------------------------------------------------------------------

@dataclass
class KVCache:
    key: np.ndarray | None = None     # [B, Hkv, L, D]
    value: np.ndarray | None = None

    def is_initialized(self) -> bool:
        return self.key is not None and self.value is not None

    def clear(self) -> None:
        self.key = None
        self.value = None


# ----------------------------------------------------------------------------------------
# Attention  (src/core/runtime/Attention.h)
# ----------------------------------------------------------------------------------------

def _softmax_lastdim(s: np.ndarray) -> np.ndarray:
    m = np.max(s, axis=-1, keepdims=True)
    e = np.exp((s - m).astype(F32)).astype(F32)
    return (e / np.sum(e, axis=-1, keepdims=True, dtype=F32)).astype(F32)


def attention_core(q: np.ndarray, k_all: np.ndarray, v_all: np.ndarray, num_heads: int,
                   num_kv_heads: int, head_dim: int, dtype: str = "f32") -> np.ndarray:
    """GQA expand + scaled scores + causal mask + softmax + PV + merge heads
    (Attention.h:220-316).  q [B,H,S,D] post-RoPE, k_all/v_all [B,Hkv,total,D] (cache
    contents).  Returns the merged-head attention output [B, S, H*D] before o_proj."""
    if num_heads % num_kv_heads != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    n_rep = num_heads // num_kv_heads
    B, H, S, D = q.shape
    total = k_all.shape[2]
    k = np.repeat(k_all, n_rep, axis=1) if n_rep > 1 else k_all          # Attention.h:220-231
    v = np.repeat(v_all, n_rep, axis=1) if n_rep > 1 else v_all
    scale = F32(1.0 / math.sqrt(float(head_dim)))                         # Attention.h:243-249
    scores = (np.matmul(np.asarray(q, F32), np.swapaxes(np.asarray(k, F32), -1, -2)).astype(F32)
              * scale).astype(F32)                                        # Attention.h:251-255
    # causal: triu(full(-inf), 1 + total - S)  (Attention.h:261-283)
    row = np.arange(S)[:, None]
    col = np.arange(total)[None, :]
    masked = col >= row + 1 + (total - S)
    scores = np.where(masked, F32(-np.inf), scores).astype(F32)
    attn = _cast(_softmax_lastdim(scores), dtype)                         # Attention.h:285-289
    out = _cast(np.matmul(attn, np.asarray(v, F32)).astype(F32), dtype)   # Attention.h:295-299
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3))).reshape(B, S, H * D)  # :309-316


def attention_forward_projected(q, k, v, w_o, num_heads: int, num_kv_heads: int, head_dim: int,
                                rope_theta: float, position_ids, kv_cache: KVCache | None,
                                dtype: str = "f32", rope_table=None) -> np.ndarray:
    """Attention::ForwardProjected (Attention.h:100-326).  q [B,H,S,D], k/v [B,Hkv,S,D].
    `rope_table` (cos, sin) overrides the table built from position_ids (used by tests that
    share one table between the oracle and the device path)."""
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise RuntimeError("Attention::ForwardProjected: q/k/v must be rank-4 tensors.")
    if num_heads % num_kv_heads != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    cos, sin = rope_table if rope_table is not None else rope_build_cos_sin(
        position_ids, head_dim, rope_theta)                               # Attention.h:157-165
    q = rope_apply(q, cos, sin, dtype)                                    # Attention.h:167-171
    k = rope_apply(k, cos, sin, dtype)                                    # Attention.h:173-177
    v = _cast(v, dtype)
    if kv_cache is not None:                                              # Attention.h:183-208
        if kv_cache.is_initialized():
            k = np.concatenate([kv_cache.key, k], axis=2)
            v = np.concatenate([kv_cache.value, v], axis=2)
        kv_cache.key, kv_cache.value = k, v
    out = attention_core(q, k, v, num_heads, num_kv_heads, head_dim, dtype)
    return linear(out, w_o, dtype)                                        # Attention.h:322-325


def attention_forward(hidden, w_q, w_k, w_v, w_o, num_heads: int, num_kv_heads: int, head_dim: int,
                      rope_theta: float, position_ids, kv_cache: KVCache | None,
                      dtype: str = "f32") -> np.ndarray:
    """Attention::Forward (Attention.h:29-86): project, view [B,S,h,D] -> transpose(1,2)."""
    if hidden.ndim != 3:
        raise RuntimeError("Attention: hidden must be [B, S, H].")
    B, S, _ = hidden.shape
    q = linear(hidden, w_q, dtype).reshape(B, S, num_heads, head_dim).transpose(0, 2, 1, 3)
    k = linear(hidden, w_k, dtype).reshape(B, S, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    v = linear(hidden, w_v, dtype).reshape(B, S, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    return attention_forward_projected(q, k, v, w_o, num_heads, num_kv_heads, head_dim,
                                       rope_theta, position_ids, kv_cache, dtype)


def qwen_qkv_prologue(h, w_q, w_k, w_v, w_q_norm, w_k_norm, num_heads: int, num_kv_heads: int,
                      head_dim: int, eps: float, dtype: str = "f32"):
    """The Qwen3 branch of TransformerBlock::Forward before ForwardProjected
    (TransformerBlock.h:82-153): project, reshape to [B,h,S,D], per-head RMSNorm on q and k."""
    B, S, _ = h.shape
    q = linear(h, w_q, dtype).reshape(B, S, num_heads, head_dim).transpose(0, 2, 1, 3)
    q = rms_norm(q, w_q_norm, eps, dtype)                                 # TransformerBlock.h:103-107
    k = linear(h, w_k, dtype).reshape(B, S, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    k = rms_norm(k, w_k_norm, eps, dtype)                                 # TransformerBlock.h:130-134
    v = linear(h, w_v, dtype).reshape(B, S, num_kv_heads, head_dim).transpose(0, 2, 1, 3)
    return q, k, v


# ----------------------------------------------------------------------------------------
# The fused epilogue as one function (what the device epilogue computes, per token)
# ----------------------------------------------------------------------------------------

def qkv_epilogue(q, k, v, cos, sin, q_gamma=None, k_gamma=None, eps: float = 1e-6,
                 dtype: str = "bf16"):
    """Composition of TransformerBlock.h:103-107,130-134 (per-head RMSNorm, Qwen only) and
    Attention.h:157-177 (RoPE) on [B,h,S,D] inputs.  Returns (q_rot, k_rot, v) in `dtype`:
    exactly the values the reference stores in KVCache::key / value (Attention.h:206-207)."""
    if q_gamma is not None:
        q = rms_norm(q, q_gamma, eps, dtype)
    if k_gamma is not None:
        k = rms_norm(k, k_gamma, eps, dtype)
    return rope_apply(q, cos, sin, dtype), rope_apply(k, cos, sin, dtype), _cast(v, dtype)


def decode_attention(q, k_cache, v_cache, seq_lens, num_heads: int, num_kv_heads: int,
                     head_dim: int, dtype: str = "f32"):
    """Single-token attention for each sequence b against its first seq_lens[b] cache rows:
    Attention.h:220-316 at S == 1 (the last query row sees every cached key), generalised to
    per-sequence lengths the way the reference would run it at batch 1 per request.
    q [B,H,D], caches [B,Hkv,Lmax,D].  Returns [B, H*D]."""
    B = q.shape[0]
    outs = []
    for b in range(B):
        L = int(seq_lens[b])
        o = attention_core(q[b:b + 1, :, None, :], k_cache[b:b + 1, :, :L], v_cache[b:b + 1, :, :L],
                           num_heads, num_kv_heads, head_dim, dtype)
        outs.append(o.reshape(-1))
    return np.stack(outs)
