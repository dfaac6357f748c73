"""Shared test helpers: tolerances, bf16 conversion between numpy and torch, and a chunked
torch fp32 reference of the attention core for shapes too large for the numpy oracle."""
from __future__ import annotations

import math

import numpy as np

# tolerance of bf16 outputs against the reference's fp32 result (rtol and atol 2e-2)
RTOL = 2e-2
ATOL = 2e-2


def np_bits_to_torch(bits: np.ndarray, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def torch_to_bits(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f32_to_torch_bf16(x: np.ndarray, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device).to(torch.bfloat16)


def torch_attention_ref(q, k_cache, v_cache, kv_lens, q_rows=None):
    """fp32 reference of Attention.h:220-316 on the GPU with torch (a plain restatement, used
    only where the numpy oracle would take minutes).  q [B,H,S,D] bf16 (the newest S rows of
    each sequence), caches [B,Hkv,cap,D], kv_lens per sequence.  q_rows restricts the query
    rows computed (a slice), to bound memory.  Returns fp32 [B, S', H, D]."""
    import torch
    B, H, S, D = q.shape
    Hkv = k_cache.shape[1]
    n_rep = H // Hkv
    rows = q_rows if q_rows is not None else slice(0, S)
    outs = []
    scale = 1.0 / math.sqrt(D)
    for b in range(B):
        L = int(kv_lens[b])
        k = k_cache[b, :, :L].float().repeat_interleave(n_rep, 0)
        v = v_cache[b, :, :L].float().repeat_interleave(n_rep, 0)
        qb = q[b, :, rows].float()
        s = torch.matmul(qb, k.transpose(-1, -2)) * scale
        r0 = rows.start
        qi = torch.arange(r0, r0 + qb.shape[1], device=q.device)[:, None] + (L - S)
        kj = torch.arange(L, device=q.device)[None, :]
        s = s.masked_fill(kj > qi, float("-inf"))
        p = torch.softmax(s, -1)
        outs.append(torch.matmul(p, v).transpose(0, 1))
    return torch.stack(outs)
