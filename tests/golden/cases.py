"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Inputs are regenerated from (seed, shape) with numpy's PCG64 generator, which is stable across
platforms, so the committed fixtures only hold the reference's outputs.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle.attention_oracle import round_bf16  # noqa: E402

GOLDEN_DIR = os.path.dirname(os.path.abspath(__file__))


@dataclass(frozen=True)
class Case:
    name: str
    batch: int
    seq: int              # prefill length
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float
    qk_norm: bool
    decode_steps: int
    seed: int
    eps: float = 1e-6


# Small shapes the CPU reference finishes in well under a second.  They cover the reference's
# edge cases: GQA groups 1/2/4/5/8, head_dim 64 and 128, odd lengths, a one-token prefill,
# decode steps that grow the cache through the reference's torch::cat path.
CASES = [
    Case("llama_d64_gqa2", 1, 16, 128, 4, 2, 64, 1e4, False, 3, 11),
    Case("llama_d64_gqa8_odd", 2, 37, 256, 16, 2, 64, 1e4, False, 2, 12),
    Case("qwen_d128_gqa4", 2, 12, 256, 8, 2, 128, 1e6, True, 3, 13),
    Case("qwen_d128_gqa5_odd", 1, 29, 320, 10, 2, 128, 1e6, True, 2, 14),
    Case("qwen_d128_mha_one_token", 3, 1, 128, 2, 2, 128, 1e6, True, 2, 15),
]


def case_by_name(name: str) -> Case:
    for c in CASES:
        if c.name == name:
            return c
    raise KeyError(name)


def make_inputs(c: Case, bf16: bool = False) -> dict:
    """hidden states N(0,1) for the prefill and each decode step, weights N(0, 0.02),
    QK-norm gammas 1 + N(0, 0.1) -- the distributions the workloads use.  With bf16=True every
    tensor is rounded to bf16 values (still carried as fp32)."""
    rng = np.random.default_rng(c.seed)
    H, Hkv, D, E = c.num_heads, c.num_kv_heads, c.head_dim, c.hidden
    f = (lambda a: round_bf16(a.astype(np.float32))) if bf16 else (lambda a: a.astype(np.float32))
    d = {
        "hidden": f(rng.standard_normal((c.batch, c.seq, E))),
        "w_q": f(rng.standard_normal((H * D, E)) * 0.02),
        "w_k": f(rng.standard_normal((Hkv * D, E)) * 0.02),
        "w_v": f(rng.standard_normal((Hkv * D, E)) * 0.02),
        "w_o": f(rng.standard_normal((E, H * D)) * 0.02),
        "decode_hidden": f(rng.standard_normal((c.decode_steps, c.batch, 1, E))),
    }
    if c.qk_norm:
        d["w_q_norm"] = f(1.0 + rng.standard_normal(D) * 0.1)
        d["w_k_norm"] = f(1.0 + rng.standard_normal(D) * 0.1)
    return d


# RoPE table rows pinned against the reference (positions up to the longest workload context).
ROPE_TABLE_CASES = [(64, 1e4), (128, 1e4), (128, 1e6)]
ROPE_POSITIONS = np.concatenate([np.arange(0, 96), np.array([255, 511, 1023, 2047, 2048, 4095,
                                                              4096, 8191, 8192, 16383, 32767, 32768]),
                                 np.random.default_rng(7).integers(0, 32769, size=64)]).astype(np.int64)


# ---------------------------------------------------------------------------------------
# Sampler (Sampler.cpp): logit rows with repeated maxima, negative and positive values, and
# histories with repeats and out-of-range ids.
# ---------------------------------------------------------------------------------------
SAMPLER_VOCAB = 1000
SAMPLER_PENALTIES = (1.0, 1.3, 2.0)


def make_sampler_inputs(seed: int = 21):
    """(logits [4, V] fp32 values that are exact bf16, histories: list of 4 int lists)."""
    rng = np.random.default_rng(seed)
    V = SAMPLER_VOCAB
    logits = (rng.standard_normal((4, V)) * 3).astype(np.float32)
    logits[1, 17] = logits[1, 900] = logits[1].max() + 1.0     # tie at the top: first index wins
    logits[2, :] = -np.abs(logits[2, :])                        # all negative
    logits = round_bf16(np.clip(logits, -60, 60).astype(np.float32))   # exact bf16 values
    hist = [
        [int(x) for x in rng.integers(0, V, 40)],
        [17, 17, 17, 900, -1, V + 5, 3],
        [int(x) for x in np.argsort(logits[2])[-8:]] * 2,       # the largest (closest to 0) twice
        [int(x) for x in rng.integers(0, V, 300)],
    ]
    return logits, hist
