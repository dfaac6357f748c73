"""Random-init Qwen3- and Llama-architecture checkpoints in the HuggingFace layout the mLLM
runners load (config.json + model.safetensors, tensor names of QwenRunner::LoadAllWeights and
LlamaRunner::LoadAllWeights, LlamaRunner.cpp:111-187).  Test helper: the tests and the
end-to-end generation bench write one into a temporary directory on the GPU machine, then load
it with both the reference runner and the drop-in runner."""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class QwenShape:
    layers: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float = 1e6
    eps: float = 1e-6


QWEN3_8B = QwenShape(layers=36, hidden=4096, heads=32, kv_heads=8, head_dim=128, intermediate=12288, vocab=151936)


def _tensor_names(s: QwenShape):
    names = [("model.embed_tokens.weight", (s.vocab, s.hidden)), ("model.norm.weight", (s.hidden,)),
             ("lm_head.weight", (s.vocab, s.hidden))]
    for i in range(s.layers):
        p = f"model.layers.{i}"
        names += [
            (f"{p}.input_layernorm.weight", (s.hidden,)),
            (f"{p}.post_attention_layernorm.weight", (s.hidden,)),
            (f"{p}.self_attn.q_proj.weight", (s.heads * s.head_dim, s.hidden)),
            (f"{p}.self_attn.k_proj.weight", (s.kv_heads * s.head_dim, s.hidden)),
            (f"{p}.self_attn.v_proj.weight", (s.kv_heads * s.head_dim, s.hidden)),
            (f"{p}.self_attn.o_proj.weight", (s.hidden, s.heads * s.head_dim)),
            (f"{p}.self_attn.q_norm.weight", (s.head_dim,)),
            (f"{p}.self_attn.k_norm.weight", (s.head_dim,)),
            (f"{p}.mlp.gate_proj.weight", (s.intermediate, s.hidden)),
            (f"{p}.mlp.up_proj.weight", (s.intermediate, s.hidden)),
            (f"{p}.mlp.down_proj.weight", (s.hidden, s.intermediate)),
        ]
    return names


def _llama_tensor_names(s: QwenShape):
    """LlamaRunner's tensors: the Qwen3 list without the per-head q/k norm weights."""
    return [(n, shape) for n, shape in _tensor_names(s) if not n.endswith(("q_norm.weight", "k_norm.weight"))]


TINYLLAMA_LAYER = QwenShape(layers=2, hidden=2048, heads=32, kv_heads=4, head_dim=64, intermediate=1024, vocab=2048,
                            rope_theta=1e4, eps=1e-5)


def write_random_qwen3(path: str, s: QwenShape, seed: int = 0, device: str = "cuda", dtype: str = "bf16") -> None:
    """Weights N(0, 0.02) (norm weights 1 + N(0, 0.1)), rounded to bf16, generated with torch on
    `device` (a seeded torch generator) and streamed to model.safetensors tensor by tensor.
    dtype="f32" stores the same bf16 values widened exactly to fp32 (a higher-precision run of
    the same model)."""
    _write(path, "qwen3", s, _tensor_names(s), seed, device, dtype)


def write_random_llama(path: str, s: QwenShape, seed: int = 0, device: str = "cuda", dtype: str = "bf16") -> None:
    """The same for the Llama architecture (model_type "llama": no QK-norm; LlamaRunner keeps
    these weights on the host)."""
    _write(path, "llama", s, _llama_tensor_names(s), seed, device, dtype)


def _write(path, model_type, s, names, seed, device, dtype):
    import torch
    os.makedirs(path, exist_ok=True)
    cfg = {"model_type": model_type, "_name_or_path": f"random-{model_type}", "hidden_size": s.hidden,
           "num_hidden_layers": s.layers, "num_attention_heads": s.heads, "num_key_value_heads": s.kv_heads,
           "head_dim": s.head_dim, "intermediate_size": s.intermediate, "vocab_size": s.vocab,
           "max_position_embeddings": 40960, "rms_norm_eps": s.eps, "rope_theta": s.rope_theta,
           "tie_word_embeddings": False, "torch_dtype": "bfloat16"}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    header = {}
    off = 0
    es, st_name = (2, "BF16") if dtype == "bf16" else (4, "F32")
    for n, shape in names:
        nbytes = int(np.prod(shape)) * es
        header[n] = {"dtype": st_name, "shape": list(shape), "data_offsets": [off, off + nbytes]}
        off += nbytes
    header["__metadata__"] = {"format": "pt"}
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    g = torch.Generator(device=device).manual_seed(seed)
    with open(os.path.join(path, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for n, shape in names:
            if n.endswith("norm.weight"):
                t = 1.0 + 0.1 * torch.randn(shape, generator=g, device=device)
            else:
                t = 0.02 * torch.randn(shape, generator=g, device=device)
            t = t.to(torch.bfloat16)
            if dtype == "bf16":
                f.write(t.view(torch.int16).cpu().numpy().tobytes())
            else:
                f.write(t.float().cpu().numpy().tobytes())
