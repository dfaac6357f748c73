"""Generate the golden fixtures in tests/golden/ by running the mLLM reference's own code.

The reference runtime (src/core/runtime/*.h) is compiled from the reference tree by
oracle/build_ref.py into oracle/_ref/.  This script runs it on the seeded inputs of
tests/golden/cases.py and saves its outputs.  It needs the reference tree, so it only runs in
the build container; the fixtures it writes are committed and travel with the tests.

  python tests/golden/make_golden.py

For each case the reference path is exactly what the runners execute per layer:
  * Llama (use_qk_norm=false): Attention::Forward (Attention.h:29-86) with a KVCache,
    prefill at positions arange(S), then decode steps at position key.size(2)
    (LlamaRunner.cpp:204-232).
  * Qwen3 (use_qk_norm=true): the TransformerBlock.h:82-153 prologue (Linear, view/transpose,
    per-head RMSNorm) composed from the reference's Linear/RMSNorm, then
    Attention::ForwardProjected (Attention.h:100-326) with the same position rule
    (QwenRunner.cpp:301-324).
Both run once in fp32 (the CPU reference path) and once in bf16 (the dtype of the device
path; its KV cache is the bit-exact target).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import build_ref  # noqa: E402
from tests.golden.cases import (CASES, ROPE_POSITIONS, ROPE_TABLE_CASES, SAMPLER_PENALTIES,  # noqa: E402
                                make_inputs, make_sampler_inputs)


def load_ref():
    path = build_ref.build()
    if path is None:
        raise SystemExit("reference tree not available; cannot regenerate fixtures")
    sys.path.insert(0, os.path.dirname(path))
    import mllm_ref  # noqa: E402
    return mllm_ref


def bits(t):
    import torch
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def run_case(R, c, dtype_name: str) -> dict:
    import torch
    dt = torch.float32 if dtype_name == "f32" else torch.bfloat16
    inp = make_inputs(c, bf16=(dtype_name == "bf16"))
    T = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dt) for k, v in inp.items()}
    H, Hkv, D = c.num_heads, c.num_kv_heads, c.head_dim
    out = {}
    key = value = None
    steps = [("prefill", T["hidden"])] + [(f"decode{i}", T["decode_hidden"][i])
                                          for i in range(c.decode_steps)]
    for tag, hid in steps:
        S = hid.shape[1]
        if key is not None and S == 1:
            pos = torch.tensor([key.shape[2]], dtype=torch.int64)
        else:
            pos = torch.arange(0, S, dtype=torch.int64)
        if not c.qk_norm:
            if dtype_name == "bf16":
                B = hid.shape[0]
                out[f"{tag}_q_proj_bits"] = bits(R.linear(hid, T["w_q"]).view(B, S, H, D).transpose(1, 2))
                out[f"{tag}_k_proj_bits"] = bits(R.linear(hid, T["w_k"]).view(B, S, Hkv, D).transpose(1, 2))
                out[f"{tag}_v_bits"] = bits(R.linear(hid, T["w_v"]).view(B, S, Hkv, D).transpose(1, 2))
            o, key, value = R.attention_forward(hid, T["w_q"], T["w_k"], T["w_v"], T["w_o"], H, Hkv,
                                                D, c.rope_theta, pos, key, value, True)
        else:
            B = hid.shape[0]
            q = R.linear(hid, T["w_q"]).view(B, S, H, D).transpose(1, 2)
            if dtype_name == "bf16":
                out[f"{tag}_q_proj_bits"] = bits(q)
            q = R.rms_norm(q, T["w_q_norm"], c.eps)
            k = R.linear(hid, T["w_k"]).view(B, S, Hkv, D).transpose(1, 2)
            if dtype_name == "bf16":
                out[f"{tag}_k_proj_bits"] = bits(k)
            k = R.rms_norm(k, T["w_k_norm"], c.eps)
            v = R.linear(hid, T["w_v"]).view(B, S, Hkv, D).transpose(1, 2)
            if dtype_name == "bf16":
                out[f"{tag}_q_normed_bits"] = bits(q)
                out[f"{tag}_k_normed_bits"] = bits(k)
                out[f"{tag}_v_bits"] = bits(v)
            o, key, value = R.attention_forward_projected(q, k, v, T["w_o"], H, Hkv, D, c.rope_theta,
                                                          pos, key, value, True)
        cos, sin = R.rope_build_cos_sin(pos, D, c.rope_theta)
        out[f"{tag}_rope_cos"] = cos.numpy()
        out[f"{tag}_rope_sin"] = sin.numpy()
        out[f"{tag}_pos"] = pos.numpy()
        if dtype_name == "f32":
            out[f"{tag}_out"] = o.numpy()
        else:
            out[f"{tag}_out_bits"] = bits(o)
            out[f"{tag}_key_bits"] = bits(key)
            out[f"{tag}_value_bits"] = bits(value)
    if dtype_name == "f32":
        out["key"] = key.numpy()
        out["value"] = value.numpy()
    return out


def main() -> None:
    import torch
    R = load_ref()
    torch.manual_seed(0)
    for c in CASES:
        for dn in ("f32", "bf16"):
            res = run_case(R, c, dn)
            path = os.path.join(HERE, f"{c.name}_{dn}.npz")
            np.savez_compressed(path, **res)
            print(f"wrote {path} ({os.path.getsize(path)} B)")
    rope = {}
    pos = torch.from_numpy(ROPE_POSITIONS)
    for D, theta in ROPE_TABLE_CASES:
        cos, sin = R.rope_build_cos_sin(pos, D, theta)
        rope[f"cos_d{D}_t{int(theta)}"] = cos[:, : D // 2].numpy()
        rope[f"sin_d{D}_t{int(theta)}"] = sin[:, : D // 2].numpy()
    rope["positions"] = ROPE_POSITIONS
    path = os.path.join(HERE, "rope_tables.npz")
    np.savez_compressed(path, **rope)
    print(f"wrote {path} ({os.path.getsize(path)} B)")
    # Sampler::Sample, greedy branch with the repetition penalty, in bf16 and fp32
    logits, hist = make_sampler_inputs()
    samp = {"logits": logits}
    for dn, dt in (("bf16", torch.bfloat16), ("f32", torch.float32)):
        for pen in SAMPLER_PENALTIES:
            for r in range(logits.shape[0]):
                tok, x = R.sample(torch.from_numpy(logits[r]).to(dt), 1.0, 0, 1.0, True, hist[r], pen)
                tag = f"{dn}_p{int(pen * 10)}_r{r}"
                samp["token_" + tag] = np.array(tok)
                samp["logits_" + tag] = x.float().numpy()
    path = os.path.join(HERE, "sampler.npz")
    np.savez_compressed(path, **samp)
    print(f"wrote {path} ({os.path.getsize(path)} B)")


if __name__ == "__main__":
    main()
