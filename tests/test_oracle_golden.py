"""Pins the numpy oracle against the reference's own outputs (golden fixtures made by
tests/golden/make_golden.py from the compiled reference runtime).  CPU only."""
import os

import numpy as np
import pytest

from oracle import attention_oracle as O
from tests.golden.cases import CASES, GOLDEN_DIR, ROPE_POSITIONS, ROPE_TABLE_CASES, make_inputs


def load(name):
    return np.load(os.path.join(GOLDEN_DIR, name))


def run_oracle(c, dtype, g=None, share_tables=False):
    """The oracle's full per-layer attention for a case: prefill then decode steps, with the
    runners' position rule (LlamaRunner.cpp:204-232 / QwenRunner.cpp:301-324)."""
    inp = make_inputs(c, bf16=(dtype == "bf16"))
    H, Hkv, D = c.num_heads, c.num_kv_heads, c.head_dim
    cache = O.KVCache()
    outs = {}
    steps = [("prefill", inp["hidden"])] + [(f"decode{i}", inp["decode_hidden"][i])
                                            for i in range(c.decode_steps)]
    for tag, hid in steps:
        S = hid.shape[1]
        pos = (np.array([cache.key.shape[2]]) if (cache.is_initialized() and S == 1)
               else np.arange(S))
        table = (g[f"{tag}_rope_cos"], g[f"{tag}_rope_sin"]) if share_tables else None
        if not c.qk_norm:
            B = hid.shape[0]
            q = O.linear(hid, inp["w_q"], dtype).reshape(B, S, H, D).transpose(0, 2, 1, 3)
            k = O.linear(hid, inp["w_k"], dtype).reshape(B, S, Hkv, D).transpose(0, 2, 1, 3)
            v = O.linear(hid, inp["w_v"], dtype).reshape(B, S, Hkv, D).transpose(0, 2, 1, 3)
        else:
            q, k, v = O.qwen_qkv_prologue(hid, inp["w_q"], inp["w_k"], inp["w_v"], inp["w_q_norm"],
                                          inp["w_k_norm"], H, Hkv, D, c.eps, dtype)
        outs[tag] = O.attention_forward_projected(q, k, v, inp["w_o"], H, Hkv, D, c.rope_theta, pos,
                                                  cache, dtype, rope_table=table)
        outs[tag + "_pos"] = pos
    return outs, cache


@pytest.mark.parametrize("c", CASES, ids=lambda c: c.name)
def test_oracle_fp32_matches_reference(c):
    g = load(f"{c.name}_f32.npz")
    outs, cache = run_oracle(c, "f32")
    for tag in ["prefill"] + [f"decode{i}" for i in range(c.decode_steps)]:
        np.testing.assert_array_equal(outs[tag + "_pos"], g[tag + "_pos"])
        np.testing.assert_allclose(outs[tag], g[tag + "_out"], rtol=1e-4, atol=2e-6, err_msg=tag)
    # the fp32 projections differ from MKL's only in summation order
    np.testing.assert_allclose(cache.key, g["key"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(cache.value, g["value"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("c", CASES, ids=lambda c: c.name)
def test_oracle_bf16_matches_reference(c):
    """bf16 pipeline: the attention output within bf16 noise, the cache within one bf16 ulp
    (projections and norms differ in fp32 summation order from the reference's CPU kernels)."""
    g = load(f"{c.name}_bf16.npz")
    outs, cache = run_oracle(c, "bf16", g, share_tables=True)
    last = f"decode{c.decode_steps - 1}"
    for tag in ["prefill"] + [f"decode{i}" for i in range(c.decode_steps)]:
        ref = O.bf16_to_f32(g[tag + "_out_bits"])
        np.testing.assert_allclose(outs[tag], ref, rtol=2e-2, atol=2e-3, err_msg=tag)
    for name, ours in (("key", cache.key), ("value", cache.value)):
        ref = O.bf16_to_f32(g[f"{last}_{name}_bits"])
        np.testing.assert_allclose(ours, ref, rtol=1.6e-2, atol=1e-3)


def _steps(c):
    return ["prefill"] + [f"decode{i}" for i in range(c.decode_steps)]


@pytest.mark.parametrize("c", CASES, ids=lambda c: c.name)
def test_epilogue_bit_exact_given_reference_inputs(c):
    """Given the reference's own bf16 projections and its RoPE table, the oracle's fused
    epilogue (per-head RMSNorm for Qwen3, RoPE, append) reproduces the reference KV cache bit
    for bit at every step (TransformerBlock.h:103-134, Attention.h:157-208)."""
    g = load(f"{c.name}_bf16.npz")
    start = 0
    for tag in _steps(c):
        cos, sin = g[f"{tag}_rope_cos"], g[f"{tag}_rope_sin"]
        q = O.bf16_to_f32(g[f"{tag}_q_proj_bits"])
        k = O.bf16_to_f32(g[f"{tag}_k_proj_bits"])
        v = O.bf16_to_f32(g[f"{tag}_v_bits"])
        gq = g_k = None
        if c.qk_norm:
            inp = make_inputs(c, bf16=True)
            gq, g_k = inp["w_q_norm"], inp["w_k_norm"]
        q_rot, k_rot, v_out = O.qkv_epilogue(q, k, v, cos, sin, gq, g_k, c.eps, "bf16")
        S = k.shape[2]
        np.testing.assert_array_equal(O.bf16_bits(k_rot), g[f"{tag}_key_bits"][:, :, start:start + S])
        np.testing.assert_array_equal(O.bf16_bits(v_out), g[f"{tag}_value_bits"][:, :, start:start + S])
        if c.qk_norm:
            np.testing.assert_array_equal(O.bf16_bits(O.rms_norm(q, gq, c.eps, "bf16")),
                                          g[f"{tag}_q_normed_bits"])
        start += S


@pytest.mark.parametrize("c", [c for c in CASES if c.qk_norm], ids=lambda c: c.name)
def test_rms_norm_bit_exact(c):
    """Per-head QK RMSNorm (RMSNorm.h:27-64) on the reference's bf16 projections: the oracle
    follows the reference's fp32 summation order, so the bf16 results are identical."""
    g = load(f"{c.name}_bf16.npz")
    inp = make_inputs(c, bf16=True)
    for tag in _steps(c):
        for x, w, ref in (("q", "w_q_norm", "q_normed"), ("k", "w_k_norm", "k_normed")):
            ours = O.rms_norm(O.bf16_to_f32(g[f"{tag}_{x}_proj_bits"]), inp[w], c.eps, "bf16")
            np.testing.assert_array_equal(O.bf16_bits(ours), g[f"{tag}_{ref}_bits"])


@pytest.mark.parametrize("D,theta", ROPE_TABLE_CASES)
def test_rope_table_matches_reference(D, theta):
    g = load("rope_tables.npz")
    np.testing.assert_array_equal(g["positions"], ROPE_POSITIONS)
    cos, sin = O.rope_build_cos_sin(ROPE_POSITIONS, D, theta)
    key = f"d{D}_t{int(theta)}"
    # The oracle's fp32 exp/cos/sin are correctly rounded; LibTorch's are 1-ulp approximations.
    # A one-ulp difference in inv_freq[j] moves the angle pos*inv_freq[j] by up to pos ulps of
    # inv_freq[j], so the bound grows with the position; elsewhere both are within 2 ulp.
    inv = O.rope_inv_freq(D, theta)
    ulp = np.spacing(inv).astype(np.float64)
    angle = ROPE_POSITIONS[:, None].astype(np.float32) * inv[None, :]
    # pos * ulp(inv) from the exp, plus one ulp of the rounded product, plus the trig itself
    bound = (ROPE_POSITIONS[:, None].astype(np.float64) * ulp[None, :] * 1.01
             + np.spacing(angle).astype(np.float64) + 2.5e-7)
    for name, ours in (("cos_", cos), ("sin_", sin)):
        err = np.abs(ours[:, : D // 2].astype(np.float64) - g[name + key].astype(np.float64))
        assert (err <= bound).all(), (name, float(err.max()))
        # the angle differs only in columns where inv_freq itself differs: most entries agree
        assert (err <= 2.5e-7).mean() > 0.97
    np.testing.assert_array_equal(cos[:, : D // 2], cos[:, D // 2:])


def test_oracle_planted_mistake_is_caught():
    """A deliberately wrong oracle (RoPE halves swapped the wrong way) must fail the pin."""
    c = CASES[2]
    g = load(f"{c.name}_bf16.npz")
    cos, sin = g["prefill_rope_cos"], g["prefill_rope_sin"]
    k = O.bf16_to_f32(g["prefill_k_normed_bits"])
    half = k.shape[-1] // 2
    wrong = np.concatenate([k[..., half:], -k[..., :half]], axis=-1)   # cat(x2, -x1): sign flip
    bad = O.round_bf16((k * cos).astype(np.float32) + (wrong * sin).astype(np.float32))
    assert not np.array_equal(O.bf16_bits(bad), g["prefill_key_bits"][:, :, : k.shape[2]])


def test_sampler_oracle_matches_reference_fixture():
    """oracle/sampler_oracle.py against the compiled reference Sampler (tests/golden/sampler.npz):
    the penalised logits bit for bit and the greedy token, bf16 and fp32, penalties 1.0/1.3/2.0."""
    from oracle import sampler_oracle as SO
    from tests.golden.cases import SAMPLER_PENALTIES, make_sampler_inputs
    g = np.load(os.path.join(GOLDEN_DIR, "sampler.npz"))
    logits, hist = make_sampler_inputs()
    np.testing.assert_array_equal(logits, g["logits"])
    for dn in ("bf16", "f32"):
        for pen in SAMPLER_PENALTIES:
            for r in range(logits.shape[0]):
                tag = f"{dn}_p{int(pen * 10)}_r{r}"
                tok, x = SO.sample_greedy(logits[r], hist[r], pen, dn)
                assert tok == int(g["token_" + tag]), tag
                np.testing.assert_array_equal(x.view(np.uint32), g["logits_" + tag].view(np.uint32), err_msg=tag)
