"""Full-size parity of the kernels at the workload shapes, against a torch fp32 restatement of
Attention.h:220-316 (tests/helpers.py) and through size-independent properties:
  * softmax rows sum to one: with every V row = 1 the output is exactly 1;
  * causality: changing cache rows after position p leaves every query row <= p bit-identical.
Needs a B200."""
import math

import numpy as np
import pytest

from tests.helpers import ATOL, RTOL, torch_attention_ref

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def rt(cuda_device):
    from mllm_b200 import build
    build.build()
    from mllm_b200 import runtime
    return runtime


def _cache(rt, B, Hkv, D, L, seed, cap=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    c = rt.KVCache(B, Hkv, D, cap or L, zero=False)
    c.key_buf.normal_(generator=g)
    c.value_buf.normal_(generator=g)
    return c


def test_decode_qwen3_8b_b32_l4096(rt):
    """Qwen3-8B decode step: fused epilogue (QK-norm, RoPE at position 4095, append) + decode
    over 4096 rows for 32 sequences, against the fp32 restatement on the same cache."""
    B, H, Hkv, D, L = 32, 32, 8, 128, 4096
    cache = _cache(rt, B, Hkv, D, L, seed=1)
    cache.set_lengths([L - 1] * B)
    g = torch.Generator(device="cuda").manual_seed(2)
    q = torch.randn(B, 1, H * D, device="cuda", generator=g).bfloat16().view(B, 1, H, D).transpose(1, 2)
    k = torch.randn(B, 1, Hkv * D, device="cuda", generator=g).bfloat16().view(B, 1, Hkv, D).transpose(1, 2)
    v = torch.randn(B, 1, Hkv * D, device="cuda", generator=g).bfloat16().view(B, 1, Hkv, D).transpose(1, 2)
    gq = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16()
    gk = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16()
    pos = torch.tensor([L - 1], device="cuda")
    qr = rt.qkv_epilogue(q, k, v, cache, pos, 1e6, gq, gk, 1e-6)
    out = rt.decode_attention(qr, cache, Hkv)
    ref = torch_attention_ref(qr, cache.key_buf, cache.value_buf, [L] * B)      # [B, 1, H, D]
    np.testing.assert_allclose(out.float().view(B, H, D).cpu().numpy(),
                               ref.view(B, H, D).cpu().numpy(), rtol=RTOL, atol=ATOL)


def test_ragged_decode_qwen3_14b_64_requests(rt):
    """Qwen3-14B head geometry (40 q heads, 8 kv heads) with 64 requests of lengths drawn
    uniformly from [256, 32768]: per-sequence lengths in one launch."""
    rng = np.random.default_rng(4)
    lens = [int(x) for x in rng.integers(256, 32769, size=64)]
    B, H, Hkv, D = 64, 40, 8, 128
    cap = max(lens)
    cache = _cache(rt, B, Hkv, D, cap, seed=5)
    cache.set_lengths(lens)
    q = torch.randn(B, H, D, device="cuda").bfloat16()
    out = rt.decode_attention(q, cache, Hkv, max_kv_len=cap).float().view(B, H, D)
    for b0 in range(0, B, 16):
        idx = list(range(b0, b0 + 16))
        ref = torch_attention_ref(q[idx][:, :, None, :], cache.key_buf[idx], cache.value_buf[idx],
                                  [lens[i] for i in idx]).view(16, H, D)
        np.testing.assert_allclose(out[idx].cpu().numpy(), ref.cpu().numpy(), rtol=RTOL, atol=ATOL)


def _prefill_setup(rt, B, H, Hkv, D, S, seed):
    cache = _cache(rt, B, Hkv, D, S, seed=seed)
    cache.set_lengths([S] * B)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    q = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
    return cache, q


def test_prefill_qwen3_8b_b4_s8192(rt):
    """Qwen3-8B causal prefill, batch 4 x 8192: sampled query blocks (start, middle, end)
    against the fp32 restatement."""
    B, H, Hkv, D, S = 4, 32, 8, 128, 8192
    cache, q = _prefill_setup(rt, B, H, Hkv, D, S, seed=7)
    out = rt.prefill_attention(q, cache, Hkv).view(B, S, H, D)
    for r0 in (0, 4000, S - 256):
        rows = slice(r0, r0 + 256)
        ref = torch_attention_ref(q, cache.key_buf, cache.value_buf, [S] * B, q_rows=rows)
        np.testing.assert_allclose(out[:, rows].float().cpu().numpy(), ref.cpu().numpy(), rtol=RTOL, atol=ATOL)


def test_prefill_rows_sum_to_one_full_size(rt):
    """Every softmax row sums to 1: with V = 1 the full 4 x 8192 output is 1 (bf16-exact)."""
    B, H, Hkv, D, S = 4, 32, 8, 128, 8192
    cache, q = _prefill_setup(rt, B, H, Hkv, D, S, seed=9)
    cache.value_buf.fill_(1.0)
    out = rt.prefill_attention(q, cache, Hkv).float()
    assert torch.isfinite(out).all()
    assert (out - 1.0).abs().max().item() <= 2 ** -7


def test_prefill_is_causal_full_size(rt):
    """Changing cache rows after position p does not change any output row <= p (bitwise)."""
    B, H, Hkv, D, S = 2, 32, 8, 128, 8192
    cache, q = _prefill_setup(rt, B, H, Hkv, D, S, seed=11)
    before = rt.prefill_attention(q, cache, Hkv).clone()
    p = 5000
    cache.key_buf[:, :, p + 1:S].mul_(-3.0)
    cache.value_buf[:, :, p + 1:S].add_(7.0)
    after = rt.prefill_attention(q, cache, Hkv)
    assert torch.equal(before[:, : p + 1], after[:, : p + 1])
    assert not torch.equal(before[:, p + 1:], after[:, p + 1:])


def test_tinyllama_layer_prefill_512_then_64_decode(rt):
    """TinyLlama-1.1B attention layer: prefill 512 then 64 decode steps through
    Attention.forward, against the numpy oracle in fp32 (Attention.h:29-86)."""
    from oracle import attention_oracle as O
    rng = np.random.default_rng(12)
    B, S, E, H, Hkv, D, theta = 1, 512, 2048, 32, 4, 64, 1e4
    r16 = lambda a: O.round_bf16(a.astype(np.float32))
    hid = r16(rng.standard_normal((B, S, E)))
    w = {n: r16(rng.standard_normal(s) * 0.02) for n, s in
         (("w_q", (H * D, E)), ("w_k", (Hkv * D, E)), ("w_v", (Hkv * D, E)), ("w_o", (E, H * D)))}
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().bfloat16()
    cache = rt.KVCache(B, Hkv, D, S + 64)
    ref_cache = O.KVCache()
    out = rt.Attention.forward(T(hid), T(w["w_q"]), T(w["w_k"]), T(w["w_v"]), T(w["w_o"]), H, Hkv, D, theta,
                               torch.arange(S, device="cuda"), cache)
    ref = O.attention_forward(hid, w["w_q"], w["w_k"], w["w_v"], w["w_o"], H, Hkv, D, theta, np.arange(S),
                              ref_cache)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    for step in range(64):
        x = r16(rng.standard_normal((B, 1, E)))
        pos = np.array([ref_cache.key.shape[2]])
        out = rt.Attention.forward(T(x), T(w["w_q"]), T(w["w_k"]), T(w["w_v"]), T(w["w_o"]), H, Hkv, D, theta,
                                   torch.from_numpy(pos).cuda(), cache)
        ref = O.attention_forward(x, w["w_q"], w["w_k"], w["w_v"], w["w_o"], H, Hkv, D, theta, pos, ref_cache)
        np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=RTOL, atol=ATOL, err_msg=f"step {step}")
    assert cache.length == S + 64
