"""Parity of the sm_100a kernels (called through the C ABI) against the oracle and the
reference's own golden outputs.  Needs a B200."""
import math
import os

import numpy as np
import pytest

from oracle import attention_oracle as O
from tests.golden.cases import CASES, GOLDEN_DIR, ROPE_POSITIONS, ROPE_TABLE_CASES, make_inputs
from tests.helpers import ATOL, RTOL, f32_to_torch_bf16, np_bits_to_torch, torch_to_bits

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def rt(cuda_device):
    from mllm_b200 import build
    build.build()
    from mllm_b200 import runtime
    return runtime


def _golden(name):
    return np.load(os.path.join(GOLDEN_DIR, name))


def _steps(c):
    return ["prefill"] + [f"decode{i}" for i in range(c.decode_steps)]


# ---------------------------------------------------------------------------------------
# RoPE table
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("D,theta", ROPE_TABLE_CASES)
def test_rope_table_vs_reference(rt, D, theta):
    g = _golden("rope_tables.npz")
    pos = torch.from_numpy(ROPE_POSITIONS).cuda()
    cos, sin = rt.RoPE.build_cos_sin(pos, D, theta)
    cos, sin = cos.cpu().numpy(), sin.cpu().numpy()
    np.testing.assert_array_equal(cos[:, : D // 2], cos[:, D // 2:])
    inv = O.rope_inv_freq(D, theta)
    angle = ROPE_POSITIONS[:, None].astype(np.float32) * inv[None, :]
    # device expf/cosf are within 2 ulp; the reference's CPU exp is within 1 ulp: the angle can
    # differ by pos * 2 ulp(inv_freq) + 1 ulp(angle)
    bound = (ROPE_POSITIONS[:, None] * np.spacing(inv)[None, :] * 2.02 + np.spacing(angle) + 5e-7)
    key = f"d{D}_t{int(theta)}"
    for name, ours in (("cos_", cos), ("sin_", sin)):
        err = np.abs(ours[:, : D // 2].astype(np.float64) - g[name + key])
        assert (err <= bound).all(), (name, float(err.max()))


def test_rope_inline_equals_table(rt):
    """The epilogue's in-kernel angles are bit-identical to mllm_rope_build_cos_sin's table."""
    B, H, Hkv, S, D = 2, 4, 2, 33, 128
    gen = torch.Generator(device="cuda").manual_seed(3)
    q = torch.randn(B, H, S, D, device="cuda", generator=gen).bfloat16()
    k = torch.randn(B, Hkv, S, D, device="cuda", generator=gen).bfloat16()
    v = torch.randn(B, Hkv, S, D, device="cuda", generator=gen).bfloat16()
    pos = torch.arange(4000, 4000 + S, device="cuda")
    c1 = rt.KVCache(B, Hkv, D, 64)
    c2 = rt.KVCache(B, Hkv, D, 64)
    q1 = rt.qkv_epilogue(q, k, v, c1, pos, 1e6)
    table = rt.RoPE.build_cos_sin(pos, D, 1e6)
    q2 = rt.qkv_epilogue(q, k, v, c2, pos, 1e6, rope_table=table)
    assert torch.equal(q1, q2)
    assert torch.equal(c1.key, c2.key) and torch.equal(c1.value, c2.value)
    # RoPE.apply with the same table gives the same rotation
    assert torch.equal(rt.RoPE.apply(q, *table), q1)


# ---------------------------------------------------------------------------------------
# Fused QKV epilogue: bit-exact KV cache against the reference (bf16 run)
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("c", CASES, ids=lambda c: c.name)
def test_epilogue_kv_cache_bit_exact(rt, c):
    """Feeding the reference's own bf16 projections and RoPE table, the fused epilogue writes
    exactly the reference's KVCache::key/value bits (Attention.h:183-208) at every step, and
    the rotated q equals the pinned oracle's."""
    g = _golden(f"{c.name}_bf16.npz")
    inp = make_inputs(c, bf16=True)
    B, H, Hkv, D = c.batch, c.num_heads, c.num_kv_heads, c.head_dim
    cap = c.seq + c.decode_steps + 5
    cache = rt.KVCache(B, Hkv, D, cap, zero=False)   # garbage beyond the rows we write
    qn = kn = None
    if c.qk_norm:
        qn = f32_to_torch_bf16(inp["w_q_norm"], "cuda")
        kn = f32_to_torch_bf16(inp["w_k_norm"], "cuda")
    for tag in _steps(c):
        # projections as [B, S, h, D] -> transposed views, exactly like TransformerBlock.h:91-96
        qp = np_bits_to_torch(g[f"{tag}_q_proj_bits"], "cuda")       # [B,H,S,D]
        kp = np_bits_to_torch(g[f"{tag}_k_proj_bits"], "cuda")
        vp = np_bits_to_torch(g[f"{tag}_v_bits"], "cuda")
        S = qp.shape[2]
        qv = qp.transpose(1, 2).contiguous().transpose(1, 2)
        kv_ = kp.transpose(1, 2).contiguous().transpose(1, 2)
        vv = vp.transpose(1, 2).contiguous().transpose(1, 2)
        cos = torch.from_numpy(g[f"{tag}_rope_cos"]).cuda()
        sin = torch.from_numpy(g[f"{tag}_rope_sin"]).cuda()
        pos = torch.from_numpy(g[f"{tag}_pos"]).cuda()
        qr = rt.qkv_epilogue(qv, kv_, vv, cache, pos, c.rope_theta, qn, kn, c.eps, rope_table=(cos, sin))
        L = cache.length
        assert L == g[f"{tag}_key_bits"].shape[2]
        np.testing.assert_array_equal(torch_to_bits(cache.key), g[f"{tag}_key_bits"], err_msg=tag)
        np.testing.assert_array_equal(torch_to_bits(cache.value), g[f"{tag}_value_bits"], err_msg=tag)
        # q: oracle (pinned bit-exact) on the same inputs
        q_in = O.bf16_to_f32(g[f"{tag}_q_proj_bits"])
        if c.qk_norm:
            q_in = O.rms_norm(q_in, inp["w_q_norm"], c.eps, "bf16")
        q_ref = O.rope_apply(q_in, g[f"{tag}_rope_cos"], g[f"{tag}_rope_sin"], "bf16")
        np.testing.assert_array_equal(torch_to_bits(qr), O.bf16_bits(q_ref), err_msg=tag)


@pytest.mark.parametrize("H,Hkv,D,qk_norm,table,S", [(32, 8, 128, True, False, 1536), (40, 8, 128, True, True, 1536),
                                                     (32, 4, 64, False, False, 1536), (4, 1, 128, True, False, 1539),
                                                     (16, 4, 128, True, True, 1536), (8, 2, 64, True, False, 1539)])
def test_epilogue_many_tokens_equals_chunked(rt, H, Hkv, D, qk_norm, table, S):
    """A call over many tokens (the TMA-box kernel) writes bit-identical q rows and cache rows to
    the same tokens epilogued in small chunks (the warp-per-row kernel, pinned bit-exact to the
    reference above): Qwen3-8B, Qwen3-14B with a RoPE table, TinyLlama geometry, and the per-rank
    head counts of Qwen3-8B split over 8 and 2 GPUs (1539 tokens per sequence: each sequence ends in a
    partial group of tokens)."""
    B, chunk = 2, 256
    g = torch.Generator(device="cuda").manual_seed(H + D)
    proj = (torch.randn(B, S, (H + 2 * Hkv) * D, device="cuda", generator=g) * 0.7).bfloat16()
    q = proj[..., : H * D].view(B, S, H, D).transpose(1, 2)
    k = proj[..., H * D:(H + Hkv) * D].view(B, S, Hkv, D).transpose(1, 2)
    v = proj[..., (H + Hkv) * D:].view(B, S, Hkv, D).transpose(1, 2)
    gq = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16() if qk_norm else None
    gk = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16() if qk_norm else None
    pos = torch.arange(S, device="cuda") + 3
    tab = rt.RoPE.build_cos_sin(pos, D, 1e6) if table else None
    whole = rt.KVCache(B, Hkv, D, S)
    q_whole = rt.qkv_epilogue(q, k, v, whole, pos, 1e6, gq, gk, 1e-6, rope_table=tab)
    parts = rt.KVCache(B, Hkv, D, S)
    q_parts = []
    for s0 in range(0, S, chunk):
        sl = slice(s0, s0 + chunk)
        tp = (tab[0][sl], tab[1][sl]) if table else None
        q_parts.append(rt.qkv_epilogue(q[:, :, sl], k[:, :, sl], v[:, :, sl], parts, pos[sl], 1e6, gq, gk, 1e-6,
                                       rope_table=tp))
    as_bits = lambda t: t.contiguous().view(torch.int16)
    assert torch.equal(as_bits(q_whole), as_bits(torch.cat(q_parts, dim=2)))
    assert torch.equal(as_bits(whole.key_buf), as_bits(parts.key_buf))
    assert torch.equal(as_bits(whole.value_buf), as_bits(parts.value_buf))


def test_epilogue_rejects_bad_slots(rt):
    """A cache slot past the capacity is not written and is reported on the device status."""
    from mllm_b200 import abi
    B, H, Hkv, S, D = 1, 2, 1, 4, 64
    q = torch.randn(B, H, S, D, device="cuda").bfloat16()
    k = torch.randn(B, Hkv, S, D, device="cuda").bfloat16()
    cache = rt.KVCache(B, Hkv, D, 6)
    cache.set_lengths([4])        # rows 4..7 requested, capacity 6: rows 6 and 7 are refused
    before = cache.key_buf.clone()
    lib = abi.load()
    abi.call("mllm_qkv_epilogue_bf16", q.data_ptr(), q.stride(0), q.stride(2), q.stride(1),
             k.data_ptr(), k.stride(0), k.stride(2), k.stride(1), k.data_ptr(), k.stride(0), k.stride(2),
             k.stride(1), B, S, H, Hkv, D, torch.arange(S, device="cuda").data_ptr(), 0, 1, 1e4, None,
             None, 0, 0, None, None, 1e-6, torch.empty_like(q).data_ptr(), cache.key_buf.data_ptr(),
             cache.value_buf.data_ptr(), *cache.strides, 6, cache.lengths.data_ptr(), 0, None)
    st = lib.mllm_attn_device_status(None)
    assert st == 7  # MLLM_ERR_DEVICE_LENGTH
    assert torch.equal(cache.key_buf[0, 0, :4], before[0, 0, :4])
    assert lib.mllm_attn_device_status(None) == 0  # cleared


def test_epilogue_many_tokens_rejects_bad_slots(rt):
    """The many-token kernel refuses the same way: tokens whose cache row is past the capacity
    get no K/V row and raise the device status, every other row is written as in a call that fits."""
    from mllm_b200 import abi
    lib = abi.load()
    B, H, Hkv, S, D, start = 1, 4, 2, 1200, 128, 100
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, Hkv, S, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, device="cuda", generator=g).bfloat16()
    pos = torch.arange(S, device="cuda")

    def run(capacity):
        cache = rt.KVCache(B, Hkv, D, capacity)
        cache.set_lengths([start])
        q_out = torch.empty_like(q)
        abi.call("mllm_qkv_epilogue_bf16", q.data_ptr(), q.stride(0), q.stride(2), q.stride(1),
                 k.data_ptr(), k.stride(0), k.stride(2), k.stride(1), v.data_ptr(), v.stride(0), v.stride(2),
                 v.stride(1), B, S, H, Hkv, D, pos.data_ptr(), 0, 1, 1e4, None, None, 0, 0, None, None, 1e-6,
                 q_out.data_ptr(), cache.key_buf.data_ptr(), cache.value_buf.data_ptr(), *cache.strides,
                 capacity, cache.lengths.data_ptr(), 0, None)
        return q_out, cache, lib.mllm_attn_device_status(None)

    q_fit, fit, st_fit = run(start + S)
    q_cut, cut, st_cut = run(S)          # rows S .. start + S - 1 do not exist
    assert st_fit == 0 and st_cut == 7   # MLLM_ERR_DEVICE_LENGTH
    assert torch.equal(q_cut, q_fit)
    assert torch.equal(cut.key_buf[:, :, start:S], fit.key_buf[:, :, start:S])
    assert torch.equal(cut.value_buf[:, :, start:S], fit.value_buf[:, :, start:S])
    assert lib.mllm_attn_device_status(None) == 0


# ---------------------------------------------------------------------------------------
# Decode
# ---------------------------------------------------------------------------------------

DECODE_CASES = [
    # B, H, Hkv, D, lengths (per sequence)
    (3, 8, 2, 128, [1, 64, 65]),
    (4, 32, 8, 128, [300, 513, 2048, 4097]),
    (2, 10, 2, 128, [777, 1]),           # GQA group 5
    (2, 32, 4, 64, [512, 129]),          # TinyLlama geometry (group 8, D=64)
    (5, 4, 4, 64, [17, 256, 255, 1000, 3]),   # MHA
]


@pytest.mark.parametrize("B,H,Hkv,D,lens", DECODE_CASES)
def test_decode_vs_oracle(rt, B, H, Hkv, D, lens):
    rng = np.random.default_rng(B * 100 + H)
    cap = max(lens) + 70
    cache = rt.KVCache(B, Hkv, D, cap, zero=False)
    cache.key_buf.fill_(float("nan"))     # rows beyond each length must never leak
    cache.value_buf.fill_(float("nan"))
    kc = O.round_bf16(rng.standard_normal((B, Hkv, cap, D)).astype(np.float32))
    vc = O.round_bf16(rng.standard_normal((B, Hkv, cap, D)).astype(np.float32))
    for b, L in enumerate(lens):
        cache.key_buf[b, :, :L] = f32_to_torch_bf16(kc[b, :, :L], "cuda")
        cache.value_buf[b, :, :L] = f32_to_torch_bf16(vc[b, :, :L], "cuda")
    cache.set_lengths(lens)
    q = O.round_bf16(rng.standard_normal((B, H, D)).astype(np.float32))
    out = rt.decode_attention(f32_to_torch_bf16(q, "cuda"), cache, Hkv)
    got = out.float().cpu().numpy().reshape(B, H * D)
    ref = O.decode_attention(q, kc, vc, lens, H, Hkv, D)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)


def test_decode_plan(rt):
    """The chunk plan: one chunk per (sequence, kv head) when the pairs alone fill the grid for
    long enough (Qwen3-8B batch 32, 4096 rows: no partials, no combine launch); several, taken
    from the workspace counter, for few pairs or long ragged caches."""
    import ctypes as C
    lib = rt.abi.load()

    def plan(*shape):
        r, c, n = C.c_int(), C.c_int(), C.c_int()
        assert lib.mllm_decode_attention_plan(*shape, C.byref(r), C.byref(c), C.byref(n)) == 0
        return r.value, c.value, n.value
    assert plan(32, 32, 8, 128, 4096) == (4096, 1, 1)
    rows, chunks, launches = plan(8, 32, 8, 128, 2048)
    assert chunks > 1 and launches == 2 and rows * chunks >= 2048 and rows % 64 == 0
    rows, chunks, launches = plan(64, 40, 8, 128, 32069)
    assert chunks > 1 and launches == 2 and rows * chunks >= 32069


def test_decode_large_ragged_batch(rt):
    """A ragged batch large enough that every persistent CTA takes several items from the
    workspace counter, with many empty chunks (short sequences in a long-plan batch): every
    sequence against a torch fp32 reference, paged bit-identical to contiguous, repeated calls
    bit-identical (items may land on other CTAs; each is computed and merged the same way)."""
    import random
    B, H, Hkv, D = 64, 40, 8, 128
    rng = np.random.default_rng(2024)
    lens = rng.integers(1, 6000, B).tolist()
    lens[0], lens[1], lens[2] = 6144, 1, 4096        # the longest plans the chunks; tile and chunk edges
    Lmax = max(lens)
    g = torch.Generator(device="cuda").manual_seed(7)
    cont = rt.KVCache(B, Hkv, D, Lmax, zero=False)
    cont.key_buf.copy_(torch.randn(cont.key_buf.shape, device="cuda", generator=g))
    cont.value_buf.copy_(torch.randn(cont.value_buf.shape, device="cuda", generator=g))
    cont.set_lengths(lens)
    q = torch.randn(B, H, D, device="cuda", generator=g).bfloat16()
    out = rt.decode_attention(q, cont, Hkv).view(B, H, D).float()
    n_rep = H // Hkv
    for b, L in enumerate(lens):
        k = cont.key_buf[b, :, :L].float().repeat_interleave(n_rep, 0)      # [H, L, D]
        v = cont.value_buf[b, :, :L].float().repeat_interleave(n_rep, 0)
        p = torch.softmax((q[b].float().unsqueeze(1) @ k.transpose(1, 2)) / math.sqrt(D), -1)
        ref = (p @ v).squeeze(1)
        torch.testing.assert_close(out[b], ref, rtol=2e-2, atol=2e-2, msg=f"sequence {b} (L={L})")
    bits = lambda t: t.contiguous().view(torch.int16)
    again = rt.decode_attention(q, cont, Hkv).view(B, H, D)
    assert torch.equal(bits(again), bits(out.bfloat16()))
    block = 256
    paged = rt.PagedKVCache(num_blocks=sum(-(-L // block) for L in lens) + 2, num_kv_heads=Hkv, head_dim=D,
                            block_size=block, max_seqs=B)
    random.Random(5).shuffle(paged._free)
    paged.set_lengths(lens)
    for b, L in enumerate(lens):
        for i, blk in enumerate(paged.blocks_of(b)):
            r0, r1 = i * block, min(L, (i + 1) * block)
            paged.k_pool[blk, :, : r1 - r0] = cont.key_buf[b, :, r0:r1]
            paged.v_pool[blk, :, : r1 - r0] = cont.value_buf[b, :, r0:r1]
    assert torch.equal(bits(rt.decode_attention(q, paged, Hkv).view(B, H, D)), bits(again))


# ---------------------------------------------------------------------------------------
# Fused decode step (epilogue of the new token + decode in one launch)
# ---------------------------------------------------------------------------------------

DECODE_STEP_CASES = [
    # B, H, Hkv, D, cache rows before the new token (per sequence), QK-norm, rope table
    (4, 32, 8, 128, [0, 1, 63, 64], True, False),          # first token of a sequence; tile edges
    (3, 32, 8, 128, [255, 256, 1023], True, False),        # the new row alone in the last chunk
    (8, 40, 8, 128, [5000, 17, 4096, 300, 2047, 2048, 999, 12000], True, False),   # ragged, GQA 5
    (2, 32, 4, 64, [511, 70], False, False),               # TinyLlama geometry (no QK-norm)
    (2, 16, 4, 128, [100, 4095], True, True),              # caller-given RoPE table rows
]


@pytest.mark.parametrize("B,H,Hkv,D,prior,qk_norm,table", DECODE_STEP_CASES)
def test_decode_step_equals_epilogue_then_decode(rt, B, H, Hkv, D, prior, qk_norm, table):
    """The fused step writes bit-identical cache rows to the epilogue kernel and the same
    attention output as the epilogue + decode pair (up to fp32 summation order); both are also
    checked against the oracle."""
    rng = np.random.default_rng(sum(prior) + H)
    cap = max(prior) + 1 + 40
    g = torch.Generator(device="cuda").manual_seed(len(prior))
    a = rt.KVCache(B, Hkv, D, cap, zero=False)
    a.key_buf.normal_(generator=g)
    a.value_buf.normal_(generator=g)
    a.key_buf[:, :, max(prior):].fill_(float("nan"))   # nothing past the new rows may leak
    a.value_buf[:, :, max(prior):].fill_(float("nan"))
    for bb, L in enumerate(prior):
        a.key_buf[bb, :, L:].fill_(float("nan"))
        a.value_buf[bb, :, L:].fill_(float("nan"))
    a.set_lengths(prior)
    bcache = rt.KVCache(B, Hkv, D, cap, zero=False)
    bcache.key_buf.copy_(a.key_buf)
    bcache.value_buf.copy_(a.value_buf)
    bcache.set_lengths(prior)
    row = (H + 2 * Hkv) * D
    proj = f32_to_torch_bf16(O.round_bf16((rng.standard_normal((B, 1, row)) * 0.7).astype(np.float32)), "cuda")
    q = proj[:, :, : H * D].view(B, 1, H, D).transpose(1, 2)
    k = proj[:, :, H * D:(H + Hkv) * D].view(B, 1, Hkv, D).transpose(1, 2)
    v = proj[:, :, (H + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
    gq = gk = None
    if qk_norm:
        gq = f32_to_torch_bf16(O.round_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)), "cuda")
        gk = f32_to_torch_bf16(O.round_bf16((1 + 0.1 * rng.standard_normal(D)).astype(np.float32)), "cuda")
    pos = torch.tensor(prior, dtype=torch.int64, device="cuda")      # each sequence at its own position
    rope_table = rt.RoPE.build_cos_sin(pos, D, 1e6) if table else None
    # the separate pair: epilogue (positions [B, 1]) then decode
    qr = rt.qkv_epilogue(q, k, v, a, pos.view(B, 1), 1e6, gq, gk, 1e-6, rope_table=rope_table)
    want = rt.decode_attention(qr, a, Hkv).float()
    got = rt.decode_step(q, k, v, bcache, pos, 1e6, Hkv, gq, gk, 1e-6, rope_table=rope_table).float()
    assert bcache.host_lengths() == [L + 1 for L in prior]
    assert torch.equal(bcache.key_buf.view(torch.int16), a.key_buf.view(torch.int16))
    assert torch.equal(bcache.value_buf.view(torch.int16), a.value_buf.view(torch.int16))
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got, want, rtol=1e-2, atol=1e-2)
    # against the oracle on the appended cache
    kc = a.key_buf.float().cpu().numpy()
    vc = a.value_buf.float().cpu().numpy()
    ref = O.decode_attention(qr.float().cpu().numpy().reshape(B, H, D), kc, vc, [L + 1 for L in prior], H, Hkv, D)
    np.testing.assert_allclose(got.cpu().numpy().reshape(B, H * D), ref, rtol=RTOL, atol=ATOL)


# ---------------------------------------------------------------------------------------
# Paged KV cache
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("B,H,Hkv,D,S,block,qk_norm", [(3, 32, 8, 128, 300, 128, True),
                                                         (2, 40, 8, 128, 513, 256, True),
                                                         (2, 32, 4, 64, 200, 128, False)])
def test_paged_cache_equals_contiguous(rt, B, H, Hkv, D, S, block, qk_norm):
    """The same layer steps over a paged cache (blocks handed out in a shuffled order) and over a
    contiguous cache: bit-identical q rows, cache rows, prefill output, fused decode steps and a
    ragged decode."""
    import random
    g = torch.Generator(device="cuda").manual_seed(S + H)
    steps = 4
    cont = rt.KVCache(B, Hkv, D, S + steps + 8)
    paged = rt.PagedKVCache(num_blocks=B * (-(-(S + steps + 8) // block)) + 3, num_kv_heads=Hkv, head_dim=D,
                            block_size=block, max_seqs=B)
    random.Random(S).shuffle(paged._free)
    row = (H + 2 * Hkv) * D
    gq = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16() if qk_norm else None
    gk = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16() if qk_norm else None
    views = lambda pr, n: (pr[..., : H * D].view(B, n, H, D).transpose(1, 2),
                           pr[..., H * D:(H + Hkv) * D].view(B, n, Hkv, D).transpose(1, 2),
                           pr[..., (H + Hkv) * D:].view(B, n, Hkv, D).transpose(1, 2))
    bits = lambda t: t.contiguous().view(torch.int16)
    proj = (torch.randn(B, S, row, device="cuda", generator=g) * 0.7).bfloat16()
    pos = torch.arange(S, device="cuda")
    qc = rt.qkv_epilogue(*views(proj, S), cont, pos, 1e6, gq, gk, 1e-6)
    qp = rt.qkv_epilogue(*views(proj, S), paged, pos, 1e6, gq, gk, 1e-6)
    assert torch.equal(bits(qc), bits(qp))
    assert torch.equal(bits(rt.prefill_attention(qc, cont, Hkv)), bits(rt.prefill_attention(qp, paged, Hkv)))
    for step in range(steps):
        x = (torch.randn(B, 1, row, device="cuda", generator=g) * 0.7).bfloat16()
        p1 = torch.tensor([S + step], device="cuda")
        oc = rt.decode_step(*views(x, 1), cont, p1, 1e6, Hkv, gq, gk, 1e-6)
        op = rt.decode_step(*views(x, 1), paged, p1, 1e6, Hkv, gq, gk, 1e-6)
        assert torch.equal(bits(oc), bits(op)), f"decode step {step}"
    L = S + steps
    for b in range(B):
        kp, vp = paged.gather(b, L)
        assert torch.equal(bits(kp), bits(cont.key_buf[b, :, :L])) and torch.equal(bits(vp), bits(cont.value_buf[b, :, :L]))
    lens = [L - 3 * b for b in range(B)]      # ragged: attend over fewer rows for later sequences
    cont.set_lengths(lens)
    paged.set_lengths(lens)
    q1 = torch.randn(B, H, D, device="cuda", generator=g).bfloat16()
    assert torch.equal(bits(rt.decode_attention(q1, cont, Hkv)), bits(rt.decode_attention(q1, paged, Hkv)))


# ---------------------------------------------------------------------------------------
# Prefill
# ---------------------------------------------------------------------------------------

PREFILL_CASES = [
    # B, H, Hkv, D, q_len, prefix (cache rows before the new block)
    (1, 4, 2, 128, 1, 0),
    (2, 8, 2, 128, 128, 0),
    (1, 8, 2, 128, 200, 0),
    (2, 10, 2, 128, 77, 51),     # chunked prefill over an existing prefix, GQA 5
    (1, 32, 4, 64, 512, 0),      # TinyLlama geometry
    (1, 4, 4, 64, 300, 200),
    (1, 8, 8, 128, 384, 1),
]


@pytest.mark.parametrize("B,H,Hkv,D,S,prefix", PREFILL_CASES)
def test_prefill_vs_oracle(rt, B, H, Hkv, D, S, prefix):
    rng = np.random.default_rng(S * 7 + prefix)
    L = prefix + S
    cache = rt.KVCache(B, Hkv, D, L + 130, zero=False)
    cache.key_buf.fill_(float("nan"))
    cache.value_buf.fill_(float("nan"))
    kc = O.round_bf16(rng.standard_normal((B, Hkv, L, D)).astype(np.float32))
    vc = O.round_bf16(rng.standard_normal((B, Hkv, L, D)).astype(np.float32))
    cache.key_buf[:, :, :L] = f32_to_torch_bf16(kc, "cuda")
    cache.value_buf[:, :, :L] = f32_to_torch_bf16(vc, "cuda")
    cache.set_lengths([L] * B)
    q = O.round_bf16(rng.standard_normal((B, H, S, D)).astype(np.float32))
    out = rt.prefill_attention(f32_to_torch_bf16(q, "cuda"), cache, Hkv)
    got = out.float().cpu().numpy()
    ref = O.attention_core(q, kc, vc, H, Hkv, D)
    assert np.isfinite(got).all()
    np.testing.assert_allclose(got, ref, rtol=RTOL, atol=ATOL)


# ---------------------------------------------------------------------------------------
# Whole attention layer (projections in torch, the rest on the new kernels) vs the reference
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("c", CASES, ids=lambda c: c.name)
def test_layer_matches_reference_fp32(rt, c):
    """Prefill then decode steps through the mirror of Attention::Forward / the Qwen3 block,
    bf16 on the device, against the reference's fp32 CPU outputs (rtol = atol = 2e-2)."""
    g = _golden(f"{c.name}_f32.npz")
    inp = make_inputs(c, bf16=True)
    T = {k: f32_to_torch_bf16(v, "cuda") for k, v in inp.items()}
    H, Hkv, D = c.num_heads, c.num_kv_heads, c.head_dim
    cache = rt.KVCache(c.batch, Hkv, D, c.seq + c.decode_steps)
    steps = [("prefill", T["hidden"])] + [(f"decode{i}", T["decode_hidden"][i]) for i in range(c.decode_steps)]
    for tag, hid in steps:
        S = hid.shape[1]
        pos = (torch.tensor([cache.length], device="cuda") if (cache.is_initialized() and S == 1)
               else torch.arange(S, device="cuda"))
        np.testing.assert_array_equal(pos.cpu().numpy(), g[tag + "_pos"])
        if c.qk_norm:
            out = rt.attention_block(hid, T["w_q"], T["w_k"], T["w_v"], T["w_o"], H, Hkv, D, c.rope_theta,
                                     pos, cache, T["w_q_norm"], T["w_k_norm"], c.eps)
        else:
            out = rt.Attention.forward(hid, T["w_q"], T["w_k"], T["w_v"], T["w_o"], H, Hkv, D,
                                       c.rope_theta, pos, cache)
        np.testing.assert_allclose(out.float().cpu().numpy(), g[tag + "_out"], rtol=RTOL, atol=ATOL,
                                   err_msg=tag)
    np.testing.assert_allclose(cache.key.float().cpu().numpy(), g["key"], rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(cache.value.float().cpu().numpy(), g["value"], rtol=RTOL, atol=ATOL)


def test_no_cache_path(rt):
    """kv_cache == nullptr (Attention.h:183): attention over the call's own rows only."""
    c = CASES[0]
    inp = make_inputs(c, bf16=True)
    T = {k: f32_to_torch_bf16(v, "cuda") for k, v in inp.items()}
    pos = torch.arange(c.seq, device="cuda")
    out = rt.Attention.forward(T["hidden"], T["w_q"], T["w_k"], T["w_v"], T["w_o"], c.num_heads,
                               c.num_kv_heads, c.head_dim, c.rope_theta, pos, None)
    ref = O.attention_forward(inp["hidden"], inp["w_q"], inp["w_k"], inp["w_v"], inp["w_o"], c.num_heads,
                              c.num_kv_heads, c.head_dim, c.rope_theta, np.arange(c.seq), None)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, rtol=RTOL, atol=ATOL)


def test_reference_errors_are_kept(rt):
    with pytest.raises(RuntimeError, match="divisible"):
        rt.Attention.forward_projected(torch.zeros(1, 6, 2, 64, device="cuda").bfloat16(),
                                       torch.zeros(1, 4, 2, 64, device="cuda").bfloat16(),
                                       torch.zeros(1, 4, 2, 64, device="cuda").bfloat16(),
                                       torch.zeros(64, 384, device="cuda").bfloat16(), 6, 4, 64, 1e4,
                                       torch.arange(2, device="cuda"), None)
    with pytest.raises(RuntimeError, match="rank-4"):
        rt.Attention.forward_projected(torch.zeros(6, 2, 64, device="cuda").bfloat16(),
                                       torch.zeros(1, 4, 2, 64, device="cuda").bfloat16(),
                                       torch.zeros(1, 4, 2, 64, device="cuda").bfloat16(),
                                       torch.zeros(64, 384, device="cuda").bfloat16(), 4, 4, 64, 1e4,
                                       torch.arange(2, device="cuda"), None)
    with pytest.raises(RuntimeError, match="CPU fallback"):
        rt.RoPE.apply(torch.zeros(1, 1, 2, 64).bfloat16(), torch.zeros(2, 64), torch.zeros(2, 64))
