"""Packed sequences of different lengths: the varlen epilogue and prefill (several prompts in one
launch each) against the oracle, and bit-identical to the same sequences run one call each.
Needs a B200."""
import random

import numpy as np
import pytest

from oracle import attention_oracle as O
from tests.helpers import ATOL, RTOL, f32_to_torch_bf16

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def rt(cuda_device):
    from mllm_b200 import build
    build.build()
    from mllm_b200 import runtime
    return runtime


def bits(t):
    return t.contiguous().view(torch.int16)


def _cache(rt, paged, B, Hkv, D, rows, seed):
    """An empty cache for B sequences of up to `rows` rows: paged (128-row blocks handed out in
    a shuffled order) or contiguous (zero-filled)."""
    if paged:
        c = rt.PagedKVCache(num_blocks=B * (-(-rows // 128)) + 2, num_kv_heads=Hkv, head_dim=D, block_size=128,
                            max_seqs=B)
        random.Random(seed).shuffle(c._free)
        return c
    return rt.KVCache(B, Hkv, D, rows)


def _fill(rt, cache, b, k, v):
    """Write rows [Hkv, L, D] into sequence b of the cache (its length must already be L)."""
    L = k.shape[1]
    if isinstance(cache, rt.PagedKVCache):
        for i, blk in enumerate(cache.blocks_of(b)):
            r0, r1 = i * cache.block_size, min(L, (i + 1) * cache.block_size)
            if r0 < r1:
                cache.k_pool[blk, :, : r1 - r0] = k[:, r0:r1]
                cache.v_pool[blk, :, : r1 - r0] = v[:, r0:r1]
    else:
        cache.key_buf[b, :, :L] = k
        cache.value_buf[b, :, :L] = v


VARLEN_CASES = [
    # H, Hkv, D, q_lens, prefixes (cache rows before the new rows), paged
    (8, 2, 128, [37, 1, 300, 0, 129], [0, 5, 0, 3, 200], True),
    (32, 8, 128, [512, 257, 1000], [0, 0, 40], True),
    (10, 2, 128, [77, 200], [51, 0], False),          # GQA group 5, contiguous cache
    (32, 4, 64, [256, 3, 640], [0, 128, 1], True),    # D = 64
    (4, 4, 64, [1, 1, 1, 2], [10, 300, 0, 0], False),
]


@pytest.mark.parametrize("H,Hkv,D,q_lens,prefixes,paged", VARLEN_CASES)
def test_prefill_varlen_vs_oracle_and_per_sequence(rt, H, Hkv, D, q_lens, prefixes, paged):
    B = len(q_lens)
    rng = np.random.default_rng(sum(q_lens) + H)
    lens = [p + s for p, s in zip(prefixes, q_lens)]
    cache = _cache(rt, paged, B, Hkv, D, max(lens) + 130, seed=B)
    cache.set_lengths(lens)
    ks, vs = [], []
    for b, L in enumerate(lens):
        k = O.round_bf16(rng.standard_normal((Hkv, L, D)).astype(np.float32))
        v = O.round_bf16(rng.standard_normal((Hkv, L, D)).astype(np.float32))
        _fill(rt, cache, b, f32_to_torch_bf16(k, "cuda"), f32_to_torch_bf16(v, "cuda"))
        ks.append(k)
        vs.append(v)
    T = sum(q_lens)
    q = O.round_bf16(rng.standard_normal((H, T, D)).astype(np.float32))
    qd = f32_to_torch_bf16(q, "cuda")
    out = rt.prefill_attention_packed(qd, cache, q_lens, Hkv)
    assert out.shape == (T, H * D)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    r0 = 0
    for b, S in enumerate(q_lens):
        if S == 0:
            continue
        qb = np.ascontiguousarray(q[:, r0:r0 + S][None])
        ref = O.attention_core(qb, ks[b][None], vs[b][None], H, Hkv, D)[0]
        np.testing.assert_allclose(got[r0:r0 + S], ref, rtol=RTOL, atol=ATOL, err_msg=f"sequence {b}")
        # the same sequence through the one-length entry point: identical bits
        if paged:
            one = rt.prefill_attention(qd[:, r0:r0 + S][None].contiguous(), cache.slot(b), Hkv)
        else:
            c1 = rt.KVCache(1, Hkv, D, lens[b])
            c1.key_buf[0] = cache.key_buf[b, :, :lens[b]]
            c1.value_buf[0] = cache.value_buf[b, :, :lens[b]]
            c1.set_lengths([lens[b]])
            one = rt.prefill_attention(qd[:, r0:r0 + S][None].contiguous(), c1, Hkv)
        assert torch.equal(bits(one[0]), bits(out[r0:r0 + S])), f"sequence {b}"
        r0 += S


@pytest.mark.parametrize("H,Hkv,D,q_lens,qk_norm", [(8, 2, 128, [5, 0, 130, 1], True),
                                                     (32, 8, 128, [700, 1, 600], True),     # > 1024 tokens
                                                     (32, 4, 64, [300, 900], False)])
def test_epilogue_varlen_equals_per_sequence(rt, H, Hkv, D, q_lens, qk_norm):
    """Packed tokens of several sequences in one launch write the same Q and cache rows, bit for
    bit, as one epilogue call per sequence; the paged and contiguous forms agree."""
    B = len(q_lens)
    T = sum(q_lens)
    prefixes = [3 * b + (128 if b == 1 else 0) for b in range(B)]
    g = torch.Generator(device="cuda").manual_seed(T + H)
    row = (H + 2 * Hkv) * D
    x = (torch.randn(T, row, device="cuda", generator=g) * 0.7).bfloat16()
    gq = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16() if qk_norm else None
    gk = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16() if qk_norm else None
    views = lambda t, n: (t[:, : H * D].view(n, H, D), t[:, H * D:(H + Hkv) * D].view(n, Hkv, D),
                          t[:, (H + Hkv) * D:].view(n, Hkv, D))
    cap = max(p + s for p, s in zip(prefixes, q_lens)) + 8
    packed = _cache(rt, True, B, Hkv, D, cap, seed=1)
    single = _cache(rt, True, B, Hkv, D, cap, seed=2)
    cont = _cache(rt, False, B, Hkv, D, cap, seed=0)
    for c in (packed, single, cont):
        c.set_lengths(prefixes)
    qp = rt.qkv_epilogue_packed(*views(x, T), packed, q_lens, 1e6, None, gq, gk, 1e-6)
    qc = rt.qkv_epilogue_packed(*views(x, T), cont, q_lens, 1e6, None, gq, gk, 1e-6)
    assert qp.shape == (H, T, D)
    assert torch.equal(bits(qp), bits(qc))
    assert packed.host_lengths() == [p + s for p, s in zip(prefixes, q_lens)] == cont.host_lengths()
    r0 = 0
    for b, S in enumerate(q_lens):
        if S == 0:
            continue
        xb = x[r0:r0 + S]
        q1, k1, v1 = (t.unsqueeze(0).transpose(1, 2) for t in views(xb, S))
        pos = torch.arange(prefixes[b], prefixes[b] + S, device="cuda")
        qs = rt.qkv_epilogue(q1, k1, v1, single.slot(b), pos, 1e6, gq, gk, 1e-6)
        assert torch.equal(bits(qs[0]), bits(qp[:, r0:r0 + S])), f"sequence {b}"
        L = prefixes[b] + S
        kp, vp = packed.gather(b, L)
        ks, vs = single.gather(b, L)
        assert torch.equal(bits(kp[:, prefixes[b]:]), bits(ks[:, prefixes[b]:])), f"sequence {b}"
        assert torch.equal(bits(vp[:, prefixes[b]:]), bits(vs[:, prefixes[b]:])), f"sequence {b}"
        assert torch.equal(bits(kp[:, prefixes[b]:]), bits(cont.key_buf[b, :, prefixes[b]:L]))
        assert torch.equal(bits(vp[:, prefixes[b]:]), bits(cont.value_buf[b, :, prefixes[b]:L]))
        r0 += S


def test_packed_block_equals_per_sequence_pipeline(rt):
    """attention_block_packed = epilogue + attention per sequence on the same projections, and
    a decode step afterwards sees the packed prefill's cache rows."""
    H, Hkv, D, E = 16, 4, 128, 1024
    q_lens = [40, 129, 7]
    B, T = len(q_lens), sum(q_lens)
    g = torch.Generator(device="cuda").manual_seed(11)
    w = lambda o, i: (torch.randn(o, i, device="cuda", generator=g) * 0.02).bfloat16()
    w_q, w_k, w_v = w(H * D, E), w(Hkv * D, E), w(Hkv * D, E)
    gq = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16()
    gk = (1 + 0.1 * torch.randn(D, device="cuda", generator=g)).bfloat16()
    h = torch.randn(T, E, device="cuda", generator=g).bfloat16()
    cache = _cache(rt, True, B, Hkv, D, 512, seed=3)
    out = rt.attention_block_packed(h, w_q, w_k, w_v, None, H, Hkv, D, 1e6, q_lens, cache, gq, gk, 1e-6)
    ref_cache = _cache(rt, True, B, Hkv, D, 512, seed=4)
    q, k, v = rt._project_qkv(h.unsqueeze(0), w_q, w_k, w_v, H, Hkv, D)   # the same projection launch
    r0 = 0
    for b, S in enumerate(q_lens):
        sl = slice(r0, r0 + S)
        qr = rt.qkv_epilogue(q[:, :, sl], k[:, :, sl], v[:, :, sl], ref_cache.slot(b),
                             torch.arange(S, device="cuda"), 1e6, gq, gk, 1e-6)
        one = rt.prefill_attention(qr, ref_cache.slot(b), Hkv)
        assert torch.equal(bits(one[0]), bits(out[sl])), f"sequence {b}"
        r0 += S
    x1 = torch.randn(B, 1, (H + 2 * Hkv) * D, device="cuda", generator=g).bfloat16()
    qv = x1[..., : H * D].view(B, 1, H, D).transpose(1, 2)
    kv_ = x1[..., H * D:(H + Hkv) * D].view(B, 1, Hkv, D).transpose(1, 2)
    vv = x1[..., (H + Hkv) * D:].view(B, 1, Hkv, D).transpose(1, 2)
    pos = torch.tensor(q_lens, device="cuda")
    d1 = rt.decode_step(qv, kv_, vv, cache, pos, 1e6, Hkv, gq, gk, 1e-6)
    d2 = rt.decode_step(qv, kv_, vv, ref_cache, pos, 1e6, Hkv, gq, gk, 1e-6)
    assert torch.equal(bits(d1), bits(d2))


def test_varlen_rejects_inconsistent_sequences(rt):
    """A sequence whose cache length is shorter than its new rows, whose range runs past the
    packed rows, or that is longer than max_q_len is reported on the device status and its
    output rows are not written; the other sequences are computed."""
    import ctypes as C
    from mllm_b200 import abi
    lib = abi.load()
    H, Hkv, D = 4, 2, 64
    cache = _cache(rt, True, 3, Hkv, D, 512, seed=5)
    cache.set_lengths([100, 100, 300])
    q = torch.randn(H, 300, D, device="cuda").bfloat16()
    kv = cache.descriptor()
    # cu_q_lens, kv_lens, max_q_len, the bad sequence's rows, a good sequence's rows
    cases = (([0, 100, 250, 300], [100, 100, 300], 150, (100, 250), (0, 100)),   # 150 new rows, 100 cached
             ([0, 100, 200, 320], [100, 100, 300], 120, (200, 300), (100, 200)),  # past the 300 packed rows
             ([0, 10, 20, 300], [100, 100, 300], 150, (20, 300), (0, 10)))        # 280 rows > max_q_len
    for cu, kvl, max_q, bad, good in cases:
        out = torch.full((300, H * D), 7.0, device="cuda").bfloat16()
        cu_d = torch.tensor(cu, dtype=torch.int32, device="cuda")
        kv_d = torch.tensor(kvl, dtype=torch.int32, device="cuda")
        abi.call("mllm_prefill_attention_varlen_paged_bf16", q.data_ptr(), C.byref(kv), cu_d.data_ptr(),
                 kv_d.data_ptr(), 3, H, Hkv, D, 300, max_q, 0.125, out.data_ptr(), None)
        assert lib.mllm_attn_device_status(None) == 7   # MLLM_ERR_DEVICE_LENGTH
        assert lib.mllm_attn_device_status(None) == 0   # cleared
        assert bool((out[bad[0]:bad[1]] == 7.0).all()), cu
        assert not bool((out[good[0]:good[1]] == 7.0).any()), cu
    # host side: more packed rows than batch * max_q_len allows
    with pytest.raises(abi.MllmError):
        abi.call("mllm_prefill_attention_varlen_paged_bf16", q.data_ptr(), C.byref(kv), cu_d.data_ptr(),
                 kv_d.data_ptr(), 3, H, Hkv, D, 300, 50, 0.125, out.data_ptr(), None)
