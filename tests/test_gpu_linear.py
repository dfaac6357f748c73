"""mllm_linear_bf16, the projection GEMM for decode-sized token counts, against an fp32 torch
reference of the same bf16 inputs: q/k/v in one launch, o_proj, the k tail, strided operands,
token counts across every padded width, the unsplit and cluster-split paths."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

from mllm_b200 import runtime as rt  # noqa: E402

CASES = [
    # tokens, in_features, out_features per weight
    (1, 4096, (4096, 1024, 1024)),     # Qwen3-8B q|k|v, one token
    (32, 4096, (4096, 1024, 1024)),    # Qwen3-8B q|k|v, decode batch 32
    (32, 4096, (4096,)),               # Qwen3-8B o_proj, decode batch 32
    (33, 512, (256,)),
    (64, 320, (128, 384)),             # 5 k-atoms: the second 4-atom stage is mostly past K
    (100, 2048, (2048, 256, 256)),     # TinyLlama q|k|v
    (200, 4096, (4096,)),              # 256-wide token tile, reduction in four rounds
    (256, 1024, (512,)),
    (17, 256, (20480,)),               # 160 tiles: one CTA per tile, no split
    (8, 64, (128,)),                   # a single k-atom
    (130, 192, (256,)),                # 3 k-atoms in 2-atom stages
    (5, 5120, (5120, 1024, 1024)),     # Qwen3-14B q|k|v
]


def _operands(T, K, ns, pad, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    xs = torch.full((T, K + pad), float("nan"), device="cuda", dtype=torch.bfloat16)
    xs[:, :K] = torch.randn(T, K, device="cuda", generator=g).bfloat16()
    ws = []
    for n in ns:
        w = torch.full((n, K + pad), float("nan"), device="cuda", dtype=torch.bfloat16)
        w[:, :K] = (0.02 * torch.randn(n, K, device="cuda", generator=g)).bfloat16()
        ws.append(w[:, :K])
    return xs[:, :K], ws


@pytest.mark.parametrize("T,K,ns", CASES)
@pytest.mark.parametrize("pad", [0, 8])
def test_linear_vs_fp32_reference(T, K, ns, pad):
    x, ws = _operands(T, K, ns, pad, seed=T * 31 + K)
    out = rt.linear(x, ws)
    assert out.shape == (T, sum(ns)) and out.dtype == torch.bfloat16
    ref = torch.cat([x.float() @ w.float().t() for w in ws], 1)
    got = out.float()
    assert torch.isfinite(got).all(), "the padding beyond K was read"
    scale = ref.pow(2).mean().sqrt().item()
    np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=1e-2, atol=1e-2 * scale)
    # fp32 accumulation rounded once: nearly every output equals the rounded fp32 reference
    same = (out == ref.bfloat16()).float().mean().item()
    assert same > 0.97, same
    # deterministic: the split partials are added in a fixed order
    assert torch.equal(rt.linear(x, ws), out)
    # the tile counters at the start of the (shared) workspace are back at zero
    wsb = rt._LINEAR_WS.get((x.device, torch.cuda.current_stream().cuda_stream))
    if wsb is not None:
        assert int(wsb[:4096].view(torch.int32).abs().sum()) == 0


def test_projection_views_feed_the_attention_step():
    """attention_block at decode size takes q|k|v from one launch; the result matches the same
    block with the projections forced through cuBLAS, within bf16 tolerance."""
    B, S, E, H, Hkv, D = 4, 1, 1024, 8, 2, 128
    g = torch.Generator(device="cuda").manual_seed(5)
    r = lambda *s, sc=1.0: (sc * torch.randn(*s, device="cuda", generator=g)).bfloat16()
    h, wq, wk, wv, wo = r(B, S, E), r(H * D, E, sc=0.02), r(Hkv * D, E, sc=0.02), r(Hkv * D, E, sc=0.02), \
        r(E, H * D, sc=0.02)
    pos = torch.tensor([7], device="cuda")
    outs = []
    for use_kernel in (True, False):
        cache = rt.KVCache(B, Hkv, D, 16)
        cache.advance(7)
        saved = rt.LINEAR_MAX_TOKENS
        if not use_kernel:
            rt.LINEAR_MAX_TOKENS = 0
        try:
            outs.append(rt.attention_block(h, wq, wk, wv, wo, H, Hkv, D, 1e6, pos, cache).float())
        finally:
            rt.LINEAR_MAX_TOKENS = saved
    np.testing.assert_allclose(outs[0].cpu().numpy(), outs[1].cpu().numpy(), rtol=2e-2, atol=2e-2)
