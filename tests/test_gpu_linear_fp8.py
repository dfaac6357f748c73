"""mllm_linear_fp8_bf16: projections with FP8 (e4m3) weights and 128 x 128 block scales, the
layout of FP8 checkpoints, against the reference's route for them -- DequantizeFP8
(QwenRunner.cpp:103-122, restated in runtime.Fp8Weight.dequantize) followed by Linear::Forward --
computed here as an fp32 GEMM of the dequantized bf16 weights.  Then a whole FP8 decoder through
the serving model against the same model dequantized the reference's way."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

from mllm_b200 import runtime as rt  # noqa: E402

CASES = [
    # tokens, in_features, out_features
    (1, 4096, 4096),       # Qwen3-8B q_proj, one token
    (32, 4096, 4096),      # Qwen3-8B o_proj / q_proj, decode batch 32
    (32, 4096, 1024),      # Qwen3-8B k_proj
    (8, 4096, 12288),      # Qwen3-8B gate / up
    (64, 12288, 4096),     # Qwen3-8B down_proj, 96 k-blocks
    (128, 1024, 512),      # the widest token tile
    (17, 384, 256),        # 3 k-blocks, odd token count
    (100, 5120, 5120),     # Qwen3-14B q_proj
]


def _weights(N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    # block scales spread over a wide range, so a wrong block index shows
    w = w * (1 + 4 * torch.rand(N // 128, 1, K // 128, 1, device="cuda", generator=g)).repeat_interleave(
        128, 1).repeat_interleave(128, 3).reshape(N, K).bfloat16()
    x = torch.randn(64 + 128, K, device="cuda", generator=g).bfloat16()
    return rt.Fp8Weight.quantize(w), x


@pytest.mark.parametrize("T,K,N", CASES)
def test_fp8_linear_vs_dequantized_reference(T, K, N):
    w8, xs = _weights(N, K, seed=T * 7 + N)
    x = xs[:T]
    out = rt.linear_fp8(x, w8)
    assert out.shape == (T, N) and out.dtype == torch.bfloat16
    wd = w8.dequantize()                       # the reference's dequantized bf16 weight
    ref = x.float() @ wd.float().t()
    got = out.float()
    assert torch.isfinite(got).all()
    scale = ref.pow(2).mean().sqrt().item()
    np.testing.assert_allclose(got.cpu().numpy(), ref.cpu().numpy(), rtol=1e-2, atol=1e-2 * scale)
    # the same bf16 operand, fp32 accumulation, one rounding: nearly every output equals the
    # once-rounded fp32 product of the dequantized weight
    same = (out == ref.bfloat16()).float().mean().item()
    assert same > 0.97, same
    # within bf16 GEMM noise of the reference's own route (cuBLAS on the dequantized weight)
    np.testing.assert_allclose(got.cpu().numpy(), torch.nn.functional.linear(x, wd).float().cpu().numpy(),
                               rtol=2e-2, atol=2e-2 * scale)
    assert torch.equal(rt.linear_fp8(x, w8), out)            # split partials in a fixed order
    from mllm_b200 import abi
    assert abi.load().mllm_attn_device_status(None) == 0      # no wait gave up, no misaligned launch
    wsb = rt._LINEAR_WS.get((x.device, torch.cuda.current_stream().cuda_stream))
    if wsb is not None:
        assert int(wsb[:4096].view(torch.int32).abs().sum()) == 0


def test_fp8_decoder_matches_its_dequantized_model():
    """serving.DecoderModel with FP8 projections (q/k/v/o and the MLP through linear_fp8) against
    the same model dequantized the reference's way: prefill then decode logits within bf16
    tolerance, greedy tokens equal except at near-ties."""
    from mllm_b200 import serving
    shape = serving.DecoderShape(vocab=2048, hidden=1024, layers=3, heads=8, kv_heads=2, head_dim=128,
                                 intermediate=2816)
    m8 = serving.DecoderModel(shape, seed=4, fp8=True)
    md = m8.dequantized()
    g = torch.Generator(device="cuda").manual_seed(6)
    ids = torch.randint(0, shape.vocab, (4, 40), device="cuda", generator=g)
    outs = []
    for m in (m8, md):
        caches = [rt.KVCache(4, shape.kv_heads, shape.head_dim, 64) for _ in range(shape.layers)]
        logits = [m.forward(ids, torch.arange(40, device="cuda"), caches)]
        for k in range(6):
            # both models are fed the FP8 model's greedy tokens
            nxt = outs[0][k].argmax(-1, keepdim=True) if outs else logits[-1].argmax(-1, keepdim=True)
            logits.append(m.forward(nxt, torch.full((4,), 40 + k, device="cuda"), caches))
        outs.append(logits)
    for k, (a, b) in enumerate(zip(*outs)):
        rng = (b.max() - b.min()).item()
        np.testing.assert_allclose(a.cpu().numpy(), b.cpu().numpy(), rtol=0, atol=0.03 * rng,
                                   err_msg=f"step {k}")
