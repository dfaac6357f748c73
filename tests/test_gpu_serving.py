"""Continuous batching on the GPU: requests of mixed prompt lengths (prefill alone into a paged
row, then shared fused decode steps with per-sequence lengths and positions, rows compacted as
requests finish) against each request run alone through contiguous KV caches, teacher-forced on
the batch's tokens.  The logits agree to bf16 tolerance and the greedy choice agrees wherever the
solo run's top-2 margin is not a near-tie."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("needs a GPU", allow_module_level=True)

from mllm_b200 import runtime as rt  # noqa: E402
from mllm_b200.serving import ContinuousBatcher, DecoderModel, DecoderShape  # noqa: E402


def _solo_logits(model, prompt, tokens):
    s = model.s
    caches = [rt.KVCache(1, s.kv_heads, s.head_dim, len(prompt) + len(tokens) + 1) for _ in model.layers]
    dev = model.embed.device
    out = [model.forward(torch.tensor([prompt], device=dev), torch.arange(len(prompt), device=dev), caches)[0]]
    for k, t in enumerate(tokens[:-1]):
        pos = torch.tensor([len(prompt) + k], device=dev)
        out.append(model.forward(torch.tensor([[t]], device=dev), pos, caches)[0])
    return torch.stack(out).float().cpu()


@pytest.mark.parametrize("qk_norm", [True, False])
def test_batched_generation_matches_solo_runs(qk_norm):
    shape = DecoderShape(vocab=2048, hidden=1024, layers=3, heads=8, kv_heads=2, head_dim=128,
                         intermediate=2048, qk_norm=qk_norm)
    model = DecoderModel(shape, seed=3)
    rng = np.random.default_rng(7)
    specs = [(int(p), int(n)) for p, n in [(5, 12), (130, 5), (37, 20), (300, 8), (1, 16), (64, 10), (257, 6)]]
    bat = ContinuousBatcher(model, max_batch=3, num_blocks=10, block_size=128, record_logits=True)
    prompts = {}
    for plen, n in specs:
        prompt = rng.integers(0, shape.vocab, plen).tolist()
        prompts[bat.submit(prompt, n)] = prompt
    out = bat.run()
    assert bat.steps > 0
    for c in bat.caches:
        assert c.free_blocks == 10
    agree = total = 0
    for rid, toks in out.items():
        r = bat.done[rid]
        assert len(toks) == r.max_new_tokens
        got = torch.stack(r.logits)
        ref = _solo_logits(model, prompts[rid], toks)
        scale = ref.abs().max().item()
        np.testing.assert_allclose(got.numpy(), ref.numpy(), atol=0.03 * scale, rtol=0,
                                   err_msg=f"request {rid}")
        top2 = ref.topk(2, dim=-1).values
        clear = (top2[:, 0] - top2[:, 1]) > 0.02 * scale
        agree += int((ref.argmax(-1) == torch.tensor(toks))[clear].sum())
        total += int(clear.sum())
    assert total > 0 and agree == total


def test_decode_graphs_match_eager_steps():
    """The same requests with the decode step replayed from CUDA graphs (one per batch size,
    recorded when a size repeats) and run eagerly: the logits agree to bf16 tolerance up to the
    first differing token, which may only fall on a near-tie, and every block comes back."""
    shape = DecoderShape(vocab=2048, hidden=1024, layers=3, heads=8, kv_heads=2, head_dim=128,
                         intermediate=2048)
    model = DecoderModel(shape, seed=5)
    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, shape.vocab, int(p)).tolist() for p in (20, 200, 3, 129, 64, 7)]
    news = [30, 25, 40, 12, 33, 9]
    runs = {}
    for graphs in (False, True):
        bat = ContinuousBatcher(model, max_batch=4, num_blocks=16, block_size=128, record_logits=True,
                                graphs=graphs)
        ids = [bat.submit(p, n) for p, n in zip(prompts, news)]
        out = bat.run()
        runs[graphs] = ([out[i] for i in ids], [torch.stack(bat.done[i].logits) for i in ids], bat.graph_steps)
        assert all(c.free_blocks == 16 for c in bat.caches)
    assert runs[False][2] == 0 and runs[True][2] > 10
    compared = 0
    for toks_e, toks_g, le, lg in zip(runs[False][0], runs[True][0], runs[False][1], runs[True][1]):
        scale = le.abs().max().item()
        for k in range(min(len(toks_e), len(toks_g))):
            np.testing.assert_allclose(lg[k].numpy(), le[k].numpy(), atol=0.03 * scale, rtol=0)
            compared += 1
            if toks_e[k] != toks_g[k]:
                top2 = le[k].topk(2).values
                assert float(top2[0] - top2[1]) < 0.02 * scale   # a near-tie
                break
    assert compared > 100
