"""The device sampler (mllm_sample, Sampler.cpp:49-232) through the C ABI: the greedy branch with
the repetition penalty bit-exact against the compiled reference's fixture and the oracle, and
the sampling branch checked by its distribution.  Needs a B200."""
import math
import os

import numpy as np
import pytest

from oracle import sampler_oracle as SO
from tests.golden.cases import GOLDEN_DIR, SAMPLER_PENALTIES, make_sampler_inputs

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def rt(cuda_device):
    from mllm_b200 import build
    build.build()
    from mllm_b200 import runtime
    return runtime


@pytest.mark.parametrize("dn", ["bf16", "f32"])
@pytest.mark.parametrize("pen", SAMPLER_PENALTIES)
def test_greedy_with_penalty_matches_reference_fixture(rt, dn, pen):
    """The four fixture rows as one batch: tokens and the in-place penalised logits, bit for bit."""
    g = np.load(os.path.join(GOLDEN_DIR, "sampler.npz"))
    logits, hist = make_sampler_inputs()
    dt = torch.bfloat16 if dn == "bf16" else torch.float32
    x = torch.from_numpy(logits).to(dt).cuda()
    tok = rt.sample(x, 1.0, 0, 1.0, True, hist, pen).cpu().numpy()
    for r in range(4):
        tag = f"{dn}_p{int(pen * 10)}_r{r}"
        assert tok[r] == int(g["token_" + tag]), tag
        np.testing.assert_array_equal(x[r].float().cpu().numpy().view(np.uint32),
                                      g["logits_" + tag].view(np.uint32), err_msg=tag)


def test_greedy_full_vocab_long_history(rt):
    """Qwen3 vocabulary (151936), 2 rows, 5000-token histories with repeats, penalty 1.2."""
    rng = np.random.default_rng(3)
    V = 151936
    logits = SO.round_bf16((rng.standard_normal((2, V)) * 2).astype(np.float32))
    hist = [[int(t) for t in rng.integers(0, V, 5000)], [int(t) for t in rng.integers(0, 64, 5000)]]
    x = torch.from_numpy(logits).bfloat16().cuda()
    tok = rt.sample(x, 0.0, 0, 1.0, False, hist, 1.2).cpu().numpy()   # temperature <= 0: greedy
    for r in range(2):
        t_ref, x_ref = SO.sample_greedy(logits[r], hist[r], 1.2, "bf16")
        assert tok[r] == t_ref
        np.testing.assert_array_equal(x[r].float().cpu().numpy().view(np.uint32), x_ref.view(np.uint32))


def _expected(logits, temperature, top_k, top_p):
    """The reference's sampling distribution (Sampler.cpp:142-222) in fp64, distinct logits."""
    z = logits.astype(np.float64) / temperature
    p = np.exp(z - z.max())
    p /= p.sum()
    order = np.argsort(-p)
    if 0 < top_k < len(p):
        keep = np.zeros_like(p, dtype=bool)
        keep[order[:top_k]] = True
        p = np.where(keep, p, 0.0)
        p /= p.sum()
    if top_p < 1.0:
        cum = np.cumsum(p[order])
        remove = cum > top_p
        remove[0] = False
        q = p.copy()
        q[order[remove]] = 0.0
        p = q / q.sum()
    return p


@pytest.mark.parametrize("temperature,top_k,top_p", [(0.7, 0, 1.0), (1.0, 10, 1.0), (0.9, 0, 0.8), (1.3, 12, 0.7)])
def test_sampling_distribution(rt, temperature, top_k, top_p):
    """20000 draws (one per batch row, the same logits) follow the reference's filtered
    distribution: nothing outside the kept set, every frequency within 5 standard deviations."""
    V, N = 50, 20000
    rng = np.random.default_rng(int(temperature * 100) + top_k)
    row = SO.round_bf16(np.linspace(-2.45, 2.45, V).astype(np.float32))[rng.permutation(V)]   # distinct in bf16
    assert len(np.unique(row)) == V
    x = torch.from_numpy(np.tile(row, (N, 1))).float().cuda()
    tok = rt.sample(x, temperature, top_k, top_p, False, None, 1.0, seed=1234, offset=7).cpu().numpy()
    p = _expected(row, temperature, top_k, top_p)
    freq = np.bincount(tok, minlength=V) / N
    assert (freq[p == 0] == 0).all(), "sampled a filtered token"
    sigma = np.sqrt(np.maximum(p * (1 - p) / N, 1e-12))
    assert (np.abs(freq - p) <= 5 * sigma + 1e-4).all(), np.max(np.abs(freq - p) / sigma)
    # another offset gives other draws, the same offset the same ones
    tok2 = rt.sample(x, temperature, top_k, top_p, False, None, 1.0, seed=1234, offset=8).cpu().numpy()
    tok3 = rt.sample(x, temperature, top_k, top_p, False, None, 1.0, seed=1234, offset=7).cpu().numpy()
    assert (tok2 != tok).any() and (tok3 == tok).all()


def test_reference_argument_errors(rt):
    x = torch.zeros(1, 8, device="cuda")
    with pytest.raises(RuntimeError, match="temperature must be finite"):
        rt.sample(x, math.inf)
    with pytest.raises(RuntimeError, match=r"top_p must be in \(0, 1\]"):
        rt.sample(x, 1.0, 0, 0.0)
    assert int(rt.sample(x, 1.0, 0, 5.0, True).item()) == 0   # top_p above 1 is clamped; ties: index 0
