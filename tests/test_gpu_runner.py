"""The drop-in headers under the reference's UNCHANGED QwenRunner (ModelRunnerFactory ->
QwenRunner::Load -> Forward / Generate), against the same runner built on the reference's own
runtime headers, on one random-init Qwen3 checkpoint.  Both run on the GPU (the reference
moves its weights to CUDA itself, QwenRunner.cpp:231-281).  Needs a B200 and the two runner
modules built by mllm_b200/dropin/build_facade.py (in the build container)."""
import importlib.util
import os

import numpy as np
import pytest

from tests.helpers import ATOL, RTOL
from tests.qwen_model import QwenShape, write_random_qwen3

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TINY = QwenShape(layers=3, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024, vocab=1024)


def _load(path, name):
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build it with mllm_b200/dropin/build_facade.py")
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def runners(tmp_path_factory, cuda_device):
    from mllm_b200 import build
    build.build()
    from mllm_b200.dropin.build_facade import runner_module_path
    ref_mod = _load(runner_module_path("reference"), "mllm_ref_runner")
    new_mod = _load(runner_module_path("dropin"), "mllm_dropin_runner")
    path = str(tmp_path_factory.mktemp("qwen3_tiny"))
    write_random_qwen3(path, TINY, seed=3)
    return ref_mod.Runner(path), new_mod.Runner(path)


def _close(a, b, what):
    np.testing.assert_allclose(a.float().cpu().numpy(), b.float().cpu().numpy(), rtol=RTOL, atol=ATOL,
                               err_msg=what)


def test_prefill_then_teacher_forced_decode(runners):
    """Batch 2: the prefill logits for all positions, then 12 decode steps fed the reference's
    greedy tokens; the runner itself decides prefill vs decode (S == 1 with a cache)."""
    ref, new = runners
    ref.reset_cache()
    new.reset_cache()
    rng = np.random.default_rng(5)
    ids = torch.from_numpy(rng.integers(0, TINY.vocab, size=(2, 37))).long()
    lr = ref.forward(ids)
    ln = new.forward(ids)
    assert lr.shape == ln.shape == (2, 37, TINY.vocab)
    _close(ln, lr, "prefill logits")
    for step in range(12):
        nxt = lr[:, -1].float().argmax(-1, keepdim=True).cpu()
        lr = ref.forward(nxt)
        ln = new.forward(nxt)
        assert ln.shape == (2, 1, TINY.vocab)
        _close(ln, lr, f"decode step {step}")


def test_generate_greedy_tokens(runners):
    """IModelRunner::Generate (batch 1, greedy, the reference's own loop and Sampler): tokens
    identical to the reference runner's, or -- where random weights leave a near-tie -- the two
    diverge only at a step whose top-2 logit margin is within bf16 noise."""
    ref, new = runners
    prompt = list(np.random.default_rng(9).integers(0, TINY.vocab, size=23))
    t_ref = ref.generate(prompt, 24)
    t_new = new.generate(prompt, 24)
    assert len(t_ref) == len(t_new) == 24
    if t_ref != t_new:
        k = next(i for i, (a, b) in enumerate(zip(t_ref, t_new)) if a != b)
        ref.reset_cache()
        logits = ref.forward(torch.tensor([prompt + t_ref[:k]]))[0, -1].float()
        top2 = torch.topk(logits, 2).values
        assert (top2[0] - top2[1]).item() < 0.05, f"diverged at step {k} with a clear margin"


def test_generate_greedy_with_repetition_penalty(runners):
    """The same with the repetition penalty (1.3): the drop-in Sampler penalises on the device
    (mllm_sample) what the reference penalises one .item() at a time."""
    from oracle import sampler_oracle as SO
    ref, new = runners
    prompt = list(np.random.default_rng(11).integers(0, TINY.vocab, size=19))
    t_ref = ref.generate(prompt, 24, 1.3)
    t_new = new.generate(prompt, 24, 1.3)
    assert len(t_ref) == len(t_new) == 24
    if t_ref != t_new:
        k = next(i for i, (a, b) in enumerate(zip(t_ref, t_new)) if a != b)
        ref.reset_cache()
        ctx = prompt + t_ref[:k]
        logits = ref.forward(torch.tensor([ctx]))[0, -1].float().cpu().numpy()
        pen = SO.apply_repetition_penalty(logits, ctx, 1.3, "bf16")
        top2 = np.sort(pen)[-2:]
        assert top2[1] - top2[0] < 0.05, f"diverged at step {k} with a clear margin"


def test_decode_graphs_match_eager(runners, monkeypatch):
    """MLLM_B200_DECODE_GRAPHS=1: every decode layer replays a CUDA graph recorded on its second
    decode call.  Against the same drop-in runner stepping kernel by kernel, on the eager run's
    tokens: logits within bf16 tolerance at every step, again after InitKVCache (every layer is
    recorded anew), and Generate's tokens across two calls (its Clear() keeps the graphs)."""
    _, new = runners
    rng = np.random.default_rng(13)
    ids = torch.from_numpy(rng.integers(0, TINY.vocab, size=(2, 41))).long()

    def run(graphs, toks=None):
        monkeypatch.setenv("MLLM_B200_DECODE_GRAPHS", "1" if graphs else "0")
        new.reset_cache()
        out = [new.forward(ids)[:, -1].float().cpu()]
        picked = []
        for k in range(10):
            nxt = out[-1].argmax(-1, keepdim=True) if toks is None else toks[:, k:k + 1]
            picked.append(nxt)
            out.append(new.forward(nxt)[:, -1].float().cpu())
        return torch.stack(out, 1), torch.cat(picked, 1)

    eager, toks = run(False)
    for rep in range(2):                       # the second pass follows an InitKVCache
        graphed, _ = run(True, toks)
        _close(graphed, eager, f"graph pass {rep}")
    prompt = list(rng.integers(0, TINY.vocab, size=17))
    monkeypatch.setenv("MLLM_B200_DECODE_GRAPHS", "0")
    t_eager = new.generate(prompt, 20)
    monkeypatch.setenv("MLLM_B200_DECODE_GRAPHS", "1")
    t1 = new.generate(prompt, 20)
    t2 = new.generate(prompt, 20)
    assert t1 == t2
    if t1 != t_eager:
        k = next(i for i, (a, b) in enumerate(zip(t1, t_eager)) if a != b)
        new.reset_cache()
        logits = new.forward(torch.tensor([prompt + t_eager[:k]]))[0, -1].float()
        top2 = torch.topk(logits, 2).values
        assert (top2[0] - top2[1]).item() < 0.05, f"diverged at step {k} with a clear margin"
