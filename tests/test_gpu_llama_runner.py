"""The drop-in headers under the reference's UNCHANGED LlamaRunner (ModelRunnerFactory ->
LlamaRunner::Load -> Forward / Generate), on one random-init checkpoint of the TinyLlama attention
geometry (hidden 2048, 32 q heads, 4 kv heads, head_dim 64, RoPE theta 1e4; 2 layers, SwiGLU 1024,
vocab 2048, weights rounded to bf16).

LlamaRunner keeps every weight on the host (LlamaRunner.cpp:111-187): the reference computes on
the CPU, and the drop-in stages each weight on the GPU once and the hidden state per call, runs
the layer there through Attention::Forward (q/k/v projections, then the epilogue + prefill or the
fused decode step), and returns the output to the host.

The yardstick is the reference's fp32 run of the same weights (the checkpoint widened exactly to
fp32).  Through two layers and a 2048-wide lm_head, bf16 itself moves these logits by a few
hundredths -- the reference's own bf16 run is up to about 0.04 away from its fp32 run -- so the
drop-in (bf16) must be no further from the fp32 run than the reference's bf16 run is, in the
largest and in the mean absolute difference, on the prefill of 512 rows and on 64 decode steps
fed the fp32 run's greedy tokens.  Greedy Generate is then compared token by token."""
import importlib.util
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _load(flavor):
    from mllm_b200.dropin.build_facade import runner_module_path
    path = runner_module_path(flavor)
    if not os.path.exists(path):
        pytest.fail(f"{path} missing: build it with mllm_b200/dropin/build_facade.py")
    spec = importlib.util.spec_from_file_location(os.path.basename(path).split(".")[0], path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def runners(tmp_path_factory, cuda_device):
    from mllm_b200 import build
    from tests.qwen_model import TINYLLAMA_LAYER, write_random_llama
    build.build()
    path = str(tmp_path_factory.mktemp("tinyllama"))
    path32 = str(tmp_path_factory.mktemp("tinyllama_f32"))
    write_random_llama(path, TINYLLAMA_LAYER, seed=4)
    write_random_llama(path32, TINYLLAMA_LAYER, seed=4, dtype="f32")
    ref_mod = _load("reference")
    ref, new, ref32 = ref_mod.Runner(path), _load("dropin").Runner(path), ref_mod.Runner(path32)
    assert ref.model_type() == new.model_type() == "llama"
    return ref, new, ref32


def test_llama_prefill_then_decode_within_the_bf16_floor(runners):
    from tests.qwen_model import TINYLLAMA_LAYER
    ref, new, ref32 = runners
    for r in runners:
        r.reset_cache()
    ids = torch.from_numpy(np.random.default_rng(1).integers(0, TINYLLAMA_LAYER.vocab, size=(1, 512))).long()
    l32, lr, ln = ref32.forward(ids).float(), ref.forward(ids).float(), new.forward(ids).float()
    assert l32.shape == lr.shape == ln.shape == (1, 512, TINYLLAMA_LAYER.vocab)
    assert not ln.is_cuda              # the runner's own lm_head runs where it keeps its weights
    e_new, e_ref = [], []
    for step in range(65):
        e_new.append((ln - l32).abs().flatten())
        e_ref.append((lr - l32).abs().flatten())
        if step == 64:
            break
        nxt = l32[:, -1].argmax(-1, keepdim=True)
        # S == 1 over an initialized cache: each runner takes its decode step
        l32, lr, ln = ref32.forward(nxt).float(), ref.forward(nxt).float(), new.forward(nxt).float()
    e_new, e_ref = torch.cat(e_new), torch.cat(e_ref)
    assert torch.isfinite(e_new).all()
    assert float(e_new.max()) <= 1.25 * float(e_ref.max()), (float(e_new.max()), float(e_ref.max()))
    assert float(e_new.mean()) <= 1.25 * float(e_ref.mean()), (float(e_new.mean()), float(e_ref.mean()))


def test_llama_generate_greedy_tokens(runners):
    """IModelRunner::Generate (batch 1, greedy, the reference's own loop; the drop-in Sampler
    samples the host logits on the device): identical tokens, or a divergence only where the
    reference's top-2 margin is within bf16 noise."""
    from tests.qwen_model import TINYLLAMA_LAYER
    ref, new, _ = runners
    prompt = list(np.random.default_rng(3).integers(0, TINYLLAMA_LAYER.vocab, size=40))
    t_ref = ref.generate(prompt, 32)
    t_new = new.generate(prompt, 32)
    assert len(t_ref) == len(t_new) == 32
    if t_ref != t_new:
        k = next(i for i, (a, b) in enumerate(zip(t_ref, t_new)) if a != b)
        ref.reset_cache()
        logits = ref.forward(torch.tensor([prompt + t_ref[:k]]))[0, -1].float()
        top2 = torch.topk(logits, 2).values
        assert (top2[0] - top2[1]).item() < 0.05, f"diverged at step {k} with a clear margin"
