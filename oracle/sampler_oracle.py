"""CPU restatement of the reference sampler's deterministic path (test infrastructure only: the
tests, smoke() and bench.py's CPU leg use it as the checker; the product never calls it).

  Sampler::ApplyRepetitionPenalty  src/core/runtime/Sampler.cpp:12-46
  Sampler::Sample, greedy branch   src/core/runtime/Sampler.cpp:49-140

Pinned against the compiled reference Sampler by tests/golden/sampler.npz
(tests/golden/make_golden.py)."""
from __future__ import annotations

import numpy as np

from oracle.attention_oracle import round_bf16


def apply_repetition_penalty(logits: np.ndarray, previous_tokens, penalty: float, dtype: str = "bf16") -> np.ndarray:
    """Sampler.cpp:12-46 on a copy of one row (float32 array holding values of `dtype`): for every
    history entry in order, a non-negative logit is divided by the penalty and a negative one
    multiplied, in fp32, and the result is written back to the tensor (rounded to its dtype), so
    a repeated token is penalised once per occurrence."""
    x = np.asarray(logits, dtype=np.float32).copy()
    if penalty <= 1.0:
        return x
    p = np.float32(penalty)
    for tok in previous_tokens:
        if tok < 0 or tok >= x.shape[0]:
            continue
        v = x[tok]
        v = np.float32(v * p) if v < 0.0 else np.float32(v / p)
        x[tok] = round_bf16(np.array([v], dtype=np.float32))[0] if dtype == "bf16" else v
    return x


def sample_greedy(logits: np.ndarray, previous_tokens, penalty: float, dtype: str = "bf16"):
    """The greedy branch (Sampler.cpp:128-140): argmax of the penalised row, the first index
    winning ties and NaN above every number (torch::argmax).  Returns (token, penalised row)."""
    x = apply_repetition_penalty(logits, previous_tokens, penalty, dtype)
    nan = np.isnan(x)
    tok = int(np.argmax(nan)) if nan.any() else int(np.argmax(x))
    return tok, x
