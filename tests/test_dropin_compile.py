"""The reference's UNCHANGED model runners compile against the drop-in runtime headers.

Needs the reference tree (present only where the fixtures are built), so it skips elsewhere.
Compiling QwenRunner.cpp / LlamaRunner.cpp proves the drop-in keeps every class, member and
signature the runners use (KVCache::key/value/IsInitialized/Clear, LayerWeights fields,
TransformerBlock::Forward, Attention::*, RoPE::*)."""
import os

import pytest

from mllm_b200.dropin import build_facade


@pytest.mark.skipif(not os.path.isdir(os.path.join(build_facade.REFERENCE, "src", "models")),
                    reason="reference tree not present")
@pytest.mark.timeout(900)
def test_reference_runners_compile_against_dropin_headers():
    objs = build_facade.check_runners()
    assert all(os.path.getsize(o) > 0 for o in objs)
