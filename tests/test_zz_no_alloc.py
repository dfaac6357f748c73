"""mllm_decode_attention_noalloc_bf16: decode for callers that cannot allocate device memory.

Callers such as an inference runtime that hands out all device memory from its own arena at
start-up, or code that runs under another framework's allocator, cannot give the decode kernel a
freshly allocated workspace.  The no-alloc entry point keeps its split-K partials in a static
scratch array inside the library instead.  These tests call it through the C ABI and check that
it returns the same bits as the workspace entry point (same kernels, same plan), on two calls in
a row (the second call reuses the scratch left behind by the first), and that an oversized batch
is refused.

This file is collected last on purpose, so a failure here never hides another test.
"""
import math

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def lib(cuda_device):
    from mllm_b200 import abi, build
    build.build()
    return abi.load()


def _problem(B, H, Hkv, D, lens, cap, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Hkv, cap, D, device="cuda", generator=g).bfloat16()
    q = torch.randn(B, H, D, device="cuda", generator=g).bfloat16()
    kv_lens = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, k, v, kv_lens


def _with_workspace(lib, q, k, v, kv_lens, H, Hkv, D, L):
    B = q.shape[0]
    out = torch.empty(B, H * D, dtype=torch.bfloat16, device="cuda")
    nbytes = lib.mllm_decode_attention_workspace_size(B, H, Hkv, D, L)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    st = lib.mllm_decode_attention_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), *k.stride()[:3],
                                        kv_lens.data_ptr(), B, H, Hkv, D, L, 1.0 / math.sqrt(D), out.data_ptr(),
                                        ws.data_ptr(), nbytes, None)
    assert st == 0, lib.mllm_attn_last_error()
    return out


def _no_alloc(lib, q, k, v, kv_lens, H, Hkv, D, L):
    B = q.shape[0]
    out = torch.empty(B, H * D, dtype=torch.bfloat16, device="cuda")
    st = lib.mllm_decode_attention_noalloc_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), *k.stride()[:3],
                                                kv_lens.data_ptr(), B, H, Hkv, D, L, 1.0 / math.sqrt(D),
                                                out.data_ptr(), None)
    assert st == 0, lib.mllm_attn_last_error()
    return out


def test_no_alloc_matches_workspace_entry_point_twice(lib):
    # first call: Qwen3-8B decode geometry, ragged lengths spanning several split-K chunks
    B, H, Hkv, D = 8, 32, 8, 128
    lens = [4096, 1, 777, 2048, 3000, 64, 4095, 1500]
    q, k, v, kv_lens = _problem(B, H, Hkv, D, lens, 4096, seed=21)
    ref1 = _with_workspace(lib, q, k, v, kv_lens, H, Hkv, D, 4096)
    got1 = _no_alloc(lib, q, k, v, kv_lens, H, Hkv, D, 4096)
    torch.cuda.synchronize()
    # the same kernels on the same plan: the outputs must be the same bits
    assert torch.equal(got1, ref1)

    # second call right after: different geometry and data on the same (now dirty) scratch
    B2, H2, Hkv2, D2 = 5, 32, 4, 64
    lens2 = [512, 129, 2000, 33, 1024]
    q2, k2, v2, kv_lens2 = _problem(B2, H2, Hkv2, D2, lens2, 2048, seed=22)
    ref2 = _with_workspace(lib, q2, k2, v2, kv_lens2, H2, Hkv2, D2, 2048)
    got2 = _no_alloc(lib, q2, k2, v2, kv_lens2, H2, Hkv2, D2, 2048)
    torch.cuda.synchronize()
    assert torch.equal(got2, ref2)
    assert lib.mllm_attn_device_status(None) == 0


def test_no_alloc_refuses_batches_beyond_its_scratch(lib):
    # 256 sequences x 8 kv heads x 32768 rows needs far more than the static 16 MiB
    B, H, Hkv, D, L = 256, 32, 8, 128, 32768
    assert lib.mllm_decode_attention_workspace_size(B, H, Hkv, D, L) > (16 << 20)
    dummy = torch.empty(16, dtype=torch.bfloat16, device="cuda")
    st = lib.mllm_decode_attention_noalloc_bf16(dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(),
                                                L * D, L * D * Hkv, D, None, B, H, Hkv, D, L, 0.088,
                                                dummy.data_ptr(), None)
    assert st == 4  # MLLM_ERR_WORKSPACE, refused on the host before any launch
    assert b"static scratch" in lib.mllm_attn_last_error()
