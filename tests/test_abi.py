"""The C-ABI library loads and exports exactly what include/mllm_attn.h declares.  CPU only:
no compute call is made without a GPU (argument validation runs on the host)."""
import ctypes as C
import subprocess

import pytest

from mllm_b200 import abi, build


@pytest.fixture(scope="module")
def lib():
    build.build()
    return abi.load()


def test_header_and_binding_agree():
    assert abi.header_functions() == sorted(abi.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", build.lib_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    declared = set(abi.header_functions())
    assert declared <= exported
    # nothing else leaks out of the library (the CUDA runtime is linked statically and hidden)
    assert {s for s in exported if s.startswith("mllm_")} == declared


def test_status_strings(lib):
    assert lib.mllm_attn_abi_version() == 6
    for code in abi.STATUS_NAMES:
        assert lib.mllm_attn_status_string(code)
    assert lib.mllm_attn_status_string(99) == b"unknown status"


def test_host_side_argument_validation(lib):
    # head_dim must be even (RoPE.h:34-37) -- rejected before any device call
    st = lib.mllm_rope_build_cos_sin(None, 4, 7, 1e4, None, None, None)
    assert st == 1 and b"even" in lib.mllm_attn_last_error()
    # num_heads % num_kv_heads (Attention.h:139-144)
    st = lib.mllm_decode_attention_bf16(None, None, None, 0, 0, 0, None, 1, 6, 4, 128, 16, 0.1, None,
                                        None, 0, None)
    assert st == 1 and b"divisible" in lib.mllm_attn_last_error()
    st = lib.mllm_prefill_attention_bf16(None, None, None, 0, 0, 0, 1, 6, 4, 128, 1, 1, 0.1, None, None)
    assert st == 1
    # unsupported head_dim
    st = lib.mllm_decode_attention_bf16(None, None, None, 0, 0, 0, None, 1, 8, 2, 96, 16, 0.1, None,
                                        None, 0, None)
    assert st == 2
    # GQA group above 8 is reported as unsupported
    st = lib.mllm_decode_attention_bf16(None, None, None, 0, 0, 0, None, 1, 32, 2, 128, 16, 0.1, None,
                                        None, 0, None)
    assert st == 2
    # fused decode step: the decode checks plus the epilogue's pairing rules
    def step(H, Hkv, D, q_norm=None, k_norm=None, theta=1e6):
        return lib.mllm_decode_step_bf16(None, 0, 0, None, 0, 0, None, 0, 0, None, 0, theta, None, None, 0,
                                         q_norm, k_norm, 1e-6, None, None, 0, 0, 0, None, 1, H, Hkv, D, 16, 0.1,
                                         None, None, 0, None)
    assert step(6, 4, 128) == 1 and b"divisible" in lib.mllm_attn_last_error()
    assert step(8, 2, 96) == 2
    assert step(8, 2, 128, q_norm=1) == 1 and b"norm weights" in lib.mllm_attn_last_error()
    assert step(8, 2, 128, theta=0.0) == 1 and b"positions" in lib.mllm_attn_last_error()


def test_linear_argument_validation(lib):
    """mllm_linear_bf16 rejects unsupported shapes before touching the device."""
    w = (C.c_void_p * 2)(16, 16)
    ws = (C.c_int64 * 2)(4096, 4096)

    def call(tokens=32, K=4096, n=(4096, 1024), nw=2):
        nf = (C.c_int64 * 2)(*n)
        return lib.mllm_linear_bf16(16, K, tokens, K, nw, w, ws, nf, 16, 8192, None, 0, None)
    assert call(tokens=257) == 1 and b"tokens" in lib.mllm_attn_last_error()
    assert call(nw=0) == 1 and call(nw=5) == 1
    assert call(K=200) == 1 and b"multiple of 64" in lib.mllm_attn_last_error()
    assert call(n=(4096, 1000)) == 1 and b"multiple of 128" in lib.mllm_attn_last_error()
    assert call(tokens=0) == 0          # nothing to do, no device needed
    # workspace: the partials of a split tile plus one counter per tile (148 SMs assumed here)
    nf = (C.c_int64 * 3)(4096, 1024, 1024)
    size = lib.mllm_linear_workspace_size(32, 3, nf, 4096)
    assert size >= 48 * 2 * 32 * 128 * 4 and size % 4 == 0
    assert lib.mllm_linear_workspace_size(300, 3, nf, 4096) == 0       # invalid -> 0


def test_decode_plan_argument_validation(lib):
    r, c, n = C.c_int(), C.c_int(), C.c_int()
    assert lib.mllm_decode_attention_plan(0, 32, 8, 128, 4096, C.byref(r), C.byref(c), C.byref(n)) == 1
    assert lib.mllm_decode_attention_plan(32, 30, 8, 128, 4096, None, None, None) == 1
    assert lib.mllm_decode_attention_plan(32, 32, 8, 96, 4096, None, None, None) == 1


def test_workspace_size(lib):
    ws = lib.mllm_decode_attention_workspace_size(32, 32, 8, 128, 4096)
    assert ws > 0 and ws % 256 == 0
    assert lib.mllm_decode_attention_workspace_size(0, 32, 8, 128, 4096) == 0
    assert lib.mllm_decode_attention_workspace_size(32, 30, 8, 128, 4096) == 0


def test_no_device_is_reported(lib):
    """In this container there is no GPU: a well-formed call reports NO_DEVICE (or a CUDA error),
    it never silently succeeds."""
    buf = (C.c_int64 * 4)()
    st = lib.mllm_rope_build_cos_sin(C.addressof(buf), 4, 8, 1e4, C.addressof(buf), C.addressof(buf), None)
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if not has_gpu:
        assert st in (3, 5)


def test_varlen_argument_validation(lib):
    """The packed-sequence entry points reject inconsistent sizes and missing arrays on the host;
    an empty packed batch needs no device."""
    kv = abi.PagedKV(16, 16, 8 * 256 * 128, 256 * 128, 128, 4, 256, 16, 4, 4)
    cu, lens = 32, 48                    # stand-in device addresses, never dereferenced here

    def attn(cu_=cu, lens_=lens, batch=2, H=8, Hkv=2, D=128, total=10, max_q=8, kvp=kv):
        return lib.mllm_prefill_attention_varlen_paged_bf16(16, C.byref(kvp), cu_, lens_, batch, H, Hkv, D, total,
                                                            max_q, 0.1, 16, None)
    assert attn(cu_=None) == 1 and b"cu_q_lens" in lib.mllm_attn_last_error()
    assert attn(lens_=None) == 1 and b"kv_lens" in lib.mllm_attn_last_error()
    assert attn(total=17) == 1 and b"max_q_len" in lib.mllm_attn_last_error()   # 17 rows > 2 x 8
    assert attn(H=6, Hkv=4) == 1 and b"divisible" in lib.mllm_attn_last_error()
    assert attn(D=96) == 2
    bad = abi.PagedKV(16, 16, 8 * 256 * 128, 256 * 128, 128, 4, 100, 16, 4, 4)   # block_size % 128
    assert attn(kvp=bad) == 1 and b"block_size" in lib.mllm_attn_last_error()
    assert attn(total=0) == 0            # no rows: nothing to launch
    st = lib.mllm_prefill_attention_varlen_bf16(16, 16, 16, 0, 0, 0, 0, cu, lens, 2, 8, 2, 128, 10, 8, 0.1, 16,
                                                None)
    assert st == 1 and b"cache_capacity" in lib.mllm_attn_last_error()

    def epi(cu_=cu, pos=64, batch=2, total=10, qn=None, kn=None):
        return lib.mllm_qkv_epilogue_varlen_paged_bf16(16, 1536, 128, 16, 1536, 128, 16, 1536, 128, total, 8, 2,
                                                       128, pos, 1e6, qn, kn, 1e-6, 16, C.byref(kv), cu_, batch,
                                                       None, None)
    assert epi(cu_=None) == 1 and b"cu_seqlens" in lib.mllm_attn_last_error()
    assert epi(pos=None) == 1
    assert epi(batch=0) == 1
    assert epi(qn=16) == 1 and b"norm weights" in lib.mllm_attn_last_error()
    assert epi(total=0, cu_=None, batch=0) == 0


def test_linear_fp8_argument_validation(lib):
    """mllm_linear_fp8_bf16 rejects unsupported shapes on the host, before any device call."""
    def call(tokens=32, K=4096, N=4096, wstride=4096):
        return lib.mllm_linear_fp8_bf16(16, K, tokens, K, 16, wstride, N, 16, K // 128, 16, N, None, 0, None)
    assert call(tokens=129) == 1 and b"tokens" in lib.mllm_attn_last_error()
    assert call(K=4160) == 1 and b"multiple of 128" in lib.mllm_attn_last_error()
    assert call(N=4000) == 1 and b"multiple of 128" in lib.mllm_attn_last_error()
    assert call(wstride=4000) == 1
    assert call(tokens=0) == 0          # nothing to do, no device needed
    assert lib.mllm_linear_fp8_workspace_size(129, 4096, 4096) == 0
