"""ctypes binding of the C ABI in include/mllm_attn.h (libmllm_attn.so).

This is the same binding a Python caller of the reference runtime would add; the C++ drop-in
facade (mllm_b200/runtime/core/runtime/*.h) calls the identical entry points.  Tensors are
passed as raw device pointers (`tensor.data_ptr()`), sizes and strides in elements.

There is no CPU fallback: loading fails loudly when the library has not been built, and every
entry point rejects a non-sm_100 device with MLLM_ERR_NO_DEVICE.
"""
from __future__ import annotations

import ctypes as C
import os
import re

from .build import lib_path

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mllm_attn.h")

MLLM_OK = 0
STATUS_NAMES = {
    0: "MLLM_OK", 1: "MLLM_ERR_INVALID_ARGUMENT", 2: "MLLM_ERR_UNSUPPORTED", 3: "MLLM_ERR_CUDA",
    4: "MLLM_ERR_WORKSPACE", 5: "MLLM_ERR_NO_DEVICE", 6: "MLLM_ERR_DEVICE_TIMEOUT",
    7: "MLLM_ERR_DEVICE_LENGTH", 8: "MLLM_ERR_COMM", 9: "MLLM_ERR_COMM_TIMEOUT",
}

_i = C.c_int
_i64 = C.c_int64
_p = C.c_void_p
_d = C.c_double
_f = C.c_float
_sz = C.c_size_t



class PagedKV(C.Structure):
    """struct mllm_paged_kv (include/mllm_attn.h): a paged KV cache's pools and block table."""
    _fields_ = [("k_pool", C.c_void_p), ("v_pool", C.c_void_p), ("block_stride", C.c_int64),
                ("head_stride", C.c_int64), ("row_stride", C.c_int64), ("num_blocks", C.c_int32),
                ("block_size", C.c_int32), ("block_table", C.c_void_p), ("table_stride", C.c_int64),
                ("max_blocks_per_seq", C.c_int32)]


_kv = C.POINTER(PagedKV)

# name -> (restype, argtypes); mirrors include/mllm_attn.h one to one
SIGNATURES = {
    "mllm_attn_abi_version": (_i, []),
    "mllm_attn_status_string": (C.c_char_p, [_i]),
    "mllm_attn_last_error": (C.c_char_p, []),
    "mllm_attn_device_status": (_i, [_p]),
    "mllm_rope_build_cos_sin": (_i, [_p, _i64, _i, _d, _p, _p, _p]),
    "mllm_rope_apply_bf16": (_i, [_p, _i64, _i64, _i64, _i, _i, _i, _i, _p, _p, _p, _p]),
    "mllm_qkv_epilogue_bf16": (_i, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                    _i, _i, _i, _i, _i, _p, _i64, _i64, _d, _p, _p, _i64, _i64,
                                    _p, _p, _d, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i64, _p]),
    "mllm_prefill_attention_bf16": (_i, [_p, _p, _p, _i64, _i64, _i64, _i, _i, _i, _i, _i, _i, _f, _p, _p]),
    "mllm_decode_attention_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "mllm_decode_attention_plan": (_i, [_i, _i, _i, _i, _i, C.POINTER(C.c_int), C.POINTER(C.c_int),
                                        C.POINTER(C.c_int)]),
    "mllm_decode_attention_bf16": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _i, _i, _i, _i, _i, _f, _p,
                                        _p, _sz, _p]),
    "mllm_decode_attention_noalloc_bf16": (_i, [_p, _p, _p, _i64, _i64, _i64, _p, _i, _i, _i, _i, _i, _f,
                                                _p, _p]),
    "mllm_decode_step_bf16": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _d, _p, _p, _i64,
                                   _p, _p, _d, _p, _p, _i64, _i64, _i64, _p, _i, _i, _i, _i, _i, _f, _p, _p,
                                   _sz, _p]),
    "mllm_qkv_epilogue_paged_bf16": (_i, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64,
                                          _i, _i, _i, _i, _i, _p, _i64, _i64, _d, _p, _p, _i64, _i64,
                                          _p, _p, _d, _p, _kv, _p, _i64, _p]),
    "mllm_prefill_attention_paged_bf16": (_i, [_p, _kv, _i, _i, _i, _i, _i, _i, _f, _p, _p]),
    "mllm_decode_attention_paged_bf16": (_i, [_p, _kv, _p, _i, _i, _i, _i, _i, _f, _p, _p, _sz, _p]),
    "mllm_decode_step_paged_bf16": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _p, _i64, _d, _p, _p,
                                         _i64, _p, _p, _d, _kv, _p, _i, _i, _i, _i, _i, _f, _p, _p, _sz, _p]),
    "mllm_qkv_epilogue_varlen_bf16": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i, _i, _i, _i, _p, _d,
                                           _p, _p, _d, _p, _p, _p, _i64, _i64, _i64, _i64, _p, _i, _p, _p]),
    "mllm_qkv_epilogue_varlen_paged_bf16": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _i64, _i64, _i, _i, _i, _i,
                                                 _p, _d, _p, _p, _d, _p, _kv, _p, _i, _p, _p]),
    "mllm_prefill_attention_varlen_bf16": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _p, _p, _i, _i, _i, _i, _i,
                                                _i, _f, _p, _p]),
    "mllm_prefill_attention_varlen_paged_bf16": (_i, [_p, _kv, _p, _p, _i, _i, _i, _i, _i, _i, _f, _p, _p]),
    "mllm_linear_workspace_size": (_sz, [_i, _i, C.POINTER(C.c_int64), _i64]),
    "mllm_linear_bf16": (_i, [_p, _i64, _i, _i64, _i, C.POINTER(C.c_void_p), C.POINTER(C.c_int64),
                              C.POINTER(C.c_int64), _p, _i64, _p, _sz, _p]),
    "mllm_linear_fp8_workspace_size": (_sz, [_i, _i64, _i64]),
    "mllm_linear_fp8_bf16": (_i, [_p, _i64, _i, _i64, _p, _i64, _i64, _p, _i64, _p, _i64, _p, _sz, _p]),
    "mllm_ipc_alloc": (_i, [_sz, C.POINTER(C.c_void_p)]),
    "mllm_ipc_free": (_i, [_p]),
    "mllm_ipc_get_handle": (_i, [_p, _p]),
    "mllm_ipc_open_handle": (_i, [_p, C.POINTER(C.c_void_p)]),
    "mllm_ipc_close_handle": (_i, [_p]),
    "mllm_copy_async": (_i, [_p, _p, _sz, _p]),
    "mllm_signal_u32": (_i, [_p, C.c_uint32, _p]),
    "mllm_wait_u32": (_i, [_p, C.c_uint32, _p]),
    "mllm_wait_u32_timeout": (_i, [_p, C.c_uint32, C.c_uint32, _p]),
    "mllm_sum_bf16": (_i, [C.POINTER(C.c_void_p), _i, C.POINTER(C.c_void_p), _i, _i64, _p]),
    "mllm_comm_unique_id": (_i, [_p]),
    "mllm_comm_init": (_i, [_p, _i, _i, _d, C.POINTER(C.c_void_p)]),
    "mllm_comm_all_reduce_bf16": (_i, [_p, _p, _p, _sz, _p]),
    "mllm_comm_all_gather_bf16": (_i, [_p, _p, _p, _sz, _p]),
    "mllm_comm_status": (_i, [_p]),
    "mllm_comm_in_flight": (_i, [_p]),
    "mllm_comm_abort": (_i, [_p]),
    "mllm_comm_destroy": (_i, [_p]),
    "mllm_sample_workspace_size": (_sz, [_i, _i]),
    "mllm_sample": (_i, [_p, _i, _i64, _i, _i, _p, _i64, _p, _f, _i, _f, _i, _f, C.c_uint64, C.c_uint64, _p, _p,
                         _sz, _p]),
}


class MllmError(RuntimeError):
    """A nonzero mllm_status; `.status` holds the code."""

    def __init__(self, status: int, fn: str, detail: str):
        self.status = status
        super().__init__(f"{fn}: {STATUS_NAMES.get(status, status)}: {detail}")


_lib = None


def load(path: str | None = None) -> C.CDLL:
    """Load libmllm_attn.so (built by `python -m mllm_b200.build`).  Raises if absent."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or lib_path()
    if not os.path.exists(p):
        raise RuntimeError(f"{p} is missing: build it with `python -m mllm_b200.build` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def header_functions() -> list[str]:
    """Entry points declared in include/mllm_attn.h."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mllm_[a-z0-9_]+)\s*\(", text)))


def call(name: str, *args) -> int:
    """Call an entry point and raise MllmError on a nonzero status."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != MLLM_OK:
        raise MllmError(st, name, lib.mllm_attn_last_error().decode())
    return st


def stream_handle(stream=None) -> int | None:
    """cudaStream_t of a torch stream (None -> torch's current stream)."""
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream or None
