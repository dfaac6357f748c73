"""Paged KV cache: the host-side allocator (CPU) and the C ABI's descriptor checks, which run on
the host before any device call."""
import ctypes as C

import pytest
import torch

from mllm_b200 import abi, build
from mllm_b200.runtime import PagedKVCache


def test_allocator_hands_out_and_reclaims_blocks():
    c = PagedKVCache(num_blocks=8, num_kv_heads=2, head_dim=64, block_size=128, max_seqs=3,
                     max_blocks_per_seq=4, device="cpu")
    assert c.capacity == 512 and c.free_blocks == 8
    c.set_lengths([300, 1, 0])
    assert [len(c.blocks_of(b)) for b in range(3)] == [3, 1, 0]
    assert c.free_blocks == 4
    assert c.block_table[0, :3].tolist() == c.blocks_of(0)
    c.k_pool[c.blocks_of(0)[0]].fill_(3.0)
    c.advance([200, 0, 0])           # 500 rows: a fourth block for sequence 0
    assert len(c.blocks_of(0)) == 4 and c.host_lengths() == [500, 1, 0]
    freed = c.blocks_of(0)
    c.release(0)
    assert c.free_blocks == 7 and c.host_lengths()[0] == 0
    assert float(c.k_pool[freed[0]].abs().max()) == 0.0    # released blocks come back zeroed
    with pytest.raises(RuntimeError, match="max_blocks_per_seq"):
        c.reserve(1, 513)
    c.set_lengths([512, 512])
    with pytest.raises(RuntimeError, match="out of blocks"):
        c.reserve(2, 1)


def test_block_size_must_be_a_multiple_of_128():
    with pytest.raises(RuntimeError, match="multiple of 128"):
        PagedKVCache(num_blocks=2, num_kv_heads=1, head_dim=64, block_size=64, device="cpu")


def test_descriptor_fields():
    c = PagedKVCache(num_blocks=4, num_kv_heads=2, head_dim=128, block_size=256, max_seqs=2, device="cpu")
    d = c.descriptor()
    assert (d.block_stride, d.head_stride, d.row_stride) == (2 * 256 * 128, 256 * 128, 128)
    assert (d.num_blocks, d.block_size, d.table_stride, d.max_blocks_per_seq) == (4, 256, 4, 4)
    assert d.k_pool == c.k_pool.data_ptr() and d.block_table == c.block_table.data_ptr()


@pytest.fixture(scope="module")
def lib():
    build.build()
    return abi.load()


def test_abi_rejects_bad_descriptors(lib):
    ok = abi.PagedKV(16, 16, 4 * 256 * 128, 256 * 128, 128, 8, 256, 16, 4, 4)

    def prefill(kv):
        return lib.mllm_prefill_attention_paged_bf16(16, kv, 1, 8, 2, 128, 4, 4, 0.1, 16, None)
    assert prefill(None) == 1   # MLLM_ERR_INVALID_ARGUMENT
    assert b"NULL" in lib.mllm_attn_last_error()
    bad = abi.PagedKV.from_buffer_copy(ok)
    bad.block_size = 192
    assert prefill(C.byref(bad)) == 1
    assert b"multiple of 128" in lib.mllm_attn_last_error()
    bad = abi.PagedKV.from_buffer_copy(ok)
    bad.block_table = None
    assert prefill(C.byref(bad)) == 1
    # more rows than max_blocks_per_seq * block_size
    st = lib.mllm_decode_attention_paged_bf16(16, C.byref(ok), None, 1, 8, 2, 128, 4 * 256 + 1, 0.1, 16, 256,
                                              1 << 20, None)
    assert st == 1 and b"max_blocks_per_seq" in lib.mllm_attn_last_error()


def test_packed_helpers_check_on_the_host():
    """The packed-sequence helpers refuse bad input before any launch: CPU tensors, ragged
    lengths that do not add up to the token count, negative lengths, and a hidden state that is
    not [T, hidden].  No cache is touched."""
    from mllm_b200 import runtime as rt
    c = PagedKVCache(num_blocks=4, num_kv_heads=2, head_dim=64, block_size=128, max_seqs=2, device="cpu")
    q = torch.zeros(10, 4, 64, dtype=torch.bfloat16)
    k = torch.zeros(10, 2, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        rt.qkv_epilogue_packed(q, k, k, c, [4, 6], 1e6)
    with pytest.raises(RuntimeError, match="lengths must be >= 0"):
        rt._cu_seqlens([3, -1], "cpu")
    assert rt._cu_seqlens([3, 0, 5], "cpu")[0] == [0, 3, 3, 8]
    with pytest.raises(RuntimeError, match="sum to the token count"):
        rt.prefill_attention_packed(torch.zeros(4, 10, 64, dtype=torch.bfloat16), c, [4, 5], 2)
    with pytest.raises(RuntimeError, match=r"\[T, hidden\]"):
        rt.attention_block_packed(torch.zeros(1, 10, 256, dtype=torch.bfloat16), None, None, None, None, 4, 2, 64,
                                  1e6, [10], c)
    assert c.host_lengths() == [0, 0] and c.free_blocks == 4
