"""Python mirror of mLLM's stateless runtime API for the attention path, on the B200 kernels.

Same names, argument meaning and error behaviour as the reference's C++ classes
(src/core/runtime/{KVCache,RoPE,Attention,TransformerBlock}.h); every device computation goes
through the C ABI of libmllm_attn.so (include/mllm_attn.h).  Projections (Linear) stay torch
GEMMs, exactly as the reference keeps them in LibTorch.  There is no CPU path: CUDA bf16
tensors are required and anything else raises RuntimeError, like the reference's checks.

  KVCache                 src/core/runtime/KVCache.h:9-28  -- preallocated bf16 rows instead of
                          a tensor grown by torch::cat; .key/.value are views of the valid rows
  RoPE.build_cos_sin      src/core/runtime/RoPE.h:29-59
  RoPE.apply              src/core/runtime/RoPE.h:68-89
  Attention.forward       src/core/runtime/Attention.h:29-86
  Attention.forward_projected  src/core/runtime/Attention.h:100-326 (+ optional fused QK-norm,
                          which the reference does in TransformerBlock.h:103-134)
  attention_block         the attention half of TransformerBlock::Forward (h -> attention out)
"""
from __future__ import annotations

import ctypes as C
import math

import torch

from . import abi

BF16 = torch.bfloat16


def _check_cuda_bf16(name: str, t: torch.Tensor) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name}: the B200 attention path needs CUDA tensors (no CPU fallback)")
    if t.dtype != BF16:
        raise RuntimeError(f"{name}: expected bfloat16, got {t.dtype}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else t.data_ptr()


class KVCache:
    """Per-layer KV cache: bf16 rows [batch, num_kv_heads, capacity, head_dim] written in place.

    Mirrors KVCache.h:9-28: `key`/`value` are the valid rows [B, Hkv, L, D] (views), so callers
    that read `key.size(2)` (the runners' decode position, QwenRunner.cpp:301-310) see the
    cache length.  `lengths` holds per-sequence lengths for ragged batches."""

    capture_max_len = None   # set while a CUDA graph of decode steps is captured (decode_step)

    def __init__(self, batch: int, num_kv_heads: int, head_dim: int, capacity: int,
                 device="cuda", zero: bool = True):
        alloc = torch.zeros if zero else torch.empty
        self.key_buf = alloc((batch, num_kv_heads, capacity, head_dim), dtype=BF16, device=device)
        self.value_buf = alloc((batch, num_kv_heads, capacity, head_dim), dtype=BF16, device=device)
        self.capacity = capacity
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=device)
        self._host_lengths = [0] * batch

    # -- reference API --
    def is_initialized(self) -> bool:
        return max(self._host_lengths) > 0

    def clear(self) -> None:
        self.lengths.zero_()
        self._host_lengths = [0] * len(self._host_lengths)

    @property
    def length(self) -> int:
        if len(set(self._host_lengths)) != 1:
            raise RuntimeError("KVCache: ragged batch has no single length")
        return self._host_lengths[0]

    @property
    def key(self) -> torch.Tensor:
        return self.key_buf[:, :, : self.length]

    @property
    def value(self) -> torch.Tensor:
        return self.value_buf[:, :, : self.length]

    # -- layout for the kernels --
    @property
    def strides(self):
        s = self.key_buf.stride()
        return s[0], s[1], s[2]

    def host_lengths(self) -> list[int]:
        return list(self._host_lengths)

    def advance(self, n: int | list[int]) -> None:
        add = n if isinstance(n, list) else [n] * len(self._host_lengths)
        self._host_lengths = [a + b for a, b in zip(self._host_lengths, add)]
        if max(self._host_lengths) > self.capacity:
            raise RuntimeError("KVCache: capacity exceeded")
        self.lengths.copy_(torch.tensor(self._host_lengths, dtype=torch.int32), non_blocking=True)

    def set_lengths(self, lens: list[int]) -> None:
        if max(lens) > self.capacity:
            raise RuntimeError("KVCache: capacity exceeded")
        self._host_lengths = list(lens)
        self.lengths.copy_(torch.tensor(lens, dtype=torch.int32), non_blocking=True)

    def advance_host(self, n: int, batch: int) -> None:
        """The host copy of the lengths after a replayed decode graph advanced the device copy."""
        for b in range(batch):
            self._host_lengths[b] += n


class RoPE:
    @staticmethod
    def build_cos_sin(positions: torch.Tensor, head_dim: int, rope_theta: float):
        """RoPE::BuildCosSin: (cos, sin) fp32 [S, D] on the positions' device."""
        if head_dim % 2 != 0:
            raise RuntimeError("RoPE: head_dim must be even.")
        if not positions.is_cuda:
            raise RuntimeError("RoPE: positions must be a CUDA tensor (no CPU fallback)")
        pos = positions.to(torch.int64).contiguous()
        n = pos.numel()
        cos = torch.empty((n, head_dim), dtype=torch.float32, device=pos.device)
        sin = torch.empty_like(cos)
        abi.call("mllm_rope_build_cos_sin", _ptr(pos), n, head_dim, float(rope_theta), _ptr(cos),
                 _ptr(sin), abi.stream_handle())
        return cos, sin

    @staticmethod
    def apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """RoPE::Apply for bf16 x [B, H, S, D] (any strides with D contiguous)."""
        _check_cuda_bf16("RoPE", x)
        if x.dim() != 4 or x.stride(3) != 1:
            raise RuntimeError("RoPE: x must be [B, H, S, D] with D contiguous")
        B, H, S, D = x.shape
        cos = cos.to(torch.float32).contiguous()
        sin = sin.to(torch.float32).contiguous()
        out = torch.empty((B, H, S, D), dtype=BF16, device=x.device)
        abi.call("mllm_rope_apply_bf16", _ptr(x), x.stride(0), x.stride(1), x.stride(2), B, H, S, D,
                 _ptr(cos), _ptr(sin), _ptr(out), abi.stream_handle())
        return out


class PagedKVCache:
    """Paged KV cache for one layer (the mllm_paged_kv layout): K and V pools of `num_blocks`
    blocks, each `block_size` rows for every kv head ([num_blocks, Hkv, block_size, D] bf16), and
    per-sequence block tables and lengths.  Sequences of any length share the pool without
    padding to the longest.  Blocks are handed out from a free list as sequences grow (`reserve`)
    and zeroed when freed (`release`), so the rows past a sequence's length in its last block are
    always finite.  The reference's KVCache (KVCache.h:9-28) is one contiguous tensor per layer;
    this is the serving-format step beyond it."""

    capture_max_len = None   # set while a CUDA graph of decode steps is captured (decode_step)

    def __init__(self, num_blocks: int, num_kv_heads: int, head_dim: int, block_size: int = 256,
                 max_seqs: int = 64, max_blocks_per_seq: int | None = None, device="cuda"):
        if block_size <= 0 or block_size % 128 != 0:
            raise RuntimeError("PagedKVCache: block_size must be a positive multiple of 128")
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.max_blocks_per_seq = max_blocks_per_seq or num_blocks
        self.k_pool = torch.zeros((num_blocks, num_kv_heads, block_size, head_dim), dtype=BF16, device=device)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.block_table = torch.zeros((max_seqs, self.max_blocks_per_seq), dtype=torch.int32, device=device)
        self.lengths = torch.zeros(max_seqs, dtype=torch.int32, device=device)
        self._blocks = [[] for _ in range(max_seqs)]
        self._host_lengths = [0] * max_seqs
        self._free = list(range(num_blocks - 1, -1, -1))   # pop() hands out block 0 first

    @property
    def capacity(self) -> int:
        """Rows one sequence can hold."""
        return self.max_blocks_per_seq * self.block_size

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def blocks_of(self, seq: int) -> list[int]:
        return list(self._blocks[seq])

    def reserve(self, seq: int, rows: int) -> None:
        """Make sure sequence `seq` has blocks for `rows` rows."""
        need = -(-rows // self.block_size)
        if need > self.max_blocks_per_seq:
            raise RuntimeError("PagedKVCache: sequence exceeds max_blocks_per_seq * block_size rows")
        blocks = self._blocks[seq]
        if need > len(blocks):
            if need - len(blocks) > len(self._free):
                raise RuntimeError("PagedKVCache: out of blocks")
            start = len(blocks)
            while len(blocks) < need:
                blocks.append(self._free.pop())
            self.block_table[seq, start:need] = torch.tensor(blocks[start:need], dtype=torch.int32)

    def release(self, seq: int) -> None:
        """Return sequence `seq`'s blocks to the pool (zeroed) and reset its length."""
        blocks = self._blocks[seq]
        if blocks:
            idx = torch.tensor(blocks, dtype=torch.long, device=self.k_pool.device)
            self.k_pool.index_fill_(0, idx, 0)
            self.v_pool.index_fill_(0, idx, 0)
            self._free.extend(reversed(blocks))
        self._blocks[seq] = []
        self._host_lengths[seq] = 0
        self.lengths[seq] = 0

    def move(self, src: int, dst: int) -> None:
        """Hand sequence `src`'s blocks and length to the empty row `dst` (its block-table row is
        copied; no K/V row moves).  A serving loop uses it to keep its live sequences in rows
        0..n-1 when one in the middle finishes."""
        if src == dst:
            return
        if self._blocks[dst] or self._host_lengths[dst]:
            raise RuntimeError("PagedKVCache: move target row is not empty")
        self.block_table[dst].copy_(self.block_table[src])
        self.lengths[dst] = self.lengths[src]
        self._blocks[dst], self._blocks[src] = self._blocks[src], []
        self._host_lengths[dst], self._host_lengths[src] = self._host_lengths[src], 0
        self.lengths[src] = 0

    def slot(self, seq: int, count: int = 1) -> "PagedSlot":
        """A view of rows seq .. seq + count - 1 as a batch of `count` (prefill of new requests
        while other rows are live)."""
        return PagedSlot(self, seq, count)

    # -- the KVCache interface the attention functions use --
    def host_lengths(self) -> list[int]:
        return list(self._host_lengths)

    def set_lengths(self, lens: list[int]) -> None:
        for b, n in enumerate(lens):
            self.reserve(b, n)
        self._host_lengths[:len(lens)] = list(lens)
        self.lengths[:len(lens)].copy_(torch.tensor(lens, dtype=torch.int32), non_blocking=True)

    def advance(self, n: int | list[int], batch: int | None = None) -> None:
        B = batch if batch is not None else (len(n) if isinstance(n, list) else len(self._host_lengths))
        add = n if isinstance(n, list) else [n] * B
        self.set_lengths([self._host_lengths[b] + add[b] for b in range(B)])

    def advance_host(self, n: int, batch: int) -> None:
        """The host copy of the lengths after a replayed decode graph advanced the device copy
        (the blocks were reserved before the graph was captured)."""
        for b in range(batch):
            self._host_lengths[b] += n

    def length_of(self, batch: int) -> int:
        lens = set(self.host_lengths()[:batch])
        if len(lens) != 1:
            raise RuntimeError("PagedKVCache: ragged batch has no single length")
        return lens.pop()

    def descriptor(self) -> abi.PagedKV:
        s = self.k_pool.stride()
        return abi.PagedKV(self.k_pool.data_ptr(), self.v_pool.data_ptr(), s[0], s[1], s[2], self.num_blocks,
                           self.block_size, self.block_table.data_ptr(), self.block_table.stride(0),
                           self.max_blocks_per_seq)

    def gather(self, seq: int, rows: int):
        """K and V rows [Hkv, rows, D] of sequence `seq`, copied out of the pool (for tests)."""
        blocks = self._blocks[seq][: -(-rows // self.block_size)]
        k = torch.cat([self.k_pool[b] for b in blocks], dim=1)[:, :rows]
        v = torch.cat([self.v_pool[b] for b in blocks], dim=1)[:, :rows]
        return k, v


class PagedSlot(PagedKVCache):
    """Rows `seq` .. `seq + count - 1` of a PagedKVCache seen as a batch of `count`: the same
    pools, the parent's block-table rows and lengths (shared memory), and reserve/advance acting
    on those rows."""

    def __init__(self, parent: PagedKVCache, seq: int, count: int = 1):   # no pool allocation: a view
        if count < 1 or seq < 0 or seq + count > parent.block_table.shape[0]:
            raise RuntimeError("PagedSlot: rows outside the parent cache")
        self._parent, self._seq, self._count = parent, seq, count
        self.block_size = parent.block_size
        self.num_blocks = parent.num_blocks
        self.max_blocks_per_seq = parent.max_blocks_per_seq
        self.k_pool, self.v_pool = parent.k_pool, parent.v_pool
        self.block_table = parent.block_table[seq:seq + count]
        self.lengths = parent.lengths[seq:seq + count]

    def _row(self, seq: int) -> int:
        if not 0 <= seq < self._count:
            raise RuntimeError("PagedSlot: sequence outside the view")
        return self._seq + seq

    @property
    def free_blocks(self) -> int:
        return self._parent.free_blocks

    def blocks_of(self, seq: int) -> list[int]:
        return self._parent.blocks_of(self._row(seq))

    def reserve(self, seq: int, rows: int) -> None:
        self._parent.reserve(self._row(seq), rows)

    def release(self, seq: int = 0) -> None:
        self._parent.release(self._row(seq))

    def move(self, src: int, dst: int) -> None:
        raise RuntimeError("PagedSlot: move rows on the parent cache")

    def host_lengths(self) -> list[int]:
        return self._parent.host_lengths()[self._seq:self._seq + self._count]

    def set_lengths(self, lens: list[int]) -> None:
        if len(lens) > self._count:
            raise RuntimeError("PagedSlot: more lengths than sequences in the view")
        for b, n in enumerate(lens):
            self._parent.reserve(self._seq + b, n)
            self._parent._host_lengths[self._seq + b] = n
        self.lengths[:len(lens)].copy_(torch.tensor(lens, dtype=torch.int32), non_blocking=True)

    def advance(self, n, batch: int | None = None) -> None:
        B = batch if batch is not None else (len(n) if isinstance(n, list) else self._count)
        add = n if isinstance(n, list) else [n] * B
        cur = self.host_lengths()
        self.set_lengths([cur[b] + add[b] for b in range(B)])

    def gather(self, seq: int, rows: int):
        return self._parent.gather(self._row(seq), rows)


class DecodeWorkspace:
    """Grow-only, zero-filled device scratch for the split-K decode partials (the C ABI never
    allocates).  Its 256-byte header must start at zero; every call leaves it zero."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != torch.device(device):
            self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf


_WS = DecodeWorkspace()


class GraphScratch:
    """Device scratch owned by one captured CUDA graph: the decode and projection workspaces
    its kernels were recorded with.  The module's shared workspaces grow by reallocation, which
    would leave a graph writing into freed memory; these buffers live as long as the graph
    (hold the object beside it) and are never replaced while a capture is recording."""

    def __init__(self):
        self._keep: list[torch.Tensor] = []
        self._cur: dict = {}

    def get(self, key: str, nbytes: int, device) -> torch.Tensor:
        buf = self._cur.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            self._keep.append(buf)      # an earlier, smaller one stays alive for the nodes that use it
            self._cur[key] = buf
        return buf


_capture_scratch: GraphScratch | None = None


class graph_scratch:
    """`with graph_scratch(s):` around a CUDA graph capture makes the kernels recorded inside it
    take their workspaces from `s`."""

    def __init__(self, scratch: GraphScratch):
        self.scratch = scratch

    def __enter__(self):
        global _capture_scratch
        self.prev, _capture_scratch = _capture_scratch, self.scratch
        return self.scratch

    def __exit__(self, *exc):
        global _capture_scratch
        _capture_scratch = self.prev
        return False


def _capturing() -> bool:
    if not torch.cuda.is_available() or not torch.cuda.is_current_stream_capturing():
        return False
    if _capture_scratch is None:
        raise RuntimeError("capturing a CUDA graph of these kernels needs runtime.graph_scratch")
    return True


def qkv_epilogue(q, k, v, kv_cache: KVCache, positions: torch.Tensor, rope_theta: float,
                 q_norm_weight=None, k_norm_weight=None, eps: float = 1e-6,
                 rope_table=None) -> torch.Tensor:
    """Fused per-head QK-RMSNorm (optional) + RoPE + KV append.  q [B,H,S,D], k/v [B,Hkv,S,D]
    as strided views of the projections; positions int64 [S] (shared) or [B, S].  Rows go to
    cache slots lengths[b] + s; the cache lengths advance by S.  Returns Q [B,H,S,D] (rotated)."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda_bf16(n, t)
        if t.dim() != 4 or t.stride(3) != 1:
            raise RuntimeError(f"Attention: {n} must be rank-4 [B, h, S, D] with D contiguous")
    B, H, S, D = q.shape
    Hkv = k.shape[1]
    if H % Hkv != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    q_out = torch.empty((B, H, S, D), dtype=BF16, device=q.device)
    pos = positions.to(torch.int64)
    if pos.dim() == 1:
        pos_sb, pos_ss = 0, pos.stride(0)
    else:
        pos_sb, pos_ss = pos.stride(0), pos.stride(1)
    cos = sin = None
    rsb = rss = 0
    if rope_table is not None:
        cos, sin = (t.to(torch.float32).contiguous() for t in rope_table)
        rsb, rss = (0, 1) if cos.shape[0] == S else (S, 1)
    qn = kn = None
    if q_norm_weight is not None:
        qn = q_norm_weight.to(BF16).contiguous()
        kn = k_norm_weight.to(BF16).contiguous()
    if isinstance(kv_cache, PagedKVCache):
        start = kv_cache.lengths[:B].clone()   # slots of the new rows: the lengths before this call
        for b in range(B):
            kv_cache.reserve(b, kv_cache.host_lengths()[b] + S)
        kv = kv_cache.descriptor()
        abi.call("mllm_qkv_epilogue_paged_bf16",
                 _ptr(q), q.stride(0), q.stride(2), q.stride(1),
                 _ptr(k), k.stride(0), k.stride(2), k.stride(1),
                 _ptr(v), v.stride(0), v.stride(2), v.stride(1),
                 B, S, H, Hkv, D, _ptr(pos), pos_sb, pos_ss, float(rope_theta),
                 _ptr(cos), _ptr(sin), rsb, rss, _ptr(qn), _ptr(kn), float(eps), _ptr(q_out),
                 C.byref(kv), _ptr(start), 0, abi.stream_handle())
        kv_cache.advance(S, batch=B)
        return q_out
    csb, csh, cst = kv_cache.strides
    abi.call("mllm_qkv_epilogue_bf16",
             _ptr(q), q.stride(0), q.stride(2), q.stride(1),
             _ptr(k), k.stride(0), k.stride(2), k.stride(1),
             _ptr(v), v.stride(0), v.stride(2), v.stride(1),
             B, S, H, Hkv, D, _ptr(pos), pos_sb, pos_ss, float(rope_theta),
             _ptr(cos), _ptr(sin), rsb, rss, _ptr(qn), _ptr(kn), float(eps), _ptr(q_out),
             _ptr(kv_cache.key_buf), _ptr(kv_cache.value_buf), csb, csh, cst, kv_cache.capacity,
             _ptr(kv_cache.lengths), 0, abi.stream_handle())
    kv_cache.advance(S)
    return q_out


def prefill_attention(q: torch.Tensor, kv_cache: KVCache, num_kv_heads: int) -> torch.Tensor:
    """Causal attention of Q [B,H,S,D] (the newest S rows) over the cache -> [B, S, H*D]."""
    B, H, S, D = q.shape
    out = torch.empty((B, S, H * D), dtype=BF16, device=q.device)
    if isinstance(kv_cache, PagedKVCache):
        kv = kv_cache.descriptor()
        abi.call("mllm_prefill_attention_paged_bf16", _ptr(q), C.byref(kv), B, H, num_kv_heads, D, S,
                 kv_cache.length_of(B), 1.0 / math.sqrt(D), _ptr(out), abi.stream_handle())
        return out
    kv_len = kv_cache.length
    csb, csh, cst = kv_cache.strides
    abi.call("mllm_prefill_attention_bf16", _ptr(q), _ptr(kv_cache.key_buf), _ptr(kv_cache.value_buf),
             csb, csh, cst, B, H, num_kv_heads, D, S, kv_len, 1.0 / math.sqrt(D), _ptr(out),
             abi.stream_handle())
    return out


def _cu_seqlens(q_lens: list[int], device) -> tuple[list[int], torch.Tensor]:
    """Row offsets of packed sequences: host list and int32 device tensor [len(q_lens) + 1]."""
    if any(n < 0 for n in q_lens):
        raise RuntimeError("packed sequences: lengths must be >= 0")
    cu = [0]
    for n in q_lens:
        cu.append(cu[-1] + n)
    return cu, torch.tensor(cu, dtype=torch.int32).to(device, non_blocking=True)


def qkv_epilogue_packed(q, k, v, kv_cache, q_lens: list[int], rope_theta: float, positions=None,
                        q_norm_weight=None, k_norm_weight=None, eps: float = 1e-6) -> torch.Tensor:
    """qkv_epilogue (TransformerBlock.h:103-107,130-134 and Attention.h:157-208) for several
    sequences of different lengths packed on one token axis, in one launch; the reference runs one
    sequence's prompt per Generate call (QwenRunner.cpp:420-545).  q [T, H, D] and k/v [T, Hkv, D] (strided views of the projections, D contiguous);
    sequence b owns the next q_lens[b] tokens, which go to cache slots lengths[b] + s of cache
    sequence b; the lengths advance by q_lens[b].  positions: int64 [T] (default: each token's
    cache slot).  Returns Q [H, T, D] (rotated), the layout prefill_attention_packed reads."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda_bf16(n, t)
        if t.dim() != 3 or t.stride(2) != 1:
            raise RuntimeError(f"Attention: {n} must be rank-3 [T, h, D] with D contiguous")
    T, H, D = q.shape
    Hkv = k.shape[1]
    if H % Hkv != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    B = len(q_lens)
    cu, cu_dev = _cu_seqlens(q_lens, q.device)
    if cu[-1] != T:
        raise RuntimeError("packed sequences: q_lens must sum to the token count")
    if T == 0:
        return torch.empty((H, 0, D), dtype=BF16, device=q.device)
    before = kv_cache.host_lengths()[:B]
    if positions is None:
        positions = torch.cat([torch.arange(before[b], before[b] + q_lens[b], dtype=torch.int64)
                               for b in range(B)]).to(q.device, non_blocking=True)
    pos = positions.to(device=q.device, dtype=torch.int64).contiguous()
    if pos.numel() != T:
        raise RuntimeError("packed sequences: one position per token")
    qn = kn = None
    if q_norm_weight is not None:
        qn = q_norm_weight.to(BF16).contiguous()
        kn = k_norm_weight.to(BF16).contiguous()
    q_out = torch.empty((H, T, D), dtype=BF16, device=q.device)
    start = kv_cache.lengths[:B].clone()    # slots of the new rows: the lengths before this call
    common = (_ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0),
              v.stride(1), T, H, Hkv, D, _ptr(pos), float(rope_theta), _ptr(qn), _ptr(kn), float(eps),
              _ptr(q_out))
    if isinstance(kv_cache, PagedKVCache):
        kv_cache.advance(list(q_lens), batch=B)   # reserves the blocks; raises before any launch
        kv = kv_cache.descriptor()
        abi.call("mllm_qkv_epilogue_varlen_paged_bf16", *common, C.byref(kv), _ptr(cu_dev), B, _ptr(start),
                 abi.stream_handle())
        return q_out
    if B != len(kv_cache.host_lengths()):
        raise RuntimeError("packed sequences: one length per cache sequence")
    kv_cache.advance(list(q_lens))                # raises before any launch if the cache is full
    csb, csh, cst = kv_cache.strides
    abi.call("mllm_qkv_epilogue_varlen_bf16", *common, _ptr(kv_cache.key_buf), _ptr(kv_cache.value_buf), csb,
             csh, cst, kv_cache.capacity, _ptr(cu_dev), B, _ptr(start), abi.stream_handle())
    return q_out


def prefill_attention_packed(q: torch.Tensor, kv_cache, q_lens: list[int], num_kv_heads: int) -> torch.Tensor:
    """Causal attention (Attention.h:220-316) of packed sequences: Q [H, T, D]
    (qkv_epilogue_packed's output, sequence b owning the next q_lens[b] rows, its newest rows) over each sequence's cache rows
    0 .. lengths[b] - 1 -> [T, H*D]."""
    H, T, D = q.shape
    B = len(q_lens)
    cu, cu_dev = _cu_seqlens(q_lens, q.device)
    if cu[-1] != T:
        raise RuntimeError("packed sequences: q_lens must sum to the token count")
    out = torch.empty((T, H * D), dtype=BF16, device=q.device)
    max_q = max(q_lens) if q_lens else 0
    kv_lens = kv_cache.lengths[:B]
    if isinstance(kv_cache, PagedKVCache):
        kv = kv_cache.descriptor()
        abi.call("mllm_prefill_attention_varlen_paged_bf16", _ptr(q), C.byref(kv), _ptr(cu_dev), _ptr(kv_lens), B,
                 H, num_kv_heads, D, T, max_q, 1.0 / math.sqrt(D), _ptr(out), abi.stream_handle())
        return out
    csb, csh, cst = kv_cache.strides
    abi.call("mllm_prefill_attention_varlen_bf16", _ptr(q), _ptr(kv_cache.key_buf), _ptr(kv_cache.value_buf),
             csb, csh, cst, kv_cache.capacity, _ptr(cu_dev), _ptr(kv_lens), B, H, num_kv_heads, D, T, max_q,
             1.0 / math.sqrt(D), _ptr(out), abi.stream_handle())
    return out


def decode_attention(q: torch.Tensor, kv_cache: KVCache, num_kv_heads: int,
                     max_kv_len: int | None = None) -> torch.Tensor:
    """One query row per sequence (Q [B,H,1,D] or [B,H,D]) over each sequence's cache rows
    (per-sequence lengths) -> [B, 1, H*D]."""
    B, H, D = q.shape[0], q.shape[1], q.shape[-1]
    qq = q.reshape(B, H, D)
    if not qq.is_contiguous():
        qq = qq.contiguous()
    L = max_kv_len or max(kv_cache.host_lengths()[:B])
    L = min(L, kv_cache.capacity)
    out = torch.empty((B, 1, H * D), dtype=BF16, device=q.device)
    lib = abi.load()
    nbytes = lib.mllm_decode_attention_workspace_size(B, H, num_kv_heads, D, L)
    ws = _capture_scratch.get("decode", nbytes, q.device) if _capturing() else _WS.get(nbytes, q.device)
    if isinstance(kv_cache, PagedKVCache):
        kv = kv_cache.descriptor()
        abi.call("mllm_decode_attention_paged_bf16", _ptr(qq), C.byref(kv), _ptr(kv_cache.lengths), B, H,
                 num_kv_heads, D, L, 1.0 / math.sqrt(D), _ptr(out), _ptr(ws), ws.numel(), abi.stream_handle())
        return out
    csb, csh, cst = kv_cache.strides
    abi.call("mllm_decode_attention_bf16", _ptr(qq), _ptr(kv_cache.key_buf), _ptr(kv_cache.value_buf),
             csb, csh, cst, _ptr(kv_cache.lengths), B, H, num_kv_heads, D, L, 1.0 / math.sqrt(D),
             _ptr(out), _ptr(ws), ws.numel(), abi.stream_handle())
    return out


def decode_step(q, k, v, kv_cache: KVCache, positions: torch.Tensor, rope_theta: float, num_kv_heads: int,
                q_norm_weight=None, k_norm_weight=None, eps: float = 1e-6, rope_table=None) -> torch.Tensor:
    """One new token per sequence through the fused step: QK-RMSNorm (optional) + RoPE + KV
    append + decode attention in one launch.  q [B,H,1,D], k/v [B,Hkv,1,D] (strided views of the
    projections); positions int64 [1] (shared) or [B] / [B, 1].  The new rows go to slot
    lengths[b] of each sequence and the lengths advance by one.  Returns [B, 1, H*D]."""
    for n, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda_bf16(n, t)
        if t.dim() != 4 or t.size(2) != 1 or t.stride(3) != 1:
            raise RuntimeError(f"Attention: {n} must be [B, h, 1, D] with D contiguous")
    B, H, _, D = q.shape
    if H % num_kv_heads != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    pos = positions.to(torch.int64).reshape(-1)
    pos_sb = 0 if pos.numel() == 1 else pos.stride(0)
    cos = sin = None
    rsb = 0
    if rope_table is not None:
        cos, sin = (t.to(torch.float32).contiguous() for t in rope_table)
        rsb = 0 if cos.shape[0] == 1 else 1
    qn = kn = None
    if q_norm_weight is not None:
        qn = q_norm_weight.to(BF16).contiguous()
        kn = k_norm_weight.to(BF16).contiguous()
    capturing = _capturing()
    if capturing:
        # Recorded into a CUDA graph that replays this step many times: the lengths advance on the
        # device (the caller advances the host copy after each replay, and reserved the blocks
        # beforehand), and the bound on every sequence's length is the one the graph was made for.
        if kv_cache.capture_max_len is None:
            raise RuntimeError("decode_step: set the cache's capture_max_len before capturing a graph")
        kv_cache.lengths[:B] += 1
        L = min(kv_cache.capture_max_len, kv_cache.capacity)
    else:
        if isinstance(kv_cache, PagedKVCache):
            kv_cache.advance(1, batch=B)   # reserves the blocks; raises before any launch if the pool is full
        else:
            kv_cache.advance(1)   # raises before any launch if the cache is full
        L = min(max(kv_cache.host_lengths()[:B]), kv_cache.capacity)
    out = torch.empty((B, 1, H * D), dtype=BF16, device=q.device)
    lib = abi.load()
    nbytes = lib.mllm_decode_attention_workspace_size(B, H, num_kv_heads, D, L)
    ws = _capture_scratch.get("decode", nbytes, q.device) if capturing else _WS.get(nbytes, q.device)
    if isinstance(kv_cache, PagedKVCache):
        kv = kv_cache.descriptor()
        abi.call("mllm_decode_step_paged_bf16",
                 _ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0),
                 v.stride(1), _ptr(pos), pos_sb, float(rope_theta), _ptr(cos), _ptr(sin), rsb, _ptr(qn), _ptr(kn),
                 float(eps), C.byref(kv), _ptr(kv_cache.lengths), B, H, num_kv_heads, D, L, 1.0 / math.sqrt(D),
                 _ptr(out), _ptr(ws), ws.numel(), abi.stream_handle())
        return out
    csb, csh, cst = kv_cache.strides
    abi.call("mllm_decode_step_bf16",
             _ptr(q), q.stride(0), q.stride(1), _ptr(k), k.stride(0), k.stride(1), _ptr(v), v.stride(0), v.stride(1),
             _ptr(pos), pos_sb, float(rope_theta), _ptr(cos), _ptr(sin), rsb, _ptr(qn), _ptr(kn), float(eps),
             _ptr(kv_cache.key_buf), _ptr(kv_cache.value_buf), csb, csh, cst, _ptr(kv_cache.lengths),
             B, H, num_kv_heads, D, L, 1.0 / math.sqrt(D), _ptr(out), _ptr(ws), ws.numel(), abi.stream_handle())
    return out


_SAMPLE_WS = DecodeWorkspace()


def sample(logits: torch.Tensor, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0,
           use_greedy: bool = False, previous_tokens=None, repetition_penalty: float = 1.0,
           seed: int = 0, offset: int = 0) -> torch.Tensor:
    """Sampler::Sample (Sampler.cpp:49-232) on the device for a batch of rows: logits [B, V] (or
    [V]) bf16 or fp32 CUDA, penalised IN PLACE like the reference; previous_tokens: a list of
    per-row token lists (or one list for a single row).  Returns the int64 token ids [B] on the
    device, without a host round trip.  The sampling draw of row b comes from Philox-4x32-10 with
    key `seed` and counter (offset, b, 0)."""
    if not logits.is_cuda:
        raise RuntimeError("Sampler: logits must be a CUDA tensor (no CPU fallback)")
    if logits.dtype not in (BF16, torch.float32):
        raise RuntimeError("Sampler: logits must be bf16 or fp32")
    x = logits if logits.dim() == 2 else logits.view(1, -1)
    if x.stride(1) != 1:
        raise RuntimeError("Sampler: logits rows must be contiguous")
    B, V = x.shape
    prev = cnt = None
    if previous_tokens is not None:
        rows = previous_tokens if (len(previous_tokens) and isinstance(previous_tokens[0], (list, tuple))) \
            else [previous_tokens]
        if len(rows) != B:
            raise RuntimeError("Sampler: one history per row")
        T = max(1, max(len(r) for r in rows))
        h = torch.full((B, T), -1, dtype=torch.int64)
        for b, r in enumerate(rows):
            h[b, : len(r)] = torch.tensor(list(r), dtype=torch.int64)
        prev = h.to(x.device, non_blocking=True)
        cnt = torch.tensor([len(r) for r in rows], dtype=torch.int32).to(x.device, non_blocking=True)
    out = torch.empty(B, dtype=torch.int64, device=x.device)
    lib = abi.load()
    ws = _SAMPLE_WS.get(lib.mllm_sample_workspace_size(B, V), x.device)
    abi.call("mllm_sample", _ptr(x), int(x.dtype == BF16), x.stride(0), B, V, _ptr(prev),
             prev.stride(0) if prev is not None else 0, _ptr(cnt), float(temperature), int(top_k), float(top_p),
             int(bool(use_greedy)), float(repetition_penalty), int(seed), int(offset), _ptr(out), _ptr(ws),
             ws.numel(), abi.stream_handle())
    return out


LINEAR_MAX_TOKENS = 256


def linear_supported(x: torch.Tensor, weights) -> bool:
    """Whether mllm_linear_bf16 takes this projection: bf16 CUDA tensors, at most 256 rows of x,
    K a multiple of 64, each weight's rows a multiple of 128, unit inner strides."""
    if not (x.is_cuda and x.dtype == BF16 and x.stride(-1) == 1 and 0 < len(weights) <= 4):
        return False
    T = x.numel() // x.size(-1) if x.size(-1) else 0
    K = x.size(-1)
    if T > LINEAR_MAX_TOKENS or K % 64 != 0:
        return False
    return all(w.is_cuda and w.dtype == BF16 and w.dim() == 2 and w.size(1) == K and w.stride(1) == 1
               and w.size(0) % 128 == 0 and w.stride(0) % 8 == 0 and w.data_ptr() % 16 == 0 for w in weights)


def linear(x: torch.Tensor, weights) -> torch.Tensor:
    """Linear::Forward (Linear.h:33-68) of up to four weights in one launch (mllm_linear_bf16):
    x [..., K] bf16 with at most 256 rows -> [..., sum of out_features], the weights' outputs
    side by side (q | k | v for the three attention projections).  fp32 accumulation, one
    rounding to bf16."""
    weights = list(weights)
    if not linear_supported(x, weights):
        raise RuntimeError("linear: needs bf16 CUDA tensors, <= 256 rows, K % 64 == 0, weight rows % 128 == 0")
    lead = x.shape[:-1]
    K = x.size(-1)
    x2 = x.reshape(-1, K)
    if x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    T = x2.size(0)
    n = [w.size(0) for w in weights]
    out = torch.empty((T, sum(n)), dtype=BF16, device=x.device)
    W = len(weights)
    wp = (C.c_void_p * W)(*[w.data_ptr() for w in weights])
    wst = (C.c_int64 * W)(*[w.stride(0) for w in weights])
    nf = (C.c_int64 * W)(*n)
    need = abi.load().mllm_linear_workspace_size(T, W, nf, K)
    if need and _capturing():
        ws = _capture_scratch.get("linear", need, x.device)
    else:
        ws = _linear_workspace(x.device, need)
    abi.call("mllm_linear_bf16", _ptr(x2), x2.stride(0), T, K, W, wp, wst, nf, _ptr(out), out.stride(0),
             _ptr(ws), ws.numel() if ws is not None else 0, abi.stream_handle())
    return out.view(*lead, sum(n))


_LINEAR_WS: dict = {}


def _linear_workspace(device, nbytes: int):
    """The split partials and tile counters of mllm_linear_bf16: one zero-filled buffer per
    (device, stream), grown on demand; every call leaves its counters at zero."""
    if nbytes == 0:
        return None
    key = (device, torch.cuda.current_stream(device).cuda_stream)
    ws = _LINEAR_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _LINEAR_WS[key] = ws
    return ws


class Fp8Weight:
    """A projection stored the way FP8 checkpoints hold it (QwenRunner.cpp:148-283 loads it with its
    `weight_scale_inv`): e4m3 values w [out, in] and fp32 scales [out/128, in/128], one per
    128 x 128 block.  The reference dequantizes it on every step (DequantizeFP8,
    QwenRunner.cpp:103-122) and multiplies in bf16; `linear_fp8` multiplies it as stored."""

    BLOCK = 128

    def __init__(self, w: torch.Tensor, scale_inv: torch.Tensor):
        if w.dtype != torch.float8_e4m3fn or w.dim() != 2:
            raise RuntimeError("Fp8Weight: e4m3 [out, in] weights")
        n, k = w.shape
        if n % self.BLOCK or k % self.BLOCK or tuple(scale_inv.shape) != (n // self.BLOCK, k // self.BLOCK):
            raise RuntimeError("Fp8Weight: 128 x 128 blocks, scales [out/128, in/128]")
        self.w = w.contiguous()
        self.scale_inv = scale_inv.float().contiguous()

    @classmethod
    def quantize(cls, w: torch.Tensor) -> "Fp8Weight":
        """Block-wise e4m3 quantization of a weight (scale = block amax / 448), the format of
        FP8 checkpoints; for building test and benchmark models."""
        n, k = w.shape
        b = cls.BLOCK
        blocks = w.float().view(n // b, b, k // b, b)
        amax = blocks.abs().amax(dim=(1, 3)).clamp_min(1e-12)
        scale = amax / 448.0
        q = (blocks / scale[:, None, :, None]).to(torch.float8_e4m3fn).view(n, k)
        return cls(q, scale)

    def size(self, dim: int) -> int:
        return self.w.size(dim)

    @property
    def shape(self):
        return self.w.shape

    def dequantize(self, dtype=BF16) -> torch.Tensor:
        """DequantizeFP8 (QwenRunner.cpp:103-122): w.to(dtype) * scale.to(dtype), block-broadcast,
        in dtype -- the weights the reference's GEMM sees."""
        n, k = self.w.shape
        b = self.BLOCK
        w_h = self.w.to(dtype).reshape(n // b, b, k // b, b)
        s_h = self.scale_inv.to(dtype).unsqueeze(1).unsqueeze(3)
        return (w_h * s_h).reshape(n, k)


FP8_MAX_TOKENS = 128


def linear_fp8(x: torch.Tensor, w: Fp8Weight) -> torch.Tensor:
    """Linear::Forward(x, DequantizeFP8(w)) for bf16 x with at most 128 rows, by
    mllm_linear_fp8_bf16: the fp8 bytes are streamed and dequantized on chip (into tensor memory) with the
    reference's rounding, so the product equals a bf16 GEMM on the dequantized weight (fp32
    accumulation, one rounding).  More rows: the reference's own route (dequantize, cuBLAS)."""
    K = x.size(-1)
    if K != w.size(1):
        raise RuntimeError("Linear: last dim of x must match weight in_features.")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    T = x2.size(0)
    if not (x.is_cuda and x.dtype == BF16) or T > FP8_MAX_TOKENS:
        return torch.nn.functional.linear(x, w.dequantize(x.dtype))
    if x2.stride(-1) != 1 or x2.stride(0) % 8 != 0 or x2.data_ptr() % 16 != 0:
        x2 = x2.contiguous()
    N = w.size(0)
    out = torch.empty((T, N), dtype=BF16, device=x.device)
    need = abi.load().mllm_linear_fp8_workspace_size(T, N, K)
    if need and _capturing():
        ws = _capture_scratch.get("linear", need, x.device)
    else:
        ws = _linear_workspace(x.device, need)
    abi.call("mllm_linear_fp8_bf16", _ptr(x2), x2.stride(0), T, K, _ptr(w.w), w.w.stride(0), N, _ptr(w.scale_inv),
             w.scale_inv.stride(0), _ptr(out), out.stride(0), _ptr(ws), ws.numel() if ws is not None else 0,
             abi.stream_handle())
    return out.view(*lead, N)


def _linear(x: torch.Tensor, w) -> torch.Tensor:
    """Linear::Forward (Linear.h:33-68): x @ w.T in the input dtype, a cuBLAS GEMM as in the
    reference (for one weight mllm_linear_bf16 is not faster than cuBLAS beyond a few tokens);
    an Fp8Weight goes through linear_fp8."""
    if isinstance(w, Fp8Weight):
        return linear_fp8(x, w)
    if x.size(-1) != w.size(1):
        raise RuntimeError("Linear: last dim of x must match weight in_features.")
    return torch.nn.functional.linear(x, w)


def _project_qkv(h: torch.Tensor, w_q, w_k, w_v, num_heads: int, num_kv_heads: int, head_dim: int):
    """The three attention projections (TransformerBlock.h:82-96, Attention.h:52-54) as q [B,H,S,D]
    and k/v [B,Hkv,S,D] views.  Up to 256 tokens: one mllm_linear_bf16 launch writes q | k | v side
    by side and the views point into it; otherwise three cuBLAS GEMMs as in the reference (FP8
    weights: three linear_fp8 launches)."""
    B, S, E = h.shape
    if not any(isinstance(w, Fp8Weight) for w in (w_q, w_k, w_v)) and linear_supported(h, [w_q, w_k, w_v]):
        qkv = linear(h, [w_q, w_k, w_v])          # [B, S, (H + 2 Hkv) D]
        hq, hk = num_heads * head_dim, num_kv_heads * head_dim
        q = qkv[..., :hq].view(B, S, num_heads, head_dim).transpose(1, 2)
        k = qkv[..., hq:hq + hk].view(B, S, num_kv_heads, head_dim).transpose(1, 2)
        v = qkv[..., hq + hk:hq + 2 * hk].view(B, S, num_kv_heads, head_dim).transpose(1, 2)
        return q, k, v
    q = _linear(h, w_q).view(B, S, num_heads, head_dim).transpose(1, 2)
    k = _linear(h, w_k).view(B, S, num_kv_heads, head_dim).transpose(1, 2)
    v = _linear(h, w_v).view(B, S, num_kv_heads, head_dim).transpose(1, 2)
    return q, k, v


class Attention:
    @staticmethod
    def forward_projected(q, k, v, w_o, num_heads: int, num_kv_heads: int, head_dim: int,
                          rope_theta: float, position_ids: torch.Tensor, kv_cache: KVCache | None,
                          q_norm_weight=None, k_norm_weight=None, rms_norm_eps: float = 1e-6):
        """Attention::ForwardProjected (Attention.h:100-326).  q [B,H,S,D], k/v [B,Hkv,S,D]
        (views of the projections).  With norm weights, the per-head QK-RMSNorm that the
        reference runs in TransformerBlock.h:103-134 is fused into the epilogue."""
        if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
            raise RuntimeError("Attention::ForwardProjected: q/k/v must be rank-4 tensors.")
        if num_heads % num_kv_heads != 0:
            raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
        B, _, S, D = q.shape
        cache = kv_cache
        if cache is None:  # no cache: attend over this call's rows only (Attention.h:183 skipped)
            cache = KVCache(B, num_kv_heads, D, S, device=q.device)
        pos = position_ids.to(device=q.device)
        if S == 1:   # decode: epilogue and attention fused in one launch
            out = decode_step(q, k, v, cache, pos, rope_theta, num_kv_heads, q_norm_weight, k_norm_weight,
                              rms_norm_eps)
        else:
            qr = qkv_epilogue(q, k, v, cache, pos, rope_theta, q_norm_weight, k_norm_weight, rms_norm_eps)
            out = prefill_attention(qr, cache, num_kv_heads)
        return out if w_o is None else _linear(out, w_o)   # w_o None: the unprojected [B, S, H*D]

    @staticmethod
    def forward(hidden, w_q, w_k, w_v, w_o, num_heads: int, num_kv_heads: int, head_dim: int,
                rope_theta: float, position_ids: torch.Tensor, kv_cache: KVCache | None):
        """Attention::Forward (Attention.h:29-86): project, view, transpose, then the above."""
        if hidden.dim() != 3:
            raise RuntimeError("Attention: hidden must be [B, S, H].")
        q, k, v = _project_qkv(hidden, w_q, w_k, w_v, num_heads, num_kv_heads, head_dim)
        return Attention.forward_projected(q, k, v, w_o, num_heads, num_kv_heads, head_dim,
                                           rope_theta, position_ids, kv_cache)


def attention_block_packed(h, w_q, w_k, w_v, w_o, num_heads: int, num_kv_heads: int, head_dim: int,
                           rope_theta: float, q_lens: list[int], kv_cache, w_q_norm=None, w_k_norm=None,
                           rms_norm_eps: float = 1e-6, positions=None):
    """attention_block (TransformerBlock.h:77-195, attention half) for several prompts (or prompt
    chunks) of different lengths in one pass:
    h [T, hidden] holds the sequences' new rows back to back, sequence b the next q_lens[b] rows,
    appended to cache sequence b.  One projection, one epilogue and one attention launch for all
    of them; returns the o_proj output [T, hidden] (or [T, H*D] with w_o None)."""
    if h.dim() != 2:
        raise RuntimeError("attention_block_packed: h must be [T, hidden]")
    q, k, v = _project_qkv(h.unsqueeze(0), w_q, w_k, w_v, num_heads, num_kv_heads, head_dim)
    qr = qkv_epilogue_packed(q[0].transpose(0, 1), k[0].transpose(0, 1), v[0].transpose(0, 1), kv_cache, q_lens,
                             rope_theta, positions, w_q_norm, w_k_norm, rms_norm_eps)
    out = prefill_attention_packed(qr, kv_cache, q_lens, num_kv_heads)
    return out if w_o is None else _linear(out, w_o)


def attention_block(h, w_q, w_k, w_v, w_o, num_heads: int, num_kv_heads: int, head_dim: int,
                    rope_theta: float, position_ids, kv_cache, w_q_norm=None, w_k_norm=None,
                    rms_norm_eps: float = 1e-6):
    """The attention half of TransformerBlock::Forward (TransformerBlock.h:77-195) after the
    input RMSNorm: Qwen3 branch when norm weights are given, Llama branch otherwise."""
    q, k, v = _project_qkv(h, w_q, w_k, w_v, num_heads, num_kv_heads, head_dim)
    return Attention.forward_projected(q, k, v, w_o, num_heads, num_kv_heads, head_dim, rope_theta,
                                       position_ids, kv_cache, w_q_norm, w_k_norm, rms_norm_eps)
