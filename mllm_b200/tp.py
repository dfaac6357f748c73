"""Tensor-parallel attention across GPUs: KV-head-group sharding + one o_proj all-reduce.

The reference runs every layer on one device (QwenRunner.cpp:236,328); across N GPUs the
attention path shards naturally by KV-head group:

  rank r owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their n_rep query heads each, so
    w_q / w_k / w_v   row slices   (the projections of the owned heads)
    QK-norm, RoPE, KV cache, prefill / decode attention   fully local
    w_o               column slice (o_proj of the owned heads' outputs) -> a partial [B, S, hidden]
  and the partial outputs are summed by ONE all-reduce (NCCL over NVLink on GPUs).

`attention_fn` computes the local attention block; the default is the B200 path
(mllm_b200.runtime.attention_block).  The all-reduce uses the given torch.distributed group.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class HeadShard:
    rank: int
    world: int
    q_heads: tuple   # [start, end)
    kv_heads: tuple  # [start, end)

    @property
    def num_heads(self) -> int:
        return self.q_heads[1] - self.q_heads[0]

    @property
    def num_kv_heads(self) -> int:
        return self.kv_heads[1] - self.kv_heads[0]


def shard_heads(num_heads: int, num_kv_heads: int, world: int, rank: int) -> HeadShard:
    """KV-head groups split evenly over `world` ranks (num_kv_heads % world == 0)."""
    if num_heads % num_kv_heads != 0:
        raise RuntimeError("Attention: num_heads must be divisible by num_kv_heads.")
    if num_kv_heads % world != 0:
        raise RuntimeError(f"tensor parallel: {num_kv_heads} kv heads do not split over {world} ranks")
    if not 0 <= rank < world:
        raise RuntimeError("tensor parallel: rank out of range")
    n_rep = num_heads // num_kv_heads
    per = num_kv_heads // world
    g0, g1 = rank * per, (rank + 1) * per
    return HeadShard(rank, world, (g0 * n_rep, g1 * n_rep), (g0, g1))


def shard_weights(shard: HeadShard, head_dim: int, w_q, w_k, w_v, w_o):
    """Row slices of w_q/w_k/w_v ([out, in], HF layout) and the column slice of w_o."""
    q0, q1 = shard.q_heads[0] * head_dim, shard.q_heads[1] * head_dim
    k0, k1 = shard.kv_heads[0] * head_dim, shard.kv_heads[1] * head_dim
    return (w_q[q0:q1].contiguous(), w_k[k0:k1].contiguous(), w_v[k0:k1].contiguous(),
            w_o[:, q0:q1].contiguous())


def oproj_allreduce(attn, w_o, group=None, chunks: int = 4):
    """o_proj of this rank's heads summed over the ranks: attn [T, H_r*D] (this rank's attention
    output rows) times its column slice of w_o, all-reduced.  The rows go in `chunks` pieces, and
    the all-reduce of piece i is enqueued (asynchronously: NCCL's stream waits for that piece's
    GEMM) before the GEMM of piece i+1, so the exchange of one piece overlaps the GEMM of the next
    instead of following the whole GEMM.  Each output row is summed exactly as by one all-reduce
    of the whole partial."""
    import torch
    import torch.distributed as dist
    T = attn.shape[0]
    out = torch.empty((T, w_o.shape[0]), dtype=attn.dtype, device=attn.device)
    step = -(-T // max(1, chunks))
    works = []
    for a in range(0, T, step):
        b = min(T, a + step)
        torch.matmul(attn[a:b], w_o.t(), out=out[a:b])
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            works.append(dist.all_reduce(out[a:b], op=dist.ReduceOp.SUM, group=group, async_op=True))
    for w in works:
        w.wait()
    return out


class PeerExchange:
    """The o_proj exchange over NVLink copy engines: each rank's o_proj partial [T, hidden] summed
    over the ranks, every rank ending with the full sum, without an NCCL all-reduce.

    The rows are split into N owner blocks (block o belongs to rank o) of `sub` pieces each.  A
    rank computes its partial piece by piece, the pieces it does not own first in each round:
      * a piece owned by rank o goes to o's receive buffer (cudaMemcpyAsync over NVLink on a copy
        stream, so it overlaps the GEMM of the next pieces), after which a flag in o's memory is
        raised to a per-call counter;
      * once its own piece is computed, the owner waits (bounded) for the other ranks' flags, sums
        the N partials of the piece in rank order (fp32, one rounding), and copies the final rows
        to every other rank the same way.
    The result for rank r's rows is bit-identical on every rank.  Buffers are CUDA IPC
    allocations shared once at construction (mllm_ipc_*); receive and output buffers alternate
    between two sets by call parity, and a rank only writes a peer's set after having received
    that peer's previous output, so no write can overtake a read.  A returned output stays valid
    until the call after next.  No multicast object or load is used."""

    def __init__(self, rows: int, hidden: int, group=None, sub: int = 2, device=None):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import abi
        self.lib = abi.load()
        self.group = group
        self.N = dist.get_world_size(group)
        self.r = dist.get_rank(group)
        self.rows, self.hidden, self.sub = rows, hidden, sub
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        N = self.N
        self.block = [(o * rows // N, (o + 1) * rows // N) for o in range(N)]
        self.pieces = {}
        for o, (a, b) in enumerate(self.block):
            self.pieces[o] = [(a + j * (b - a) // sub, a + (j + 1) * (b - a) // sub) for j in range(sub)]
        self.max_block = max(b - a for a, b in self.block)
        es = 2
        self.recv_bytes = N * self.max_block * hidden * es     # per set: [sender][block row][hidden]
        self.out_bytes = rows * hidden * es                   # per set
        self.flag_bytes = 4096                                 # recv flags [N], out flags [N]
        total = self.flag_bytes + 2 * (self.recv_bytes + self.out_bytes)
        base = C.c_void_p()
        abi.call("mllm_ipc_alloc", total, C.byref(base))
        self.base = base.value
        h = (C.c_ubyte * 64)()
        abi.call("mllm_ipc_get_handle", self.base, h)
        handles = [None] * N
        dist.all_gather_object(handles, bytes(h), group=group)
        self.peer = []
        for s in range(N):
            if s == self.r:
                self.peer.append(self.base)
                continue
            p = C.c_void_p()
            hh = (C.c_ubyte * 64).from_buffer_copy(handles[s])
            abi.call("mllm_ipc_open_handle", hh, C.byref(p))
            self.peer.append(p.value)
        self.partial = torch.empty((rows, hidden), dtype=torch.bfloat16, device=self.device)
        # one send and one gather stream per peer, so transfers to different peers run on
        # different copy engines at the same time
        self.s_send = {p: torch.cuda.Stream(device=self.device) for p in range(self.N) if p != self.r}
        self.s_gather = {p: torch.cuda.Stream(device=self.device) for p in range(self.N) if p != self.r}
        self.s_reduce = torch.cuda.Stream(device=self.device)
        self.calls = 0
        dist.barrier(group=group)

    # addresses inside rank s's shared allocation
    def _recv_flag(self, s, sender):
        return self.peer[s] + 4 * sender

    def _out_flag(self, s, sender):
        return self.peer[s] + 4 * (self.N + sender)

    def _recv(self, s, st, sender, row_in_block):
        return (self.peer[s] + self.flag_bytes + st * (self.recv_bytes + self.out_bytes)
                + ((sender * self.max_block + row_in_block) * self.hidden) * 2)

    def _out(self, s, st, row):
        return self.peer[s] + self.flag_bytes + st * (self.recv_bytes + self.out_bytes) + self.recv_bytes + \
            row * self.hidden * 2

    def _tensor(self, ptr, rows):
        import torch

        class _View:
            pass
        v = _View()
        v.__cuda_array_interface__ = {"shape": (rows, self.hidden), "typestr": "<i2", "data": (ptr, False),
                                      "version": 3, "strides": None}
        return torch.as_tensor(v, device=self.device).view(torch.bfloat16)

    def __call__(self, attn, w_o):
        """attn [rows, H_r*D] (this rank's heads), w_o [hidden, H_r*D] (its column slice): returns the
        all-rank sum of attn @ w_o.T as a [rows, hidden] bf16 view of the output set."""
        import ctypes as C

        import torch

        from . import abi
        assert attn.shape[0] == self.rows and w_o.shape[0] == self.hidden
        N, r, sub, H = self.N, self.r, self.sub, self.hidden
        st = self.calls % 2
        base = (self.calls * sub) & 0xFFFFFFFF
        self.calls += 1
        cur = torch.cuda.current_stream(self.device)
        h = lambda s: s.cuda_stream
        for j in range(sub):
            for k in range(1, N + 1):
                o = (r + k) % N
                a, b = self.pieces[o][j]
                torch.matmul(attn[a:b], w_o.t(), out=self.partial[a:b])
                ev = torch.cuda.Event()
                ev.record(cur)
                nbytes = (b - a) * H * 2
                if o != r:
                    ss = self.s_send[o]
                    ss.wait_event(ev)
                    dst = self._recv(o, st, r, a - self.block[o][0])
                    abi.call("mllm_copy_async", dst, self.partial[a:b].data_ptr(), nbytes, h(ss))
                    abi.call("mllm_signal_u32", self._recv_flag(o, r), (base + j + 1) & 0xFFFFFFFF, h(ss))
                    continue
                # own piece: wait for the others' partials, sum, send the final rows everywhere
                self.s_reduce.wait_event(ev)
                srcs = (C.c_void_p * N)()
                for s in range(N):
                    if s == r:
                        srcs[s] = self.partial[a:b].data_ptr()
                    else:
                        abi.call("mllm_wait_u32", self._recv_flag(r, s), (base + j + 1) & 0xFFFFFFFF,
                                 h(self.s_reduce))
                        srcs[s] = self._recv(r, st, s, a - self.block[r][0])
                abi.call("mllm_sum_bf16", self._out(r, st, a), srcs, N, (b - a) * H, h(self.s_reduce))
                ev2 = torch.cuda.Event()
                ev2.record(self.s_reduce)
                for p, sg in self.s_gather.items():
                    sg.wait_event(ev2)
                    abi.call("mllm_copy_async", self._out(p, st, a), self._out(r, st, a), nbytes, h(sg))
                    abi.call("mllm_signal_u32", self._out_flag(p, r), (base + j + 1) & 0xFFFFFFFF, h(sg))
        # the output is complete once every other rank has delivered all its pieces
        cur.wait_stream(self.s_reduce)
        for s in range(N):
            if s != r:
                abi.call("mllm_wait_u32", self._out_flag(r, s), (base + sub) & 0xFFFFFFFF, h(cur))
        for st_ in list(self.s_send.values()) + list(self.s_gather.values()):
            cur.wait_stream(st_)         # the next call's GEMMs overwrite `partial`
        return self._tensor(self._out(r, st, 0), self.rows)

    def close(self):
        from . import abi
        if getattr(self, "base", None) is None:
            return
        import torch
        torch.cuda.synchronize(self.device)
        for s, p in enumerate(self.peer):
            if s != self.r:
                abi.call("mllm_ipc_close_handle", p)
        abi.call("mllm_ipc_free", self.base)
        self.base = None


def tp_attention_block(h, shard: HeadShard, head_dim: int, rope_theta: float, position_ids, kv_cache,
                       w_q, w_k, w_v, w_o, w_q_norm=None, w_k_norm=None, rms_norm_eps: float = 1e-6,
                       group=None, attention_fn=None, overlap_chunks: int = 4, exchange=None):
    """The attention half of TransformerBlock::Forward on this rank's heads, then the o_proj
    all-reduce.  Weights are this rank's slices (shard_weights); kv_cache holds only the owned
    kv heads.  Returns the full [B, S, hidden] attention output on every rank.  On the B200 path
    (attention_fn None) the o_proj GEMM and the all-reduce are overlapped chunk by chunk
    (oproj_allreduce), or, with a PeerExchange for this many rows, exchanged over NVLink copy
    engines; a given attention_fn projects itself and its result is all-reduced whole."""
    import torch.distributed as dist
    if attention_fn is None:
        from .runtime import attention_block
        B, S, _ = h.shape
        attn = attention_block(h, w_q, w_k, w_v, None, shard.num_heads, shard.num_kv_heads, head_dim, rope_theta,
                               position_ids, kv_cache, w_q_norm, w_k_norm, rms_norm_eps)
        if exchange is not None and shard.world > 1 and exchange.rows == B * S:
            return exchange(attn.reshape(B * S, -1), w_o).view(B, S, -1)
        return oproj_allreduce(attn.reshape(B * S, -1), w_o, group, overlap_chunks).view(B, S, -1)
    partial = attention_fn(h, w_q, w_k, w_v, w_o, shard.num_heads, shard.num_kv_heads, head_dim, rope_theta,
                           position_ids, kv_cache, w_q_norm, w_k_norm, rms_norm_eps)
    if shard.world > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
