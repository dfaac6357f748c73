"""Tensor-parallel attention across GPUs: KV-head-group sharding + one o_proj all-reduce.

The reference runs every layer on one device (QwenRunner.cpp:236,328); across N GPUs the
attention path shards naturally by KV-head group:

  rank r owns kv heads [r*Hkv/N, (r+1)*Hkv/N) and their n_rep query heads each, so
    w_q / w_k / w_v   row slices   (the projections of the owned heads)
    QK-norm, RoPE, KV cache, prefill / decode attention   fully local
    w_o               column slice (o_proj of the owned heads' outputs) -> a partial [B, S, hidden]
  and the partial outputs are summed by ONE all-reduce (NCCL over NVLink on GPUs), or -- the
  same exchange by token rows (SeqParallelOProj) -- the attention rows go to their row's owner,
  which runs o_proj with the whole w_o, and the output rows are all-gathered.

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
    """The o_proj exchange over NVLink peer memory: each rank's o_proj partial [T, hidden] summed
    over the ranks, every rank ending with the full sum, without an NCCL all-reduce.

    The rows are split into N owner blocks (block o belongs to rank o) of `sub` pieces each.  A
    rank computes its partial piece by piece into a buffer the other ranks can read, the pieces
    it does not own first in each round, and after each piece raises a flag in the owner's
    memory.  Once its own piece is computed, the owner waits (bounded) for the other ranks'
    flags and runs one kernel (mllm_sum_bf16) that reads the piece from every rank's buffer over
    NVLink, adds the N partials in rank order (fp32, one rounding) and stores the result into
    every rank's output buffer; then it raises a flag in each rank's memory.  So the SMs move
    the data, the transfers of one piece overlap the GEMM of the next, and NVLink carries
    partials in and final rows out at the same time.

    Buffers are CUDA IPC allocations shared once at construction (mllm_ipc_*).  Output buffers
    alternate between two sets by call parity (a returned output stays valid until the call after
    next); the partial buffer needs one copy, because a call ends only after every owner has
    stored its rows, i.e. after every read of this rank's partial.  Flags count up monotonically.
    No multicast object or load is used, and no library kernel touches a peer's memory (the GEMM
    writes this rank's own buffer)."""

    def __init__(self, rows: int, hidden: int, group=None, sub: int = 2, device=None):
        import ctypes as C

        import torch
        import torch.distributed as dist

        from . import abi
        self.lib = abi.load()
        self.group = group
        self.N = dist.get_world_size(group)
        self.r = dist.get_rank(group)
        if self.N > 8:
            raise ValueError("PeerExchange: at most 8 ranks")
        if hidden % 8 != 0:
            raise ValueError("PeerExchange: hidden must be a multiple of 8")
        self.rows, self.hidden, self.sub = rows, hidden, sub
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        N = self.N
        self.block = [(o * rows // N, (o + 1) * rows // N) for o in range(N)]
        self.pieces = {}
        for o, (a, b) in enumerate(self.block):
            self.pieces[o] = [(a + j * (b - a) // sub, a + (j + 1) * (b - a) // sub) for j in range(sub)]
        self.flag_bytes = 4096                         # ready flags [N], arrived flags [N]
        self.part_bytes = (rows * hidden * 2 + 255) // 256 * 256
        self.out_bytes = (rows * hidden * 2 + 255) // 256 * 256   # per set
        total = self.flag_bytes + self.part_bytes + 2 * self.out_bytes
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
        self.partial = self._tensor(self._part(self.r, 0), rows)
        self.s_sig = {o: torch.cuda.Stream(device=self.device) for o in range(N) if o != self.r}
        self.s_reduce = torch.cuda.Stream(device=self.device)
        self.calls = 0
        dist.barrier(group=group)

    # addresses inside rank s's shared allocation
    def _ready_flag(self, s, sender):
        return self.peer[s] + 4 * sender

    def _arrived_flag(self, s, sender):
        return self.peer[s] + 4 * (self.N + sender)

    def _part(self, s, row):
        return self.peer[s] + self.flag_bytes + row * self.hidden * 2

    def _out(self, s, st, row):
        return self.peer[s] + self.flag_bytes + self.part_bytes + st * self.out_bytes + row * self.hidden * 2

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
            flag = (base + j + 1) & 0xFFFFFFFF
            for k in range(1, N + 1):
                o = (r + k) % N
                a, b = self.pieces[o][j]
                torch.matmul(attn[a:b], w_o.t(), out=self.partial[a:b])
                ev = torch.cuda.Event()
                ev.record(cur)
                if o != r:
                    ss = self.s_sig[o]
                    ss.wait_event(ev)
                    abi.call("mllm_signal_u32", self._ready_flag(o, r), flag, h(ss))
                    continue
                # own piece: once every rank's piece is ready, pull, sum and push to every rank
                sr = self.s_reduce
                sr.wait_event(ev)
                for s in range(N):
                    if s != r:
                        abi.call("mllm_wait_u32", self._ready_flag(r, s), flag, h(sr))
                srcs = (C.c_void_p * N)(*[self._part(s, a) for s in range(N)])
                dsts = (C.c_void_p * N)(*[self._out(p, st, a) for p in range(N)])
                abi.call("mllm_sum_bf16", dsts, N, srcs, N, (b - a) * H, h(sr))
                for p in range(N):
                    if p != r:
                        abi.call("mllm_signal_u32", self._arrived_flag(p, r), flag, h(sr))
        # the output is complete once every owner has stored its rows here; that is also the
        # point after which no rank reads this rank's partial any more
        cur.wait_stream(self.s_reduce)
        for s in range(N):
            if s != r:
                abi.call("mllm_wait_u32", self._arrived_flag(r, s), (base + sub) & 0xFFFFFFFF, h(cur))
        for ss in self.s_sig.values():
            cur.wait_stream(ss)
        return self._tensor(self._out(r, st, 0), self.rows)

    def close(self):
        """Collective: every rank calls it.  Each rank unmaps the other ranks' buffers, and frees
        its own only after all ranks have unmapped it (an exported allocation must outlive every
        mapping of it)."""
        from . import abi
        if getattr(self, "base", None) is None:
            return
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize(self.device)
        for s, p in enumerate(self.peer):
            if s != self.r:
                abi.call("mllm_ipc_close_handle", p)
        dist.barrier(group=self.group)
        abi.call("mllm_ipc_free", self.base)
        self.base = None


class SeqParallelOProj:
    """The o_proj exchange by token rows instead of by partial sums.

    Head sharding leaves rank q with the attention output of its heads for every token,
    attn_q [T, Hr*D].  The all-reduce form multiplies that by w_o's column slice and sums the N
    partials [T, hidden] over the ranks: each rank sends and receives about 2 (N-1)/N of the
    partial (ring), and every output is a sum of N bf16-rounded partials.  This form moves the
    attention output instead:

      1. all-to-all: the rows of attn_q split into N blocks; block r goes to rank r, so rank r
         holds rows [r T/N, (r+1) T/N) of every rank's heads, i.e. the full [T/N, H*D] input
         of o_proj for its rows (the ranks' heads are contiguous and in rank order);
      2. one GEMM with the whole w_o (replicated, [hidden, H*D]) for those rows, written into
         this rank's slice of the output;
      3. all-gather of the slices: every rank ends with the full [T, hidden].

    Per rank that is (N-1)/N of attn_q (Hr*D wide, 1/N of the hidden size) out and in, plus
    (N-1)/N of the output in: about half the NVLink bytes of the ring all-reduce.  And every
    output row is ONE full-K GEMM, as on a single GPU, with no bf16 rounding of partials.  The
    reference's o_proj is that single GEMM (Attention.h:322-325).  T must be a multiple of N.
    Collectives run on the given torch.distributed group (NCCL), or the all-gather on a
    `Communicator` when one is given."""

    def __init__(self, rows: int, hidden: int, group=None, comm=None, device=None):
        import torch
        import torch.distributed as dist
        self.group, self.comm = group, comm
        self.N = dist.get_world_size(group)
        self.r = dist.get_rank(group)
        if rows % self.N != 0:
            raise ValueError(f"SeqParallelOProj: {rows} rows do not split over {self.N} ranks")
        self.rows, self.hidden = rows, hidden
        self.device = device or torch.device("cuda", torch.cuda.current_device())

    def __call__(self, attn, w_o):
        """attn [rows, Hr*D] (this rank's heads), w_o [hidden, H*D] (the whole weight): returns
        attn_all @ w_o.T as [rows, hidden] on every rank."""
        import torch
        import torch.distributed as dist
        N, r, T = self.N, self.r, self.rows
        Tn, Hd = T // N, attn.shape[1]
        assert attn.shape[0] == T and w_o.shape == (self.hidden, N * Hd)
        recv = torch.empty((N, Tn, Hd), dtype=attn.dtype, device=attn.device)
        dist.all_to_all_single(recv, attn.contiguous(), group=self.group)
        a = recv.permute(1, 0, 2).reshape(Tn, N * Hd)
        out = torch.empty((T, self.hidden), dtype=attn.dtype, device=attn.device)
        mine = out[r * Tn:(r + 1) * Tn]
        torch.matmul(a, w_o.t(), out=mine)
        if self.comm is not None:
            self.comm.all_gather(mine, out)
        else:
            dist.all_gather_into_tensor(out, mine, group=self.group)
        return out


class UlyssesLayout:
    """Head-parallel attention with token-parallel layer input and output.

    Tensor parallelism replicates the layer's output: every rank ends with all T rows (an
    all-reduce of partials, or an all-gather of rows), which moves about (N-1)/N of the whole
    [T, hidden] output into every GPU per layer.  In this layout rank r owns token rows
    [r T/N, (r+1) T/N) between attention blocks -- the norms, the q/k/v projections (whole
    weights) and the MLP run on those rows only -- and attention still runs on its KV-head group
    over all tokens:

      heads_from_tokens: q/k/v of my token rows, all heads [T/N, (H + 2 Hkv) D]  ->  q/k/v of
          all token rows, my heads [T, (Hr + 2 Hkvr) D]   (one all-to-all)
      attention on my heads (epilogue + prefill, unchanged)
      tokens_from_heads: attention output of my heads [T, Hr D]  ->  all heads' outputs of my
          token rows [T/N, H D]   (one all-to-all), then o_proj with the whole w_o on those rows.

    Per rank and layer that is (N-1)/N of [T/N, (H + 2 Hkv) D] and of [T, Hr D] -- for Qwen3-8B,
    T = 32768 at 8 GPUs, 44 MB and 29 MB -- instead of 235 MB or more.  Every o_proj row is one
    full-K GEMM, as on one GPU.  T must be a multiple of N; the heads' order is the ranks' order
    (shard_heads), so rank q's columns are heads [q Hr, (q+1) Hr) of q, k and v."""

    def __init__(self, shard: HeadShard, num_heads: int, num_kv_heads: int, head_dim: int, group=None):
        import torch.distributed as dist
        self.shard, self.group = shard, group
        self.N = dist.get_world_size(group)
        self.H, self.Hkv, self.D = num_heads, num_kv_heads, head_dim

    def pack_qkv_weights(self, w_q, w_k, w_v):
        """The q/k/v weights regrouped by destination rank: [N, (Hr + 2 Hkvr) D, hidden], rank q's
        block its q heads, then its k heads, then its v heads.  project() with it writes the
        all-to-all's send buffer directly."""
        import torch
        N, D = self.N, self.D
        Hr, Hkvr = self.H // N, self.Hkv // N
        blocks = []
        for q in range(N):
            blocks.append(torch.cat([w_q[q * Hr * D:(q + 1) * Hr * D], w_k[q * Hkvr * D:(q + 1) * Hkvr * D],
                                     w_v[q * Hkvr * D:(q + 1) * Hkvr * D]], 0))
        return torch.stack(blocks, 0).contiguous()

    def project(self, h_tok, w_packed):
        """q/k/v projections of this rank's token rows h_tok [T/N, hidden] with pack_qkv_weights'
        weights: the send buffer [N, T/N, (Hr + 2 Hkvr) D] of heads_from_tokens_packed."""
        import torch
        return torch.matmul(h_tok.unsqueeze(0), w_packed.transpose(1, 2))

    def heads_from_tokens_packed(self, send):
        """send [N, T/N, (Hr + 2 Hkvr) D] (block q for rank q) -> [T, (Hr + 2 Hkvr) D], every token
        row of this rank's heads, in token order: one all-to-all, no copy."""
        import torch
        import torch.distributed as dist
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv.view(-1, send.shape[2])

    def heads_from_tokens(self, qkv_tok):
        """qkv_tok [T/N, (H + 2 Hkv) D] (q | k | v of this rank's token rows) -> [T, (Hr + 2 Hkvr) D]
        (q | k | v of this rank's heads for every token row, rows in token order)."""
        import torch
        import torch.distributed as dist
        N, D = self.N, self.D
        Hr, Hkvr = self.H // N, self.Hkv // N
        Tn = qkv_tok.shape[0]
        x = qkv_tok.view(Tn, -1)
        q = x[:, :self.H * D].view(Tn, N, Hr * D)
        k = x[:, self.H * D:(self.H + self.Hkv) * D].view(Tn, N, Hkvr * D)
        v = x[:, (self.H + self.Hkv) * D:].view(Tn, N, Hkvr * D)
        send = torch.cat([q, k, v], dim=2).transpose(0, 1).contiguous()   # [N, Tn, (Hr + 2 Hkvr) D]
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv.view(N * Tn, -1)

    def tokens_from_heads(self, attn):
        """attn [T, Hr D] (this rank's heads, every token row) -> [T/N, H D] (every head, this rank's
        token rows)."""
        import torch
        import torch.distributed as dist
        N = self.N
        T, Hd = attn.shape
        recv = torch.empty((N, T // N, Hd), dtype=attn.dtype, device=attn.device)
        dist.all_to_all_single(recv, attn.contiguous(), group=self.group)
        return recv.permute(1, 0, 2).reshape(T // N, N * Hd)

    def run_sequences(self, send_of, attend, finish, count: int, side_stream=None):
        """The layer in this layout one sequence at a time, pipelined.  Here rank r owns rows
        [r S/N, (r+1) S/N) of EVERY sequence, so the moves of one sequence involve every rank
        evenly and heads_from_tokens_packed / tokens_from_heads apply to it unchanged (T = S).

          send_of(b) -> [N, S/N, (Hr + 2 Hkvr) D]: this rank's q/k/v projections of its rows of
              sequence b, grouped by destination (project() with pack_qkv_weights' weights); ready
              on the current stream when run_sequences is called;
          attend(b, qkv [S, (Hr + 2 Hkvr) D]) -> [S, Hr D]: epilogue + attention of this rank's heads
              over sequence b, on the current stream;
          finish(b, rows [S/N, H D]): this rank's rows of sequence b after attention (o_proj).

        With a side stream, sequence b+1's input all-to-all and sequence b-1's output all-to-all
        and finish run on it while sequence b is attended on the current stream; only the first
        input move and the last output move are exposed.  The current stream waits for the side
        stream before this returns.  Without one (CPU ranks) the steps run in order.  Every rank
        must call it with the same count (the collectives are matched in order)."""
        import torch
        if side_stream is None:
            for b in range(count):
                finish(b, self.tokens_from_heads(attend(b, self.heads_from_tokens_packed(send_of(b)))))
            return
        cur = torch.cuda.current_stream()
        side_stream.wait_stream(cur)
        recv, ev_in = [None] * count, [None] * count

        def move_in(b):
            with torch.cuda.stream(side_stream):
                recv[b] = self.heads_from_tokens_packed(send_of(b))
                ev_in[b] = torch.cuda.Event()
                ev_in[b].record(side_stream)

        move_in(0)
        for b in range(count):
            cur.wait_event(ev_in[b])
            recv[b].record_stream(cur)
            att = attend(b, recv[b])
            ev_att = torch.cuda.Event()
            ev_att.record(cur)
            if b + 1 < count:
                move_in(b + 1)
            side_stream.wait_event(ev_att)
            att.record_stream(side_stream)
            with torch.cuda.stream(side_stream):
                finish(b, self.tokens_from_heads(att))
            recv[b] = None
        cur.wait_stream(side_stream)


def run_micro_batches(compute, exchange, count: int, comm_stream=None):
    """Overlaps the o_proj exchange of one micro-batch with the attention of the next.

    The prefill rows of a head-sharded layer are independent per sequence, so the layer can run
    in `count` micro-batches (groups of sequences): compute(m) enqueues micro-batch m's epilogue
    and attention on the current stream; exchange(m) -- its o_proj GEMM and collective -- is
    enqueued on `comm_stream` (a high-priority stream, so its kernels take SMs as soon as the
    attention grid frees them) after an event that marks compute(m).  The exchange of micro-batch
    m therefore runs while micro-batch m + 1 computes, and only the last exchange is exposed.
    The current stream waits for every exchange before it returns.  Every rank must call it with
    the same count (the collectives are matched in order)."""
    import torch
    cur = torch.cuda.current_stream()
    if comm_stream is None:
        comm_stream = torch.cuda.Stream(device=cur.device, priority=-1)
    for m in range(count):
        compute(m)
        ev = torch.cuda.Event()
        ev.record(cur)
        comm_stream.wait_event(ev)
        with torch.cuda.stream(comm_stream):
            exchange(m)
    cur.wait_stream(comm_stream)
    return comm_stream


def tp_attention_block(h, shard: HeadShard, head_dim: int, rope_theta: float, position_ids, kv_cache,
                       w_q, w_k, w_v, w_o, w_q_norm=None, w_k_norm=None, rms_norm_eps: float = 1e-6,
                       group=None, attention_fn=None, overlap_chunks: int = 4, exchange=None, comm=None):
    """The attention half of TransformerBlock::Forward on this rank's heads, then the o_proj
    all-reduce.  Weights are this rank's slices (shard_weights); kv_cache holds only the owned
    kv heads.  Returns the full [B, S, hidden] attention output on every rank.  On the B200 path
    (attention_fn None) the o_proj exchange is, by what the caller passes:
      - an `exchange` built for this many rows: a PeerExchange (an SM kernel pulls the partials
        over NVLink peer memory, sums them and pushes the rows back, mllm_sum_bf16) with w_o this
        rank's column slice, or a SeqParallelOProj with w_o the WHOLE weight;
      - a `comm` (Communicator): the column-slice GEMM, then one mllm_comm_all_reduce_bf16;
      - otherwise the GEMM and torch.distributed's all-reduce overlapped chunk by chunk
        (oproj_allreduce).
    A given attention_fn projects itself and its result is all-reduced whole."""
    import torch.distributed as dist
    if attention_fn is None:
        import torch

        from .runtime import attention_block
        B, S, _ = h.shape
        attn = attention_block(h, w_q, w_k, w_v, None, shard.num_heads, shard.num_kv_heads, head_dim, rope_theta,
                               position_ids, kv_cache, w_q_norm, w_k_norm, rms_norm_eps)
        if exchange is not None and shard.world > 1 and exchange.rows == B * S:
            return exchange(attn.reshape(B * S, -1), w_o).view(B, S, -1)
        if comm is not None and shard.world > 1:
            part = torch.matmul(attn.reshape(B * S, -1), w_o.t())
            return comm.all_reduce(part).view(B, S, -1)
        return oproj_allreduce(attn.reshape(B * S, -1), w_o, group, overlap_chunks).view(B, S, -1)
    partial = attention_fn(h, w_q, w_k, w_v, w_o, shard.num_heads, shard.num_kv_heads, head_dim, rope_theta,
                           position_ids, kv_cache, w_q_norm, w_k_norm, rms_norm_eps)
    if shard.world > 1:
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial
