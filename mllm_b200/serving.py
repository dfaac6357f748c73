"""Batched generation over the paged KV cache: the serving loop the reference plans but does not
have.  Its `Generate` runs one sequence at a time (QwenRunner.cpp:420-545, LlamaRunner.cpp:283-386:
batch 1, a host sync per token in Sampler.cpp:105-109) and its `Scheduler` feeds it one request at
a time (Scheduler.cpp:45-77).  Here requests of any length share the GPU:

  * every layer has one `PagedKVCache`; the live sequences always occupy block-table rows
    0..n-1, so one decode step over all of them is one fused decode launch per layer
    (`mllm_decode_step_paged_bf16`, per-sequence lengths and positions);
  * a request joins when a row is free and every layer has blocks for its whole length (prompt
    plus new tokens), so a running request is never preempted; the prompts that join in one
    step are prefilled together, packed back to back, into rows n.. through a view of those rows
    (`PagedSlot`): one projection, epilogue and attention launch per layer for all of them
    (`mllm_qkv_epilogue_varlen_paged_bf16`, `mllm_prefill_attention_varlen_paged_bf16`);
  * a finished request's blocks go back to the pools and the last live row moves into its row
    (`PagedKVCache.move`: a block-table row copy, no K/V copy);
  * the next tokens of all live rows come from one device sampler call (`mllm_sample`) and one
    device-to-host read per step;
  * while the batch keeps its size, the decode step replays a CUDA graph recorded for that size
    (`DecodeGraph`): one launch per step instead of several hundred.

`DecoderModel` is the layer stack of TransformerBlock::Forward (TransformerBlock.h:51-195) with
the reference's RMSNorm (RMSNorm.h:27-64) and SwiGLU MLP (MLP.h:31-43) as LibTorch ops, the
attention step through this package's kernels, and QwenRunner::Forward's embedding, final norm
and lm_head (QwenRunner.cpp:285-418).  Its weights are random (there is no checkpoint here).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import runtime as rt


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm::Forward (RMSNorm.h:27-64): fp32 x * rsqrt(mean(x^2) + eps) * w, cast back."""
    xf = x.float()
    out = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    return out.to(x.dtype)


def swiglu_mlp(x, w_gate, w_up, w_down):
    """MLP::Forward (MLP.h:31-43): down(gate * sigmoid(gate) * up); FP8 weights through
    runtime.linear_fp8."""
    gate = rt._linear(x, w_gate)
    up = rt._linear(x, w_up)
    return rt._linear(gate * torch.sigmoid(gate) * up, w_down)


@dataclass
class DecoderShape:
    vocab: int = 4096
    hidden: int = 1024
    layers: int = 4
    heads: int = 8
    kv_heads: int = 2
    head_dim: int = 128
    intermediate: int = 2816
    rope_theta: float = 1e6
    eps: float = 1e-6
    qk_norm: bool = True          # Qwen3 (True) or Llama (False) attention branch


class DecoderModel:
    """Random-init decoder (Qwen3 or Llama layout) whose attention step runs on the B200 path."""

    def __init__(self, shape: DecoderShape, seed: int = 0, device="cuda", fp8: bool = False):
        """fp8: every projection (q/k/v/o and the MLP) held as e4m3 with 128 x 128 block scales,
        the layout of FP8 checkpoints, and multiplied as stored (runtime.linear_fp8)."""
        self.s = shape
        g = torch.Generator(device=device).manual_seed(seed)
        E, H, Hkv, D, I = shape.hidden, shape.heads, shape.kv_heads, shape.head_dim, shape.intermediate

        def w(*size, scale=0.02):
            return (scale * torch.randn(*size, device=device, generator=g)).bfloat16()

        def gamma(n):
            return (1 + 0.1 * torch.randn(n, device=device, generator=g)).bfloat16()

        self.embed = w(shape.vocab, E, scale=1.0)
        self.lm_head = w(shape.vocab, E)
        self.norm = gamma(E)
        self.layers = []
        for _ in range(shape.layers):
            self.layers.append({
                "ln1": gamma(E), "ln2": gamma(E),
                "w_q": w(H * D, E), "w_k": w(Hkv * D, E), "w_v": w(Hkv * D, E), "w_o": w(E, H * D),
                "q_norm": gamma(D) if shape.qk_norm else None, "k_norm": gamma(D) if shape.qk_norm else None,
                "w_gate": w(I, E), "w_up": w(I, E), "w_down": w(E, I)})
        if fp8:
            for lw in self.layers:
                for name in ("w_q", "w_k", "w_v", "w_o", "w_gate", "w_up", "w_down"):
                    lw[name] = rt.Fp8Weight.quantize(lw[name])

    def dequantized(self) -> "DecoderModel":
        """The same model with every FP8 projection dequantized the reference's way
        (DequantizeFP8, QwenRunner.cpp:103-122): what the reference runner multiplies."""
        import copy
        m = copy.copy(self)
        m.layers = [{k: (v.dequantize() if isinstance(v, rt.Fp8Weight) else v) for k, v in lw.items()}
                    for lw in self.layers]
        return m

    def new_caches(self, num_blocks: int, block_size: int = 256, max_seqs: int = 64,
                   max_blocks_per_seq: int | None = None):
        return [rt.PagedKVCache(num_blocks, self.s.kv_heads, self.s.head_dim, block_size, max_seqs,
                                max_blocks_per_seq, device=self.embed.device) for _ in self.layers]

    def forward(self, ids: torch.Tensor, positions: torch.Tensor, caches) -> torch.Tensor:
        """ids int64 [B, S]; positions int64 [S] (shared) or [B] (one new token per sequence);
        caches: one KV cache per layer.  Returns the fp32 logits of each sequence's last row
        [B, vocab]."""
        s = self.s
        h = self.embed[ids]
        for lw, cache in zip(self.layers, caches):
            x = rms_norm(h, lw["ln1"], s.eps)
            h = h + rt.attention_block(x, lw["w_q"], lw["w_k"], lw["w_v"], lw["w_o"], s.heads, s.kv_heads,
                                       s.head_dim, s.rope_theta, positions, cache, lw["q_norm"], lw["k_norm"],
                                       s.eps)
            x = rms_norm(h, lw["ln2"], s.eps)
            h = h + swiglu_mlp(x, lw["w_gate"], lw["w_up"], lw["w_down"])
        x = rms_norm(h[:, -1], self.norm, s.eps)
        return torch.nn.functional.linear(x, self.lm_head).float()

    def forward_packed(self, ids: torch.Tensor, q_lens: list[int], caches) -> torch.Tensor:
        """Several prompts in one pass: ids int64 [T] holds them back to back (prompt b the next
        q_lens[b] tokens, appended to cache sequence b at its current length).  Returns the fp32
        logits of each prompt's last row [len(q_lens), vocab]."""
        s = self.s
        h = self.embed[ids]
        for lw, cache in zip(self.layers, caches):
            x = rms_norm(h, lw["ln1"], s.eps)
            h = h + rt.attention_block_packed(x, lw["w_q"], lw["w_k"], lw["w_v"], lw["w_o"], s.heads, s.kv_heads,
                                              s.head_dim, s.rope_theta, q_lens, cache, lw["q_norm"], lw["k_norm"],
                                              s.eps)
            x = rms_norm(h, lw["ln2"], s.eps)
            h = h + swiglu_mlp(x, lw["w_gate"], lw["w_up"], lw["w_down"])
        last = torch.tensor([sum(q_lens[:b + 1]) - 1 for b in range(len(q_lens))], device=h.device)
        x = rms_norm(h[last], self.norm, s.eps)
        return torch.nn.functional.linear(x, self.lm_head).float()


class DecodeGraph:
    """One decode step of `n` live rows (embedding, every layer, final norm, lm_head) recorded
    once as a CUDA graph and then replayed each step: the host issues one graph launch instead of
    the step's several hundred kernel launches.  A replay is valid while the batch has exactly n
    rows, every row's cache length stays below `max_len` (the decode plan recorded in the graph)
    and its blocks are reserved; block-table rows may change between replays, since the kernels
    read the tables from device memory.  The caches' device lengths advance inside the graph;
    the caller advances their host copies after each replay (PagedKVCache.advance_host)."""

    def __init__(self, model, caches, n: int, max_len: int):
        dev = model.embed.device
        self.n, self.max_len = n, max_len
        self.ids = torch.zeros((n, 1), dtype=torch.int64, device=dev)
        self.pos = torch.zeros(n, dtype=torch.int64, device=dev)
        self.scratch = rt.GraphScratch()
        self.graph = torch.cuda.CUDAGraph()
        for c in caches:
            c.capture_max_len = max_len
        try:
            with rt.graph_scratch(self.scratch), torch.cuda.graph(self.graph):
                self.logits = model.forward(self.ids, self.pos, caches)
        finally:
            for c in caches:
                c.capture_max_len = None

    def replay(self, ids: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """ids int64 [n, 1], pos int64 [n] -> the logits [n, vocab] (overwritten by the next
        replay)."""
        self.ids.copy_(ids)
        self.pos.copy_(pos)
        self.graph.replay()
        return self.logits


@dataclass
class Request:
    rid: int
    prompt: list[int]
    max_new_tokens: int
    eos: int | None = None
    tokens: list[int] = field(default_factory=list)
    logits: list[torch.Tensor] = field(default_factory=list)   # kept when record_logits is set

    @property
    def rows(self) -> int:
        """Cache rows the request can need: prompt plus generated tokens (the last one is never fed)."""
        return len(self.prompt) + self.max_new_tokens


class ContinuousBatcher:
    """Greedy batched generation with requests joining and leaving between steps (see the module
    docstring).  `model` provides forward(ids, positions, caches) -> [B, vocab] logits and
    new_caches(num_blocks, block_size, max_seqs, max_blocks_per_seq)."""

    def __init__(self, model, max_batch: int, num_blocks: int, block_size: int = 256,
                 max_blocks_per_seq: int | None = None, record_logits: bool = False, graphs: bool = True,
                 max_graphs: int = 8):
        self.model = model
        # CUDA graphs of the decode step, one per batch size, recorded when a size repeats
        emb = getattr(model, "embed", None)
        self.graphs = graphs and emb is not None and emb.is_cuda
        self.max_graphs = max_graphs
        self._graphs: dict[int, DecodeGraph] = {}
        self._last_n = 0
        self.graph_steps = 0   # decode steps that replayed a recorded graph
        self.max_batch = max_batch
        self.caches = model.new_caches(num_blocks, block_size, max_batch, max_blocks_per_seq)
        self.block_size = block_size
        self.record_logits = record_logits
        self.waiting: list[Request] = []
        self.live: list[Request] = []          # live[i] occupies row i of every cache
        self.done: dict[int, Request] = {}
        self._next_id = 0
        self.steps = 0

    def submit(self, prompt, max_new_tokens: int, eos: int | None = None) -> int:
        if len(prompt) == 0 or max_new_tokens < 1:
            raise ValueError("a request needs a prompt and at least one new token")
        r = Request(self._next_id, list(prompt), max_new_tokens, eos)
        need = -(-r.rows // self.block_size)
        if need > self.caches[0].max_blocks_per_seq or need > self.caches[0].num_blocks:
            raise ValueError("request longer than one sequence's cache can hold")
        self._next_id += 1
        self.waiting.append(r)
        return r.rid

    def _pick(self, logits: torch.Tensor) -> list[int]:
        if logits.is_cuda:
            return rt.sample(logits, use_greedy=True).tolist()
        return logits.argmax(-1).tolist()

    def _emit(self, r: Request, token: int, logits_row) -> None:
        r.tokens.append(token)
        if self.record_logits:
            r.logits.append(logits_row.detach().float().cpu())

    def _finished(self, r: Request) -> bool:
        return len(r.tokens) >= r.max_new_tokens or (r.eos is not None and r.tokens and r.tokens[-1] == r.eos)

    def _admit(self) -> None:
        dev = self.model.embed.device if hasattr(self.model, "embed") else "cpu"
        first = len(self.live)
        joined: list[Request] = []
        while self.waiting and first + len(joined) < self.max_batch:
            r = self.waiting[0]
            need = -(-r.rows // self.block_size)
            if any(c.free_blocks < need for c in self.caches):
                break                        # first come, first served: wait for blocks
            self.waiting.pop(0)
            row = first + len(joined)
            for c in self.caches:
                c.reserve(row, r.rows)       # the whole request's blocks, up front
            joined.append(r)
        if not joined:
            return
        if hasattr(self.model, "forward_packed"):
            # every joining prompt in one pass: rows first .. first+k-1, one launch per kernel
            views = [c.slot(first, len(joined)) for c in self.caches]
            ids = torch.tensor([t for r in joined for t in r.prompt], dtype=torch.int64, device=dev)
            logits = self.model.forward_packed(ids, [len(r.prompt) for r in joined], views)
        else:
            rows = []
            for i, r in enumerate(joined):
                views = [c.slot(first + i) for c in self.caches]
                ids = torch.tensor([r.prompt], dtype=torch.int64, device=dev)
                pos = torch.arange(len(r.prompt), dtype=torch.int64, device=dev)
                rows.append(self.model.forward(ids, pos, views))
            logits = torch.cat(rows)
        for r, t, row in zip(joined, self._pick(logits), logits):
            self._emit(r, t, row)
            self.live.append(r)

    def _retire(self) -> None:
        i = 0
        while i < len(self.live):
            r = self.live[i]
            if not self._finished(r):
                i += 1
                continue
            self.done[r.rid] = r
            last = len(self.live) - 1
            for c in self.caches:
                c.release(i)
                if i != last:
                    c.move(last, i)
            self.live[i] = self.live[last]
            self.live.pop()

    def step(self) -> None:
        """Retire finished requests, admit waiting ones (prefill), then one decode step for all
        live rows."""
        self._retire()
        self._admit()
        self._retire()                       # a request may finish with its first token
        if not self.live:
            return
        dev = self.model.embed.device if hasattr(self.model, "embed") else "cpu"
        n = len(self.live)
        ids = torch.tensor([[r.tokens[-1]] for r in self.live], dtype=torch.int64, device=dev)
        lens = self.caches[0].host_lengths()[:n]
        pos = torch.tensor(lens, dtype=torch.int64, device=dev)   # the new token's position
        g = self._decode_graph(n)
        if g is not None:
            logits = g.replay(ids, pos)
            for c in self.caches:
                c.advance_host(1, n)
            self.graph_steps += 1
        else:
            logits = self.model.forward(ids, pos, self.caches)
        for r, t, row in zip(self.live, self._pick(logits), logits):
            self._emit(r, t, row)
        self.steps += 1

    def _decode_graph(self, n: int):
        """The recorded decode step for n rows, recorded now if the previous step had n rows too
        (a batch that keeps its size); None: run the step eagerly."""
        if not self.graphs:
            return None
        repeat, self._last_n = self._last_n == n, n
        # every live row stays below its request's rows; round up so that one graph serves a while
        need = max(r.rows for r in self.live)
        bound = min(-(-need // 256) * 256, self.caches[0].capacity)
        g = self._graphs.get(n)
        if g is not None and g.max_len >= need:
            return g
        if not repeat:
            return None
        self._graphs.pop(n, None)
        while len(self._graphs) >= self.max_graphs:
            self._graphs.pop(next(iter(self._graphs)))
        g = DecodeGraph(self.model, self.caches, n, bound)
        self._graphs[n] = g
        return g

    def run(self) -> dict[int, list[int]]:
        """Step until every submitted request has finished; returns the tokens of each."""
        while self.waiting or self.live:
            before = (len(self.waiting), len(self.live))
            self.step()
            if not self.live and self.waiting and (len(self.waiting), len(self.live)) == before:
                raise RuntimeError("a waiting request can never be admitted")
        return {rid: r.tokens for rid, r in sorted(self.done.items())}
