"""Tensor-parallel host logic on CPU: 2 gloo ranks, each computing its KV-head group's attention
with the numpy oracle (as a stand-in compute backend for the test) plus its partial o_proj,
summed by the all-reduce, must equal the unsharded oracle layer (prefill then decode steps)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mllm_b200 import tp
from oracle import attention_oracle as O
from tests.golden.cases import case_by_name, make_inputs


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_attention_fn(caches):
    """attention_fn backed by the oracle (test only): same signature as runtime.attention_block."""
    def fn(h, w_q, w_k, w_v, w_o, H, Hkv, D, theta, pos, cache_key, gq, gk, eps):
        x = h.numpy()
        q, k, v = O.qwen_qkv_prologue(x, w_q.numpy(), w_k.numpy(), w_v.numpy(), gq.numpy(), gk.numpy(), H, Hkv, D, eps)
        out = O.attention_forward_projected(q, k, v, w_o.numpy(), H, Hkv, D, theta, pos.numpy(), caches[cache_key])
        return torch.from_numpy(np.ascontiguousarray(out))
    return fn


def _worker(rank, world, port, case_name, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        c = case_by_name(case_name)
        inp = make_inputs(c)
        shard = tp.shard_heads(c.num_heads, c.num_kv_heads, world, rank)
        T = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in inp.items()}
        wq, wk, wv, wo = tp.shard_weights(shard, c.head_dim, T["w_q"], T["w_k"], T["w_v"], T["w_o"])
        caches = {"layer0": O.KVCache()}
        fn = _oracle_attention_fn(caches)
        outs = []
        steps = [inp["hidden"]] + [inp["decode_hidden"][i] for i in range(c.decode_steps)]
        for i, x in enumerate(steps):
            S = x.shape[1]
            pos = np.array([caches["layer0"].key.shape[2]]) if i > 0 else np.arange(S)
            out = tp.tp_attention_block(torch.from_numpy(x), shard, c.head_dim, c.rope_theta, torch.from_numpy(pos),
                                        "layer0", wq, wk, wv, wo, T["w_q_norm"], T["w_k_norm"], c.eps,
                                        attention_fn=fn)
            outs.append(out.numpy())
        q.put((rank, outs, caches["layer0"].key.shape))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case_name", ["qwen_d128_gqa4"])
def test_two_rank_head_sharding_matches_unsharded(case_name):
    c = case_by_name(case_name)
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, outs, kshape = q.get(timeout=120)
        res[rank] = (outs, kshape)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # unsharded oracle layer
    inp = make_inputs(c)
    cache = O.KVCache()
    steps = [inp["hidden"]] + [inp["decode_hidden"][i] for i in range(c.decode_steps)]
    for i, x in enumerate(steps):
        S = x.shape[1]
        pos = np.array([cache.key.shape[2]]) if i > 0 else np.arange(S)
        qq, kk, vv = O.qwen_qkv_prologue(x, inp["w_q"], inp["w_k"], inp["w_v"], inp["w_q_norm"], inp["w_k_norm"],
                                         c.num_heads, c.num_kv_heads, c.head_dim, c.eps)
        ref = O.attention_forward_projected(qq, kk, vv, inp["w_o"], c.num_heads, c.num_kv_heads, c.head_dim,
                                            c.rope_theta, pos, cache)
        for r in range(world):
            np.testing.assert_allclose(res[r][0][i], ref, rtol=1e-4, atol=1e-5, err_msg=f"rank {r} step {i}")
    # each rank's cache holds only its kv heads
    for r in range(world):
        assert res[r][1][1] == c.num_kv_heads // world


def test_shard_heads_layout():
    s = [tp.shard_heads(32, 8, 4, r) for r in range(4)]
    assert [x.kv_heads for x in s] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    assert [x.q_heads for x in s] == [(0, 8), (8, 16), (16, 24), (24, 32)]
    assert tp.shard_heads(40, 8, 8, 7).q_heads == (35, 40)   # Qwen3-14B: one kv head (5 q heads) per GPU
    with pytest.raises(RuntimeError, match="do not split"):
        tp.shard_heads(32, 8, 3, 0)
    with pytest.raises(RuntimeError, match="divisible"):
        tp.shard_heads(30, 8, 2, 0)


def _oproj_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        attn_full = torch.randn(37, 2 * 48, generator=g)          # 37 rows, 2 ranks x 48 columns
        w_o_full = torch.randn(64, 2 * 48, generator=g)
        sl = slice(rank * 48, (rank + 1) * 48)
        out = tp.oproj_allreduce(attn_full[:, sl].contiguous(), w_o_full[:, sl].contiguous(), chunks=5)
        q.put((rank, out.numpy(), (attn_full @ w_o_full.t()).numpy()))
    finally:
        dist.destroy_process_group()


def test_oproj_allreduce_chunks_equal_the_whole_exchange():
    """o_proj in row pieces, each piece all-reduced asynchronously while the next piece's GEMM
    runs: every rank holds the full projection (2 gloo ranks, 37 rows in 5 pieces)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_oproj_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, out, ref in res:
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-4, err_msg=f"rank {rank}")


def _seqpar_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, E, H, D = 24, 64, 8, 16
        g = torch.Generator().manual_seed(7)
        attn_all = torch.randn(T, H * D, generator=g)          # every head's attention rows
        w_o = torch.randn(E, H * D, generator=g) * 0.1
        shard = tp.shard_heads(H, H // 2, world, rank)
        mine = attn_all[:, shard.q_heads[0] * D:shard.q_heads[1] * D].contiguous()
        ex = tp.SeqParallelOProj(T, E, device=torch.device("cpu"))
        out = ex(mine, w_o)
        q.put((rank, out.numpy(), (attn_all @ w_o.t()).numpy()))
    finally:
        dist.destroy_process_group()


def test_sequence_parallel_oproj_equals_unsharded():
    """SeqParallelOProj (all-to-all of the attention rows, full-K o_proj per row block,
    all-gather): every rank holds the unsharded o_proj output, each row one full-K GEMM."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_seqpar_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, got, want in res:
        np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-5, err_msg=f"rank {r}")


def _ulysses_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, H, Hkv, D = 16, 8, 4, 8
        g = torch.Generator().manual_seed(11)
        qkv_all = torch.randn(T, (H + 2 * Hkv) * D, generator=g)     # every token's q | k | v
        shard = tp.shard_heads(H, Hkv, world, rank)
        lay = tp.UlyssesLayout(shard, H, Hkv, D)
        Tn = T // world
        mine = qkv_all[rank * Tn:(rank + 1) * Tn]
        heads = lay.heads_from_tokens(mine)
        # the expected rows: q | k | v columns of this rank's heads, every token
        q0, q1 = shard.q_heads[0] * D, shard.q_heads[1] * D
        k0, k1 = shard.kv_heads[0] * D, shard.kv_heads[1] * D
        want = torch.cat([qkv_all[:, q0:q1], qkv_all[:, H * D + k0:H * D + k1],
                          qkv_all[:, (H + Hkv) * D + k0:(H + Hkv) * D + k1]], 1)
        attn_all = torch.randn(T, H * D, generator=g)                 # every head's attention rows
        back = lay.tokens_from_heads(attn_all[:, q0:q1].contiguous())
        q.put((rank, torch.equal(heads, want), torch.equal(back, attn_all[rank * Tn:(rank + 1) * Tn])))
    finally:
        dist.destroy_process_group()


def test_ulysses_layout_moves_rows_between_token_and_head_owners():
    """UlyssesLayout: q/k/v of token rows to the owners of their heads, and attention rows back to
    the owners of their tokens, exactly (2 gloo ranks)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ulysses_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, heads_ok, back_ok in res:
        assert heads_ok and back_ok, r


def _ulysses_packed_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, E, H, Hkv, D = 16, 24, 8, 4, 8
        g = torch.Generator().manual_seed(12)
        h = torch.randn(T, E, generator=g)
        w_q, w_k, w_v = (torch.randn(n * D, E, generator=g) for n in (H, Hkv, Hkv))
        shard = tp.shard_heads(H, Hkv, world, rank)
        lay = tp.UlyssesLayout(shard, H, Hkv, D)
        Tn = T // world
        got = lay.heads_from_tokens_packed(lay.project(h[rank * Tn:(rank + 1) * Tn],
                                                       lay.pack_qkv_weights(w_q, w_k, w_v)))
        q0, q1 = shard.q_heads[0] * D, shard.q_heads[1] * D
        k0, k1 = shard.kv_heads[0] * D, shard.kv_heads[1] * D
        want = torch.cat([h @ w_q[q0:q1].t(), h @ w_k[k0:k1].t(), h @ w_v[k0:k1].t()], 1)
        q.put((rank, float((got - want).abs().max())))
    finally:
        dist.destroy_process_group()


def test_ulysses_packed_projection_lands_on_the_head_owners():
    """UlyssesLayout.project with pack_qkv_weights writes the all-to-all's send buffer directly;
    after heads_from_tokens_packed every rank holds its heads' q/k/v for every token row."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ulysses_packed_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, err in res:
        assert err < 1e-5, (r, err)


def _ulysses_seq_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, S, E, H, Hkv, D = 3, 8, 24, 8, 4, 8
        g = torch.Generator().manual_seed(13)
        h = torch.randn(B, S, E, generator=g)
        w_q, w_k, w_v = (torch.randn(n * D, E, generator=g) for n in (H, Hkv, Hkv))
        w_o = torch.randn(E, H * D, generator=g)
        shard = tp.shard_heads(H, Hkv, world, rank)
        lay = tp.UlyssesLayout(shard, H, Hkv, D)
        Sn = S // world
        w_packed = lay.pack_qkv_weights(w_q, w_k, w_v)
        q0, q1 = shard.q_heads[0] * D, shard.q_heads[1] * D
        k0, k1 = shard.kv_heads[0] * D, shard.kv_heads[1] * D
        # a stand-in for attention that mixes every row of the sequence (so that a row taken from
        # the wrong sequence or position shows): q * (row-sum of k) + cumulative sum of v per head
        def attend(b, qkv):
            Hr, Hkvr = shard.num_heads, shard.num_kv_heads
            qq = qkv[:, :Hr * D].view(S, Hr, D)
            kk = qkv[:, Hr * D:(Hr + Hkvr) * D].view(S, Hkvr, D).repeat_interleave(Hr // Hkvr, 1)
            vv = qkv[:, (Hr + Hkvr) * D:].view(S, Hkvr, D).repeat_interleave(Hr // Hkvr, 1)
            return (qq * kk.sum(0, keepdim=True) + vv.cumsum(0)).reshape(S, Hr * D)
        out = torch.empty(B, Sn, E)

        def finish(b, rows):
            out[b] = rows @ w_o.t()
        lay.run_sequences(lambda b: lay.project(h[b, rank * Sn:(rank + 1) * Sn], w_packed), attend, finish, B)
        # the same on one process: every head, every sequence
        want = torch.empty(B, Sn, E)
        for b in range(B):
            qa, ka, va = h[b] @ w_q.t(), h[b] @ w_k.t(), h[b] @ w_v.t()
            qq = qa.view(S, H, D)
            kk = ka.view(S, Hkv, D).repeat_interleave(H // Hkv, 1)
            vv = va.view(S, Hkv, D).repeat_interleave(H // Hkv, 1)
            att = (qq * kk.sum(0, keepdim=True) + vv.cumsum(0)).reshape(S, H * D)
            want[b] = (att @ w_o.t())[rank * Sn:(rank + 1) * Sn]
        q.put((rank, float((out - want).abs().max() / want.abs().max())))
    finally:
        dist.destroy_process_group()


def test_ulysses_per_sequence_pipeline_gives_each_rank_its_rows():
    """UlyssesLayout.run_sequences (rank r owns rows [r S/N, (r+1) S/N) of every sequence): each
    sequence's q/k/v reach the head owners, the per-head results come back to the row owners and
    every rank ends with its rows of every sequence, as one process computing all heads would
    (2 gloo ranks, 3 sequences)."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ulysses_seq_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r, err in res:
        assert err < 1e-5, (r, err)
