"""Tensor parallelism on the B200 path: 2 NCCL ranks, each running its KV-head group's attention
(prefill, then fused decode steps) with the o_proj exchange overlapped chunk by chunk
(mllm_b200.tp.oproj_allreduce) or run over NVLink copy engines (mllm_b200.tp.PeerExchange),
against the unsharded layer on one GPU.  Needs 2 GPUs (skipped
otherwise)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(E, H, Hkv, D, device):
    g = torch.Generator(device=device).manual_seed(0)
    r = lambda *shape: (0.02 * torch.randn(*shape, device=device, generator=g)).bfloat16()
    return {"w_q": r(H * D, E), "w_k": r(Hkv * D, E), "w_v": r(Hkv * D, E), "w_o": r(E, H * D),
            "gq": (1 + 0.1 * torch.randn(D, device=device, generator=g)).bfloat16(),
            "gk": (1 + 0.1 * torch.randn(D, device=device, generator=g)).bfloat16()}


def _inputs(B, S, E, steps, device):
    g = torch.Generator(device=device).manual_seed(1)
    return [torch.randn(B, S, E, device=device, generator=g).bfloat16()] + \
           [torch.randn(B, 1, E, device=device, generator=g).bfloat16() for _ in range(steps)]


def _worker(rank, world, port, q, mode):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from mllm_b200 import runtime as rt, tp
        B, S, E, H, Hkv, D, steps = 2, 300, 512, 8, 4, 128, 3
        w = _weights(E, H, Hkv, D, dev)
        xs = _inputs(B, S, E, steps, dev)
        shard = tp.shard_heads(H, Hkv, world, rank)
        wq, wk, wv, wo = tp.shard_weights(shard, D, w["w_q"], w["w_k"], w["w_v"], w["w_o"])
        cache = rt.KVCache(B, shard.num_kv_heads, D, S + steps)
        ex = {B * S: tp.PeerExchange(B * S, E), B: tp.PeerExchange(B, E, sub=1)} if mode == "peer" else {}
        outs = []
        for i, x in enumerate(xs):
            pos = torch.arange(S, device=dev) if i == 0 else torch.tensor([S + i - 1], device=dev)
            outs.append(tp.tp_attention_block(x, shard, D, 1e6, pos, cache, wq, wk, wv, wo, w["gq"], w["gk"],
                                              1e-6, overlap_chunks=3,
                                              exchange=ex.get(x.shape[0] * x.shape[1])).float().cpu().numpy())
        for e in ex.values():
            e.close()
        q.put((rank, outs))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("mode", ["chunked", "peer"])
def test_two_rank_layer_matches_unsharded(mode):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from mllm_b200 import runtime as rt
    dev = torch.device("cuda", 0)
    B, S, E, H, Hkv, D, steps = 2, 300, 512, 8, 4, 128, 3
    w = _weights(E, H, Hkv, D, dev)
    xs = _inputs(B, S, E, steps, dev)
    cache = rt.KVCache(B, Hkv, D, S + steps)
    for i, x in enumerate(xs):
        pos = torch.arange(S, device=dev) if i == 0 else torch.tensor([S + i - 1], device=dev)
        ref = rt.attention_block(x, w["w_q"], w["w_k"], w["w_v"], w["w_o"], H, Hkv, D, 1e6, pos, cache,
                                 w["gq"], w["gk"], 1e-6).float().cpu().numpy()
        for r in range(world):
            np.testing.assert_allclose(res[r][i], ref, rtol=2e-2, atol=2e-2, err_msg=f"rank {r} step {i}")


def _exchange_worker(rank, world, port, q):
    """Each rank holds a seeded partial attn @ w_o.T; PeerExchange must return the all-rank sum,
    the same bits on every rank and the bits of NCCL's all-reduce of the same partials (at two
    ranks both add two bf16 values in fp32 and round once)."""
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from mllm_b200 import abi, tp
        torch.matmul(torch.ones(8, 8, device=dev), torch.ones(8, 8, device=dev))   # library set-up first
        torch.cuda.synchronize()
        out = {}
        for rows, hidden, k, sub in ((600, 512, 512, 2), (2, 4096, 2048, 1), (257, 1024, 256, 3)):
            ex = tp.PeerExchange(rows, hidden, sub=sub)
            g = torch.Generator(device=dev).manual_seed(100 + rank)
            got, want, keep = [], [], []
            for call in range(5):
                attn = torch.randn(rows, k, device=dev, generator=g).bfloat16()
                w_o = (0.05 * torch.randn(hidden, k, device=dev, generator=g)).bfloat16()
                y = ex(attn, w_o)
                keep.append(y)
                # what the same ranks get from the library all-reduce of the same per-piece GEMMs
                part = torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16)
                for o in range(world):
                    for a, b in ex.pieces[o]:
                        torch.matmul(attn[a:b], w_o.t(), out=part[a:b])
                dist.all_reduce(part)
                got.append(y.clone().cpu())
                want.append(part.cpu())
                if call >= 1:   # the previous call's output is still intact
                    assert torch.equal(keep[call - 1].cpu(), got[call - 1])
            torch.cuda.synchronize()
            assert abi.load().mllm_attn_device_status(None) == 0
            ex.close()
            out[(rows, hidden)] = (torch.stack(got).view(torch.int16).numpy(),
                                   torch.stack(want).view(torch.int16).numpy())
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_exchange_matches_nccl_allreduce():
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for key in res[0]:
        got0, want0 = res[0][key]
        got1, _ = res[1][key]
        np.testing.assert_array_equal(got0, got1, err_msg=f"{key}: ranks disagree")
        np.testing.assert_array_equal(got0, want0, err_msg=f"{key}: differs from NCCL all-reduce")


def _exchange_worker_n(rank, world, port, q):
    """PeerExchange at `world` ranks: every rank holds the same result, equal to the fp32 sum of
    the ranks' bf16 partials (in rank order) rounded once."""
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from mllm_b200 import abi, tp
        torch.matmul(torch.ones(8, 8, device=dev), torch.ones(8, 8, device=dev))
        torch.cuda.synchronize()
        rows, hidden, k = 1000, 1024, 256
        ex = tp.PeerExchange(rows, hidden, sub=2)
        got = []
        parts = []
        for call in range(4):
            g = torch.Generator(device=dev).manual_seed(1000 * call + rank)
            attn = torch.randn(rows, k, device=dev, generator=g).bfloat16()
            w_o = (0.05 * torch.randn(hidden, k, device=dev, generator=g)).bfloat16()
            part = torch.empty(rows, hidden, device=dev, dtype=torch.bfloat16)
            for o in range(world):
                for a, b in ex.pieces[o]:
                    torch.matmul(attn[a:b], w_o.t(), out=part[a:b])
            y = ex(attn, w_o)
            got.append(y.clone().cpu())
            parts.append(part.cpu())
        torch.cuda.synchronize()
        assert abi.load().mllm_attn_device_status(None) == 0
        ex.close()
        q.put((rank, torch.stack(got).view(torch.int16).numpy(), torch.stack(parts).float().numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 3, reason="needs 3+ GPUs")
def test_peer_exchange_on_all_gpus():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker_n, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, got, part = q.get(timeout=300)
        res[r] = (got, part)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(1, world):
        np.testing.assert_array_equal(res[r][0], res[0][0], err_msg=f"rank {r} differs from rank 0")
    acc = np.zeros_like(res[0][1])
    for r in range(world):
        acc = acc + res[r][1]          # fp32, rank order
    want = torch.from_numpy(acc).bfloat16().view(torch.int16).numpy()
    np.testing.assert_array_equal(res[0][0], want)
