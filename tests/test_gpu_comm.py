"""Communicators and bounded waits on the GPU, with every failure made on the host or by a wait
that nothing ends (no GPU fault, no hung kernel):

* a time-bounded device wait on a flag nobody raises gives up after its deadline and reports
  MLLM_ERR_DEVICE_TIMEOUT, and the context stays usable;
* a one-rank communicator: all-reduce and all-gather, the watchdog's bookkeeping, and an abort
  on request after which calls are refused with MLLM_ERR_COMM;
* two ranks (2 GPUs; skipped otherwise): all-reduce and all-gather against torch, then one rank
  leaves between steps; the other learns it from the heartbeat before its next launch, aborts its
  communicator, and its next collective is refused on the host.  NVLS is off in both ranks."""
import math
import os
import socket
import time

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


@pytest.fixture(scope="module")
def lib(cuda_device):
    from mllm_b200 import abi, build
    build.build()
    return abi.load()


def test_bounded_wait_gives_up_and_context_survives(lib):
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.monotonic()
    assert lib.mllm_wait_u32_timeout(flag.data_ptr(), 1, 20000, None) == 0   # 20 ms, nothing raises it
    assert lib.mllm_attn_device_status(None) == 6                             # MLLM_ERR_DEVICE_TIMEOUT
    assert time.monotonic() - t0 < 10.0
    assert lib.mllm_attn_device_status(None) == 0                             # read and cleared
    # a flag that is already up passes at once
    flag.fill_(5)
    assert lib.mllm_wait_u32_timeout(flag.data_ptr(), 5, 20000, None) == 0
    assert lib.mllm_attn_device_status(None) == 0
    # the context still runs kernels: a decode call on a small cache
    B, H, Hkv, D, L = 2, 8, 2, 128, 300
    k = torch.randn(B, Hkv, L, D, device="cuda").bfloat16()
    v = torch.randn_like(k)
    q = torch.randn(B, H, D, device="cuda").bfloat16()
    out = torch.empty(B, H * D, dtype=torch.bfloat16, device="cuda")
    ws_bytes = lib.mllm_decode_attention_workspace_size(B, H, Hkv, D, L)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    assert lib.mllm_decode_attention_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), *k.stride()[:3], None, B, H,
                                          Hkv, D, L, 1 / math.sqrt(D), out.data_ptr(), ws.data_ptr(), ws_bytes,
                                          None) == 0
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    # out-of-range deadlines are refused on the host
    assert lib.mllm_wait_u32_timeout(flag.data_ptr(), 1, 0, None) == 1
    assert lib.mllm_wait_u32_timeout(flag.data_ptr(), 1, 61_000_000, None) == 1


def test_single_rank_communicator(lib):
    from mllm_b200 import abi
    from mllm_b200.comm import MLLM_ERR_COMM, Communicator, unique_id
    comm = Communicator(0, 1, unique_id(), timeout_s=20.0)
    try:
        x = torch.randn(3, 1000, device="cuda").bfloat16()
        want = x.clone()
        comm.all_reduce(x)
        out = torch.empty_like(x)
        comm.all_gather(want, out)
        torch.cuda.synchronize()
        assert torch.equal(x, want) and torch.equal(out, want)
        deadline = time.monotonic() + 5
        while comm.in_flight() > 0 and time.monotonic() < deadline:
            time.sleep(0.01)
        assert comm.in_flight() == 0
        assert comm.status() == 0
        comm.abort()
        assert comm.status() == MLLM_ERR_COMM
        with pytest.raises(abi.MllmError) as e:
            comm.all_reduce(x)
        assert e.value.status == MLLM_ERR_COMM
    finally:
        comm.close()


def test_watchdog_does_not_disturb_graph_capture(lib):
    """A collective tracked by the watchdog, then a CUDA graph recorded (torch's default global
    capture mode) for longer than the watchdog's poll interval: the watchdog's event query runs
    during the recording and must not invalidate it; the graph then replays the collective."""
    from mllm_b200.comm import Communicator, unique_id
    comm = Communicator(0, 1, unique_id(), timeout_s=20.0)
    try:
        x = torch.randn(4096, device="cuda").bfloat16()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            comm.all_reduce(x)          # tracked: its event sits in the watchdog's queue
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        y = torch.zeros_like(x)
        with torch.cuda.graph(g):
            time.sleep(0.05)            # several watchdog polls happen while recording
            y.add_(x)
            comm.all_reduce(y)
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y, x)
        assert comm.status() == 0
        del g
    finally:
        comm.close()


def _two_rank_worker(rank, port, q):
    import datetime

    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    # a CPU group only carries the id and the heartbeat store; the data moves by mllm_comm_*
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    from mllm_b200 import abi
    from mllm_b200.comm import MLLM_ERR_COMM, Communicator
    from mllm_b200.failure import PeerLost, PeerMonitor
    res = {}
    mon = PeerMonitor(dist.distributed_c10d._get_default_store(), rank, 2, interval=0.05, timeout=1.0)
    comm = Communicator.from_process_group(timeout_s=20.0)
    try:
        dev = torch.device("cuda", rank)
        for n in (8, 4096 * 7 + 8, 1 << 20):
            g = torch.Generator(device=dev).manual_seed(10 * n + rank)
            x = torch.randn(n, device=dev, generator=g).bfloat16()
            res[("in", n)] = x.float().cpu().numpy()
            comm.all_reduce(x)
            res[("sum", n)] = x.float().cpu().numpy()
            gat = torch.empty(2 * n, dtype=torch.bfloat16, device=dev)
            comm.all_gather(x, gat)
            res[("gather", n)] = gat.float().cpu().numpy()
        torch.cuda.synchronize()
        mon.check()
        dist.barrier()
        if rank == 1:
            # leave between steps, nothing in flight: tell the peer, drop the communicator
            mon.leave()
            comm.abort()
            q.put((rank, res, "left"))
            return
        t0 = time.monotonic()
        lost = None
        while time.monotonic() - t0 < 10:
            try:
                mon.check()
            except PeerLost as e:
                lost = e
                break
            time.sleep(0.02)
        assert lost is not None and lost.rank == 1
        comm.abort()                  # the host learned it first: no collective is launched
        try:
            comm.all_reduce(torch.ones(8, dtype=torch.bfloat16, device=dev))
            refused = None
        except abi.MllmError as e:
            refused = e.status
        res["refused"] = refused == MLLM_ERR_COMM
        q.put((rank, res, "survived"))
    finally:
        mon.close()
        comm.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_communicator_and_a_peer_that_leaves():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_rank_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(2):
        r, res, how = q.get(timeout=300)
        got[r] = (res, how)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got[1][1] == "left" and got[0][1] == "survived"
    assert got[0][0]["refused"]
    for n in (8, 4096 * 7 + 8, 1 << 20):
        a, b = got[0][0][("in", n)], got[1][0][("in", n)]
        want = torch.from_numpy(a + b).bfloat16().float().numpy()   # one fp32 add, one rounding
        for r in range(2):
            np.testing.assert_array_equal(got[r][0][("sum", n)], want)
            np.testing.assert_array_equal(got[r][0][("gather", n)], np.concatenate([want, want]))
