"""Failure detection between tensor-parallel ranks, on CPU ranks (gloo), with the failure made
on the host: a rank that leaves between steps, a rank that dies without a word, and a rank that
never joins a collective.

* leave / death: every rank runs steps of an all-reduce; before each launch it calls
  PeerMonitor.check().  When one rank leaves (or dies by os._exit) after step 2, the others must
  raise PeerLost naming it before launching step 3's collective -- within the heartbeat timeout
  for a silent death.
* a peer that never joins: with a short process-group timeout the waiting rank's all-reduce
  must end with an error instead of hanging."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mllm_b200.failure import PeerLost, PeerMonitor


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _steps_worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    store = dist.distributed_c10d._get_default_store()
    mon = PeerMonitor(store, rank, world, interval=0.05, timeout=0.6)
    leaver = world - 1
    result = ("done", None, None)
    try:
        for step in range(6):
            if rank == leaver and step == 3:
                if mode == "leave":
                    mon.leave()
                    q.put((rank, ("left", step, None)))
                    return
                q.put((rank, ("died", step, None)))
                q.close()
                q.join_thread()   # the message is out before the process vanishes
                os._exit(0)       # no goodbye: the heartbeat just stops
            # host-side check between steps, before the next launch; a silent death is noticed
            # once the heartbeat has been still for the timeout, so poll for up to 5 s
            t0 = time.monotonic()
            while True:
                try:
                    mon.check()
                except PeerLost as e:
                    result = ("lost", step, (e.rank, str(e), time.monotonic() - t0))
                    raise
                if step < 3 or time.monotonic() - t0 > 5.0:
                    break
                time.sleep(0.05)
            t = torch.full((4,), float(rank + 1))
            dist.all_reduce(t)
            assert t[0].item() == world * (world + 1) / 2
    except PeerLost:
        pass
    finally:
        mon.close()
    q.put((rank, result))


@pytest.mark.parametrize("mode", ["leave", "die"])
def test_survivors_detect_a_lost_peer_before_the_next_collective(mode):
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_steps_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, res = q.get(timeout=120)
        got[r] = res
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[world - 1][0] == ("left" if mode == "leave" else "died")
    for r in range(world - 1):
        kind, step, info = got[r]
        assert kind == "lost", got
        assert step == 3                   # noticed before step 3's collective was launched
        assert info[0] == world - 1
        if mode == "leave":
            assert "left" in info[1]
        else:
            assert "no heartbeat" in info[1] and info[2] < 5.0


def _never_joins_worker(rank, port, q, release):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=2))
    if rank == 1:
        release.wait(60)   # alive, but never enters the collective
        q.put((1, "idle"))
        return
    t0 = time.monotonic()
    try:
        dist.all_reduce(torch.ones(4))
        q.put((0, ("completed", time.monotonic() - t0)))
    except Exception as e:   # gloo reports the timeout as a RuntimeError
        q.put((0, ("error", time.monotonic() - t0, type(e).__name__)))
    finally:
        release.set()


def test_collective_with_a_peer_that_never_joins_ends_in_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    release = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_never_joins_worker, args=(r, port, q, release)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[0][0] == "error", got
    assert got[0][1] < 30.0
