"""The C++ drop-in's tensor-parallel mode under the reference's UNCHANGED QwenRunner: two
processes, one GPU each, both running the same runner on the same ids with
b200::SetTensorParallel set (each rank computes its kv-head group of every layer's attention and
the o_proj partials are summed by mllm_comm_all_reduce_bf16).  Their logits -- prefill of 37 rows
for 2 sequences, then 8 decode steps fed fixed tokens -- must equal each other and match the same
runner on one GPU at rtol = atol = 2e-2.  Needs 2 GPUs (skipped otherwise); NVLS off."""
import importlib.util
import os
import socket

import numpy as np
import pytest

from tests.helpers import ATOL, RTOL
from tests.qwen_model import QwenShape, write_random_qwen3

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

TINY = QwenShape(layers=3, hidden=512, heads=4, kv_heads=2, head_dim=128, intermediate=1024, vocab=1024)
B, S, STEPS = 2, 37, 8


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _load_dropin():
    from mllm_b200.dropin.build_facade import runner_module_path
    path = runner_module_path("dropin")
    spec = importlib.util.spec_from_file_location("mllm_dropin_runner", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ids():
    rng = np.random.default_rng(17)
    prompt = torch.from_numpy(rng.integers(0, TINY.vocab, size=(B, S))).long()
    steps = torch.from_numpy(rng.integers(0, TINY.vocab, size=(B, STEPS))).long()
    return prompt, steps


def _run(runner):
    prompt, steps = _ids()
    runner.reset_cache()
    out = [runner.forward(prompt).float().cpu()]
    for k in range(STEPS):
        out.append(runner.forward(steps[:, k:k + 1]).float().cpu())
    return out


def _worker(rank, port, path, q):
    import datetime

    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    from mllm_b200.comm import Communicator
    comm = Communicator.from_process_group(timeout_s=30.0)
    mod = _load_dropin()
    try:
        runner = mod.Runner(path)
        mod.set_tensor_parallel(comm.handle, rank, 2)
        out = _run(runner)
        torch.cuda.synchronize()
        mod.set_tensor_parallel(0, 0, 1)
        q.put((rank, [o.numpy() for o in out], comm.status()))
        del runner
    finally:
        comm.close()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dropin_tensor_parallel_runner_matches_one_gpu(tmp_path, cuda_device):
    import torch.multiprocessing as mp
    from mllm_b200 import build
    build.build()
    path = str(tmp_path / "qwen3_tiny")
    write_random_qwen3(path, TINY, seed=23)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, path, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, out, status = q.get(timeout=300)
        res[r] = (out, status)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert res[0][1] == 0 and res[1][1] == 0
    single = _run(_load_dropin().Runner(path))
    for k, want in enumerate(single):
        np.testing.assert_array_equal(res[0][0][k], res[1][0][k], err_msg=f"ranks differ at step {k}")
        np.testing.assert_allclose(res[0][0][k], want.numpy(), rtol=RTOL, atol=ATOL, err_msg=f"step {k}")
