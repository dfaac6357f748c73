#!/usr/bin/env python
"""Benchmark of the B200 attention path: decode KV-read GB/s and prefill attention TFLOP/s.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Headline (`value`): Qwen3-8B-shaped decode attention -- 32 sequences, one new token each,
against a bf16 KV cache of 4096 rows per sequence (hidden 4096, 32 q heads, 8 kv heads,
head_dim 128, per-head QK-RMSNorm eps 1e-6, RoPE theta 1e6).  One step = the QKV epilogue of
the new token (QK-norm + RoPE + KV append) + split-K flash-decode over 4096 rows, i.e. the
attention step between the q/k/v projections and o_proj, run as the fused decode step
(mllm_decode_step_bf16: one split-kernel launch, plus the chunk combine when the plan splits the
cache; at this shape it does not).  Metric = algorithmic
KV bytes read (2 * B * Hkv * L * D * 2 B = 536,870,912 B per step) / step time.  The cache
(537 MB) is larger than L2 (126 MB), so every step streams it from HBM.  `unfused` reports the
same step as two calls (mllm_qkv_epilogue_bf16, then mllm_decode_attention_bf16).

Secondary (`prefill`): Qwen3-8B causal prefill attention, batch 4 x 8192 rows, same head
geometry; FLOPs = 4 * B * H * D * S(S+1)/2 = 2.199e12 per step.  `prefill.varlen`: 32 prompts of
U[512, 8192] rows packed into one launch over a paged cache, against one launch per prompt.

Secondary (`ragged_decode`): Qwen3-14B-shaped decode over a ragged batch -- 64 requests whose
cache lengths are drawn from U[256, 32768] with a fixed seed, 40 q heads / 8 kv heads,
head_dim 128; one layer's decode call timed back to back (a 40-layer step is 40 such calls).
Metric = algorithmic KV bytes (sum_b L_b * 2 * Hkv * D * 2 B) / call time.

Multi-GPU (torchrun, one rank per GPU): decode is split by request batches -- every rank owns
its own 32 sequences (weak scaling, no collective on the data path); prefill is split by
KV-head groups (H/N query heads and Hkv/N kv heads per rank).  Timing is max over ranks.

`--impl reference` times the reference's own CPU LibTorch path (oracle/_ref, compiled from the
reference sources) on this host's cores on bounded samples of the same decode workload.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "prefill attn TFLOP/s & decode KV-read GB/s per B200, 1/2/4/8 GPU vs CPU ref"

# Qwen3-8B attention geometry
HIDDEN, H, HKV, D = 4096, 32, 8, 128
THETA, EPS = 1e6, 1e-6
DEC_B, DEC_L = 32, 4096
PRE_B, PRE_S = 4, 8192
# Qwen3-14B ragged decode: 64 requests, lengths U[256, 32768] (seeded), 40 layers
RAG_B, RAG_H, RAG_HKV, RAG_LAYERS, RAG_HIDDEN = 64, 40, 8, 40, 5120
RAG_LMIN, RAG_LMAX, RAG_SEED = 256, 32768, 14


def ragged_lengths():
    import numpy as np
    return np.random.default_rng(RAG_SEED).integers(RAG_LMIN, RAG_LMAX + 1, size=RAG_B)


def decode_kv_bytes(b, hkv, L, d):
    return 2 * b * hkv * L * d * 2


def prefill_flops(b, h, d, s):
    return 4.0 * b * h * d * s * (s + 1) / 2


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            j = json.load(f)
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes recorded from an ncu capture in profiles/<name>.md
    (a line 'traffic_bytes_per_launch: N'), or None."""
    p = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(p):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.gpu = gpu_index
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "20",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out = ""
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------------------------------
# CPU reference arm
# ------------------------------------------------------------------------------------------

def cpu_reference_decode(steps: int, warmup: int, budget_s: float = 90.0):
    """The reference's fp32 CPU path on a bounded sample of the decode workload, timed for the
    same work the GPU step does: QK-norm + RoPE + KV append + attention over the cache, without
    the q/k/v projections and o_proj.  The reference has no entry point for that part alone (its
    Attention::ForwardProjected ends with o_proj, Attention.h:322-325), so each sample times the
    whole Qwen3 attention step (q/k/v Linear, the per-head RMSNorm of TransformerBlock.h:103-134,
    ForwardProjected) and, right after, its four Linear calls alone on the same shapes, and the
    attention time is the difference of the medians.  `sample_b` of the 32 sequences at full
    cache length and all heads; oracle/_ref is the reference compiled from its sources, the numpy
    port of the oracle stands in when it is absent.  Returns a dict for the JSON line."""
    import numpy as np
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    sample_b = 1
    kind = "reference"
    try:
        sys.path.insert(0, os.path.join(ROOT, "oracle", "_ref"))
        import mllm_ref as R  # compiled from the reference sources
        R.set_num_threads(cores)
    except Exception:
        R = None
        kind = "port"
    g = torch.Generator().manual_seed(1234)
    L = DEC_L
    kc = torch.randn(sample_b, HKV, L - 1, D, generator=g)
    vc = torch.randn(sample_b, HKV, L - 1, D, generator=g)
    h = torch.randn(sample_b, 1, HIDDEN, generator=g)
    a = torch.randn(sample_b, 1, H * D, generator=g)
    w_q = torch.randn(H * D, HIDDEN, generator=g) * 0.02
    w_k = torch.randn(HKV * D, HIDDEN, generator=g) * 0.02
    w_v = torch.randn(HKV * D, HIDDEN, generator=g) * 0.02
    w_o = torch.randn(HIDDEN, H * D, generator=g) * 0.02
    gq = 1 + 0.1 * torch.randn(D, generator=g)
    gk = 1 + 0.1 * torch.randn(D, generator=g)
    pos = torch.tensor([L - 1])

    def full():
        if R is not None:
            q = R.linear(h, w_q).view(sample_b, 1, H, D).transpose(1, 2)
            q = R.rms_norm(q, gq, EPS)
            k = R.linear(h, w_k).view(sample_b, 1, HKV, D).transpose(1, 2)
            k = R.rms_norm(k, gk, EPS)
            v = R.linear(h, w_v).view(sample_b, 1, HKV, D).transpose(1, 2)
            R.attention_forward_projected(q, k, v, w_o, H, HKV, D, THETA, pos, kc, vc, True)
        else:
            from oracle import attention_oracle as O
            hn = h.numpy()
            q, k, v = O.qwen_qkv_prologue(hn, w_q.numpy(), w_k.numpy(), w_v.numpy(), gq.numpy(), gk.numpy(),
                                          H, HKV, D, EPS)
            cache = O.KVCache(kc.numpy(), vc.numpy())
            O.attention_forward_projected(q, k, v, w_o.numpy(), H, HKV, D, THETA, pos.numpy(), cache)

    def linears():
        if R is not None:
            R.linear(h, w_q)
            R.linear(h, w_k)
            R.linear(h, w_v)
            R.linear(a, w_o)
        else:
            hn, an = h.numpy(), a.numpy()
            for w_, x_ in ((w_q, hn), (w_k, hn), (w_v, hn), (w_o, an)):
                x_ @ w_.numpy().T

    for _ in range(max(1, min(warmup, 2))):
        full()
        linears()
    t_full, t_lin = [], []
    t_start = time.perf_counter()
    for _ in range(steps):
        t0 = time.perf_counter()
        full()
        t1 = time.perf_counter()
        linears()
        t2 = time.perf_counter()
        t_full.append(t1 - t0)
        t_lin.append(t2 - t1)
        if time.perf_counter() - t_start > budget_s:
            break
    med_full, med_lin = statistics.median(t_full), statistics.median(t_lin)
    med = med_full - med_lin
    nbytes = decode_kv_bytes(sample_b, HKV, L, D)
    return {"value": nbytes / med / 1e9, "unit": "GB/s", "cores": cores, "kind": kind,
            "sample": f"{sample_b} of {DEC_B} sequences (L={L}, all {H} q heads), fp32 CPU: QK-norm + RoPE + KV "
                      f"append + attention = median of the whole attention step ({med_full * 1e3:.2f} ms) minus "
                      f"median of its q/k/v/o Linear calls timed alone ({med_lin * 1e3:.2f} ms), {len(t_full)} runs",
            "steps_timed": len(t_full), "ms_per_step": med * 1e3, "full_step_ms": med_full * 1e3,
            "linear_ms": med_lin * 1e3}


# ------------------------------------------------------------------------------------------
# GPU arm
# ------------------------------------------------------------------------------------------

def run_gpu(args, rank, world, device):
    import torch
    from mllm_b200 import abi, build

    if rank == 0 or not os.path.exists(build.lib_path()):
        build.build()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    lib = abi.load()
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    gen = torch.Generator(device=device).manual_seed(1000 + rank)
    comm = None
    if world > 1:
        # the library's own communicator (mllm_comm_*: non-blocking NCCL with a watchdog)
        from mllm_b200.comm import Communicator
        comm = Communicator.from_process_group(timeout_s=60.0)

    # ------------------------------- decode workload -------------------------------
    B, L = DEC_B, DEC_L
    kbuf = torch.randn(B, HKV, L, D, device=device, generator=gen).bfloat16()
    vbuf = torch.randn(B, HKV, L, D, device=device, generator=gen).bfloat16()
    qkv = (torch.randn(B, (H + 2 * HKV) * D, device=device, generator=gen) * 0.5).bfloat16()
    gq = (1 + 0.1 * torch.randn(D, device=device, generator=gen)).bfloat16()
    gk = (1 + 0.1 * torch.randn(D, device=device, generator=gen)).bfloat16()
    pos = torch.full((B,), L - 1, dtype=torch.int64, device=device)
    start = torch.full((B,), L - 1, dtype=torch.int32, device=device)   # new token -> row L-1
    lens = torch.full((B,), L, dtype=torch.int32, device=device)        # attend over L rows
    q_rot = torch.empty(B, H, D, dtype=torch.bfloat16, device=device)
    out = torch.empty(B, H * D, dtype=torch.bfloat16, device=device)
    ws_bytes = lib.mllm_decode_attention_workspace_size(B, H, HKV, D, L)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)   # the header starts at zero
    csb, csh, cst = kbuf.stride()[:3]
    row = (H + 2 * HKV) * D
    scale = 1.0 / math.sqrt(D)

    def epilogue(src):
        st = lib.mllm_qkv_epilogue_bf16(
            src.data_ptr(), row, row, D,
            src.data_ptr() + H * D * 2, row, row, D,
            src.data_ptr() + (H + HKV) * D * 2, row, row, D,
            B, 1, H, HKV, D, pos.data_ptr(), 1, 0, THETA, None, None, 0, 0,
            gq.data_ptr(), gk.data_ptr(), EPS, q_rot.data_ptr(),
            kbuf.data_ptr(), vbuf.data_ptr(), csb, csh, cst, L, start.data_ptr(), 0, sh)
        assert st == 0, lib.mllm_attn_last_error()

    def decode(dst):
        st = lib.mllm_decode_attention_bf16(q_rot.data_ptr(), kbuf.data_ptr(), vbuf.data_ptr(), csb, csh, cst,
                                            lens.data_ptr(), B, H, HKV, D, L, scale, dst.data_ptr(),
                                            ws.data_ptr(), ws_bytes, sh)
        assert st == 0, lib.mllm_attn_last_error()

    def step(src, dst):
        # the fused step: the new token (row L-1 of every sequence, position L-1) and the decode
        # over all L rows in one split-kernel launch (+ the chunk combine)
        st = lib.mllm_decode_step_bf16(
            src.data_ptr(), row, D, src.data_ptr() + H * D * 2, row, D, src.data_ptr() + (H + HKV) * D * 2, row, D,
            pos.data_ptr(), 1, THETA, None, None, 0, gq.data_ptr(), gk.data_ptr(), EPS,
            kbuf.data_ptr(), vbuf.data_ptr(), csb, csh, cst, lens.data_ptr(), B, H, HKV, D, L, scale,
            dst.data_ptr(), ws.data_ptr(), ws_bytes, sh)
        assert st == 0, lib.mllm_attn_last_error()

    # our kernel launches per fused step: the split kernel, plus the combine when the plan
    # splits each sequence's cache into several chunks
    plan_rows, plan_chunks, plan_launches = C.c_int(), C.c_int(), C.c_int()
    assert lib.mllm_decode_attention_plan(B, H, HKV, D, L, C.byref(plan_rows), C.byref(plan_chunks),
                                          C.byref(plan_launches)) == 0, lib.mllm_attn_last_error()
    launches_per_step = plan_launches.value

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        import torch.distributed as dist
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step(qkv, out)
        epilogue(qkv)
        decode(out)
    torch.cuda.synchronize()

    # the head-sharded layer against the unsharded one, before anything is timed
    tp_parity = tp_parity_leg(rank, world, device, comm, barrier) if world > 1 else None

    sampler = ClockSampler(torch.cuda.current_device() if "CUDA_VISIBLE_DEVICES" not in os.environ
                           else int(os.environ.get("LOCAL_RANK", 0)))
    if rank == 0:
        sampler.start()
        time.sleep(0.3)
    # timed region: K fused steps back to back between two events, nothing else in the loop;
    # the step's kernels are the whole step, so this is also the roofline timing
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0.record(stream)
    for i in range(args.steps):
        step(qkv, out)
    t1.record(stream)
    torch.cuda.synchronize()
    barrier()
    elapsed_ms = max_over_ranks(t0.elapsed_time(t1))
    # the same step as two calls (epilogue kernel, then the decode kernels), and the decode
    # kernels alone, for comparison
    u0 = torch.cuda.Event(enable_timing=True)
    u1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    u0.record(stream)
    for i in range(args.steps):
        epilogue(qkv)
        decode(out)
    u1.record(stream)
    torch.cuda.synchronize()
    barrier()
    unfused_ms = max_over_ranks(u0.elapsed_time(u1) / args.steps)
    barrier()
    torch.cuda.synchronize()
    u0.record(stream)
    for i in range(args.steps):
        decode(out)
    u1.record(stream)
    torch.cuda.synchronize()
    barrier()
    dec_ms = max_over_ranks(u0.elapsed_time(u1) / args.steps)

    # ---- e2e through the C ABI with host buffers: every step copies its q/k/v in from pinned
    # host memory and its output back out.  Copies run on a second stream, double-buffered, so
    # step i+1's input copy and step i-1's output copy overlap step i's kernels (the way a
    # serving loop drives the path).
    h_in = torch.empty_like(qkv, device="cpu").pin_memory()
    h_in.copy_(qkv.cpu())
    h_out = [torch.empty(out.shape, dtype=out.dtype, device="cpu").pin_memory() for _ in range(2)]
    d_in = [torch.empty_like(qkv) for _ in range(2)]
    d_out = [torch.empty_like(out) for _ in range(2)]
    cs = torch.cuda.Stream(device=device)
    ev = lambda: torch.cuda.Event()

    def e2e_run(n):
        ev_in = [ev(), ev()]      # input copy into buffer j done
        ev_used = [ev(), ev()]    # the step finished reading input buffer j
        ev_done = [ev(), ev()]    # output buffer j written
        ev_out = [ev(), ev()]     # output buffer j copied back to the host
        with torch.cuda.stream(cs):
            d_in[0].copy_(h_in, non_blocking=True)
            ev_in[0].record(cs)
        for i in range(n):
            j = i % 2
            if i + 1 < n:
                with torch.cuda.stream(cs):
                    if i >= 1:
                        cs.wait_event(ev_used[(i + 1) % 2])
                    d_in[(i + 1) % 2].copy_(h_in, non_blocking=True)
                    ev_in[(i + 1) % 2].record(cs)
            stream.wait_event(ev_in[j])
            if i >= 2:
                stream.wait_event(ev_out[j])
            step(d_in[j], d_out[j])
            ev_used[j].record(stream)
            ev_done[j].record(stream)
            with torch.cuda.stream(cs):
                cs.wait_event(ev_done[j])
                h_out[j].copy_(d_out[j], non_blocking=True)
                ev_out[j].record(cs)
        stream.wait_stream(cs)

    e2e_run(args.warmup)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    cs.wait_event(e0)
    e2e_run(args.steps)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))

    # ---- the attention step's q/k/v projections at decode size (Qwen3-8B, batch DEC_B): one
    # mllm_linear_bf16 launch against the reference's three cuBLAS GEMMs and against one cuBLAS
    # GEMM over concatenated weights.  Steady state: 40 launches captured in a CUDA graph over a
    # ring of 4 weight sets (192 MB, larger than L2), timed with events around the replays.
    from mllm_b200 import runtime as rt
    F = torch.nn.functional
    hx = torch.randn(B, HIDDEN, device=device, generator=gen).bfloat16()
    ring = [[(0.02 * torch.randn(n, HIDDEN, device=device, generator=gen)).bfloat16()
             for n in (H * D, HKV * D, HKV * D)] for _ in range(4)]
    ring_cat = [torch.cat(ws_, 0) for ws_ in ring]

    def graphed_us(fn, n=40, reps=5):
        side = torch.cuda.Stream(device=device)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for i in range(4):
                fn(i)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        scratch = rt.GraphScratch()   # the recorded launches' workspace, alive as long as the graph
        with rt.graph_scratch(scratch), torch.cuda.graph(gr):
            for i in range(n):
                fn(i)
        gr.replay()
        torch.cuda.synchronize()
        barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(reps):
            gr.replay()
        a1.record(stream)
        torch.cuda.synchronize()
        del gr, scratch
        return max_over_ranks(a0.elapsed_time(a1) / (reps * n) * 1e3)

    proj = {"ours_us": graphed_us(lambda i: rt.linear(hx, ring[i % 4])),
            "cublas_three_us": graphed_us(lambda i: [F.linear(hx, w) for w in ring[i % 4]]),
            "cublas_concat_us": graphed_us(lambda i: F.linear(hx, ring_cat[i % 4])),
            "bytes": (ring_cat[0].numel() + hx.numel() + B * ring_cat[0].shape[0]) * 2}
    del ring, ring_cat
    # FP8 block-scaled weights (the FP8 checkpoint layout): the Qwen3-8B gate projection
    # [12288 x 4096] at 32 tokens, one mllm_linear_fp8_bf16 launch against the reference's route
    # for such weights on every step -- DequantizeFP8 (QwenRunner.cpp:103-122) then a cuBLAS GEMM --
    # and against bf16 weights through cuBLAS; a ring of 4 weight sets (201 MB of fp8 > L2)
    NF = 12288
    ring8 = [rt.Fp8Weight.quantize((0.02 * torch.randn(NF, HIDDEN, device=device, generator=gen)).bfloat16())
             for _ in range(4)]
    ring16 = [w.dequantize() for w in ring8]
    proj["fp8"] = {"ours_us": graphed_us(lambda i: rt.linear_fp8(hx, ring8[i % 4])),
                   "reference_route_us": graphed_us(lambda i: F.linear(hx, ring8[i % 4].dequantize())),
                   "cublas_bf16_weights_us": graphed_us(lambda i: F.linear(hx, ring16[i % 4])),
                   "bytes": NF * HIDDEN + (NF // 128) * (HIDDEN // 128) * 4 + (B * HIDDEN + B * NF) * 2,
                   "out_features": NF}
    del ring8, ring16

    # ------------------------------- prefill workload -------------------------------
    pre = None
    if not args.skip_prefill and H % world == 0 and HKV % world == 0:
        Hr, Hkvr = H // world, HKV // world
        Bp, S = PRE_B, PRE_S
        qkv_p = (torch.randn(Bp, S, (Hr + 2 * Hkvr) * D, device=device, generator=gen) * 0.5).bfloat16()
        kp = torch.empty(Bp, Hkvr, S, D, dtype=torch.bfloat16, device=device)
        vp = torch.empty_like(kp)
        qp = torch.empty(Bp, Hr, S, D, dtype=torch.bfloat16, device=device)
        op = torch.empty(Bp, S, Hr * D, dtype=torch.bfloat16, device=device)
        pos_p = torch.arange(S, dtype=torch.int64, device=device)
        start_p = torch.zeros(Bp, dtype=torch.int32, device=device)
        prow = (Hr + 2 * Hkvr) * D
        psb, psh, pst = kp.stride()[:3]

        def epi_p():
            st = lib.mllm_qkv_epilogue_bf16(
                qkv_p.data_ptr(), S * prow, prow, D,
                qkv_p.data_ptr() + Hr * D * 2, S * prow, prow, D,
                qkv_p.data_ptr() + (Hr + Hkvr) * D * 2, S * prow, prow, D,
                Bp, S, Hr, Hkvr, D, pos_p.data_ptr(), 0, 1, THETA, None, None, 0, 0,
                gq.data_ptr(), gk.data_ptr(), EPS, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                psb, psh, pst, S, start_p.data_ptr(), 0, sh)
            assert st == 0, lib.mllm_attn_last_error()

        def attn_p():
            st = lib.mllm_prefill_attention_bf16(qp.data_ptr(), kp.data_ptr(), vp.data_ptr(), psb, psh, pst,
                                                 Bp, Hr, Hkvr, D, S, S, scale, op.data_ptr(), sh)
            assert st == 0, lib.mllm_attn_last_error()

        # tensor-parallel exchange: this rank's column slice of o_proj, then the all-reduce of the
        # partial [B*S, hidden] outputs (NCCL over NVLink), as mllm_b200.tp.tp_attention_block does
        w_o = (0.02 * torch.randn(HIDDEN, Hr * D, device=device, generator=gen)).bfloat16()
        o_part = torch.empty(Bp * S, HIDDEN, dtype=torch.bfloat16, device=device)

        def oproj_p():
            torch.matmul(op.view(Bp * S, Hr * D), w_o.t(), out=o_part)

        def allreduce_p():
            if world > 1:
                import torch.distributed as dist
                dist.all_reduce(o_part)

        ksteps = max(3, min(args.steps, 20))
        for _ in range(args.warmup):
            epi_p()
            attn_p()
            oproj_p()
            allreduce_p()
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        p0.record(stream)
        for i in range(ksteps):
            epi_p()
            attn_p()
        p1.record(stream)
        torch.cuda.synchronize()
        barrier()
        pre_ms = max_over_ranks(p0.elapsed_time(p1)) / ksteps
        # the attention kernel alone, back to back, for the roofline
        barrier()
        torch.cuda.synchronize()
        p0.record(stream)
        for i in range(ksteps):
            attn_p()
        p1.record(stream)
        torch.cuda.synchronize()
        barrier()
        attn_ms = max_over_ranks(p0.elapsed_time(p1)) / ksteps
        # the QKV epilogue alone (QK-norm + RoPE + cache append of all 4 x 8192 tokens)
        barrier()
        torch.cuda.synchronize()
        p0.record(stream)
        for i in range(ksteps):
            epi_p()
        p1.record(stream)
        torch.cuda.synchronize()
        barrier()
        epi_ms = max_over_ranks(p0.elapsed_time(p1)) / ksteps
        epi_bytes = 2 * qkv_p.numel() * 2   # each head row read once and written once
        varlen = prefill_varlen_leg(args, lib, device, gen, Hr, Hkvr, scale, sh, stream, barrier, max_over_ranks,
                                    ksteps)
        # the layer's exchange step, timed separately (o_proj GEMM, then the all-reduce)
        evo = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(ksteps)]
        barrier()
        torch.cuda.synchronize()
        for i in range(ksteps):
            evo[i][0].record(stream)
            oproj_p()
            evo[i][1].record(stream)
            allreduce_p()
            evo[i][2].record(stream)
        torch.cuda.synchronize()
        barrier()
        oproj_ms = max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in evo))
        ar_ms = max_over_ranks(statistics.mean(e[1].elapsed_time(e[2]) for e in evo))
        ar_bytes = o_part.numel() * 2
        # the same exchange as tp_attention_block runs it: o_proj in 4 row pieces, each piece's
        # all-reduce overlapping the next piece's GEMM (mllm_b200.tp.oproj_allreduce)
        from mllm_b200.tp import oproj_allreduce
        attn2d = op.view(Bp * S, Hr * D)
        for _ in range(2):
            oproj_allreduce(attn2d, w_o)
        barrier()
        torch.cuda.synchronize()
        p0.record(stream)
        for i in range(ksteps):
            oproj_allreduce(attn2d, w_o)
        p1.record(stream)
        torch.cuda.synchronize()
        barrier()
        overlap_ms = max_over_ranks(p0.elapsed_time(p1)) / ksteps
        # the exchange over NVLink peer memory: each GEMM piece lands in a buffer the other ranks
        # can read; its owner pulls it from every rank, sums and pushes the rows to every rank
        # (mllm_b200.tp.PeerExchange)
        peer_ms = None
        from mllm_b200.tp import PeerExchange
        if world > 1:
            ex = PeerExchange(Bp * S, HIDDEN, sub=4)
            for _ in range(2):
                ex(attn2d, w_o)
            barrier()
            torch.cuda.synchronize()
            p0.record(stream)
            for i in range(ksteps):
                ex(attn2d, w_o)
            p1.record(stream)
            torch.cuda.synchronize()
            barrier()
            peer_ms = max_over_ranks(p0.elapsed_time(p1)) / ksteps
            ex.close()
        # The whole attention layer of the step (QKV epilogue + attention + o_proj + exchange), for
        # every exchange, with the total work fixed (4 x 8192 tokens, 32 q heads) whatever N is.
        from mllm_b200.tp import SeqParallelOProj
        w_o_full = (0.02 * torch.randn(HIDDEN, H * D, device=device, generator=gen)).bfloat16()
        layer_modes = {}
        if world == 1:
            layer_modes["single_gpu"] = lambda: torch.matmul(op.view(Bp * S, H * D), w_o_full.t(), out=o_part)
        else:
            import torch.distributed as dist
            layer_modes["gemm_then_nccl_allreduce"] = lambda: (oproj_p(), dist.all_reduce(o_part))
            layer_modes["gemm_then_comm_allreduce"] = lambda: (oproj_p(), comm.all_reduce(o_part))
            layer_modes["chunked_overlap"] = lambda: oproj_allreduce(attn2d, w_o)
            sp_nccl = SeqParallelOProj(Bp * S, HIDDEN)
            sp_comm = SeqParallelOProj(Bp * S, HIDDEN, comm=comm)
            layer_modes["seqpar_nccl"] = lambda: sp_nccl(attn2d, w_o_full)
            layer_modes["seqpar_comm"] = lambda: sp_comm(attn2d, w_o_full)
            ex_l = PeerExchange(Bp * S, HIDDEN, sub=4)
            layer_modes["peer_exchange"] = lambda: ex_l(attn2d, w_o)
        # The same layer in micro-batches of sequences: each micro-batch's o_proj + exchange runs
        # on a high-priority side stream while the next micro-batch's epilogue + attention runs
        # (mllm_b200.tp.run_micro_batches); Bp / M sequences per micro-batch.
        from mllm_b200.tp import run_micro_batches

        def epi_mb(b0, nb):
            off = b0 * S * prow * 2
            kv_off = b0 * psb * 2
            st = lib.mllm_qkv_epilogue_bf16(
                qkv_p.data_ptr() + off, S * prow, prow, D,
                qkv_p.data_ptr() + off + Hr * D * 2, S * prow, prow, D,
                qkv_p.data_ptr() + off + (Hr + Hkvr) * D * 2, S * prow, prow, D,
                nb, S, Hr, Hkvr, D, pos_p.data_ptr(), 0, 1, THETA, None, None, 0, 0,
                gq.data_ptr(), gk.data_ptr(), EPS, qp.data_ptr() + b0 * Hr * S * D * 2,
                kp.data_ptr() + kv_off, vp.data_ptr() + kv_off, psb, psh, pst, S, start_p.data_ptr(), 0,
                torch.cuda.current_stream().cuda_stream)
            assert st == 0, lib.mllm_attn_last_error()

        def attn_mb(b0, nb):
            kv_off = b0 * psb * 2
            st = lib.mllm_prefill_attention_bf16(qp.data_ptr() + b0 * Hr * S * D * 2, kp.data_ptr() + kv_off,
                                                 vp.data_ptr() + kv_off, psb, psh, pst, nb, Hr, Hkvr, D, S, S, scale,
                                                 op.data_ptr() + b0 * S * Hr * D * 2,
                                                 torch.cuda.current_stream().cuda_stream)
            assert st == 0, lib.mllm_attn_last_error()

        pipelined = {}
        if world > 1:
            comm_side = torch.cuda.Stream(device=device, priority=-1)
            for M in (2, 4):
                nb = Bp // M
                rows = nb * S

                def compute(m, nb=nb):
                    epi_mb(m * nb, nb)
                    attn_mb(m * nb, nb)

                def ex_allreduce(m, rows=rows):
                    a, b = m * rows, (m + 1) * rows
                    torch.matmul(attn2d[a:b], w_o.t(), out=o_part[a:b])
                    comm.all_reduce(o_part[a:b])

                sp_m = SeqParallelOProj(rows, HIDDEN, comm=comm)

                def ex_seqpar(m, rows=rows, sp_m=sp_m):
                    a, b = m * rows, (m + 1) * rows
                    sp_m(attn2d[a:b], w_o_full)

                pipelined[f"micro{M}_gemm_then_comm_allreduce"] = (compute, ex_allreduce, M)
                pipelined[f"micro{M}_seqpar_comm"] = (compute, ex_seqpar, M)
            for name, (compute, exch, M) in pipelined.items():
                layer_modes[name] = (lambda compute=compute, exch=exch, M=M:
                                     run_micro_batches(compute, exch, M, comm_side))
        if world > 1:
            # token rows in, token rows out (tp.UlyssesLayout): this rank's q/k/v projections of
            # its T/N token rows (all heads), one all-to-all to the head owners, the epilogue and
            # attention on this rank's heads, one all-to-all back, o_proj of its rows with the
            # whole w_o.  The layer's input and output stay sharded by token rows.
            from mllm_b200.tp import UlyssesLayout, shard_heads
            uly = UlyssesLayout(shard_heads(H, HKV, world, rank), H, HKV, D)
            # the projections of this rank's rows, as UlyssesLayout.project writes them: [N, T/N, cols]
            qkv_send = (torch.randn(world, Bp * S // world, (Hr + 2 * Hkvr) * D, device=device, generator=gen)
                        * 0.5).bfloat16()
            out_tok = torch.empty(Bp * S // world, HIDDEN, dtype=torch.bfloat16, device=device)

            def ulysses_layer():
                qkv_h = uly.heads_from_tokens_packed(qkv_send)   # [B*S, (Hr + 2 Hkvr) D], qkv_p's layout
                st = lib.mllm_qkv_epilogue_bf16(
                    qkv_h.data_ptr(), S * prow, prow, D,
                    qkv_h.data_ptr() + Hr * D * 2, S * prow, prow, D,
                    qkv_h.data_ptr() + (Hr + Hkvr) * D * 2, S * prow, prow, D,
                    Bp, S, Hr, Hkvr, D, pos_p.data_ptr(), 0, 1, THETA, None, None, 0, 0,
                    gq.data_ptr(), gk.data_ptr(), EPS, qp.data_ptr(), kp.data_ptr(), vp.data_ptr(),
                    psb, psh, pst, S, start_p.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
                assert st == 0, lib.mllm_attn_last_error()
                attn_p()
                torch.matmul(uly.tokens_from_heads(attn2d), w_o_full.t(), out=out_tok)

            layer_modes["micro1_ulysses_token_rows_io"] = ulysses_layer

            # the same layout one sequence at a time (rank r owns rows [r S/N, (r+1) S/N) of every
            # sequence), pipelined by UlyssesLayout.run_sequences: sequence b+1's input all-to-all
            # and sequence b-1's output all-to-all + o_proj run on a side stream under sequence b's
            # epilogue + attention
            seq_send = [(torch.randn(world, S // world, prow, device=device, generator=gen) * 0.5).bfloat16()
                        for _ in range(Bp)]
            out_seq = torch.empty(Bp, S // world, HIDDEN, dtype=torch.bfloat16, device=device)
            side_u = torch.cuda.Stream(device=device, priority=-1)

            def attend_seq(b, qkv_h):
                kv_off = b * psb * 2
                st = lib.mllm_qkv_epilogue_bf16(
                    qkv_h.data_ptr(), S * prow, prow, D,
                    qkv_h.data_ptr() + Hr * D * 2, S * prow, prow, D,
                    qkv_h.data_ptr() + (Hr + Hkvr) * D * 2, S * prow, prow, D,
                    1, S, Hr, Hkvr, D, pos_p.data_ptr(), 0, 1, THETA, None, None, 0, 0,
                    gq.data_ptr(), gk.data_ptr(), EPS, qp.data_ptr() + b * Hr * S * D * 2,
                    kp.data_ptr() + kv_off, vp.data_ptr() + kv_off, psb, psh, pst, S, start_p.data_ptr(), 0,
                    torch.cuda.current_stream().cuda_stream)
                assert st == 0, lib.mllm_attn_last_error()
                attn_mb(b, 1)
                return attn2d[b * S:(b + 1) * S]

            def finish_seq(b, rows):
                torch.matmul(rows, w_o_full.t(), out=out_seq[b])

            layer_modes["micro4_ulysses_per_sequence"] = lambda: uly.run_sequences(
                lambda b: seq_send[b], attend_seq, finish_seq, Bp, side_u)
        layer_ms = {}
        for name, exch in layer_modes.items():
            if name.startswith("micro"):
                # the whole layer is the schedule itself
                for _ in range(2):
                    exch()
                barrier()
                torch.cuda.synchronize()
                p0.record(stream)
                for i in range(ksteps):
                    exch()
                p1.record(stream)
                torch.cuda.synchronize()
                barrier()
                layer_ms[name] = max_over_ranks(p0.elapsed_time(p1)) / ksteps
                continue
            for _ in range(2):
                epi_p()
                attn_p()
                exch()
            barrier()
            torch.cuda.synchronize()
            p0.record(stream)
            for i in range(ksteps):
                epi_p()
                attn_p()
                exch()
            p1.record(stream)
            torch.cuda.synchronize()
            barrier()
            layer_ms[name] = max_over_ranks(p0.elapsed_time(p1)) / ksteps
        if world > 1:
            ex_l.close()
        del w_o_full
        pre = {"layer_ms": layer_ms, "epi_ms": epi_ms, "epi_bytes": epi_bytes,
               "varlen": varlen, "peer_ms": peer_ms, "pre_ms": pre_ms, "attn_ms": attn_ms, "steps": ksteps, "oproj_ms": oproj_ms, "overlap_ms": overlap_ms,
               "allreduce_ms": ar_ms if world > 1 else 0.0, "allreduce_bytes": ar_bytes if world > 1 else 0,
               "allreduce_busbw_gbs": (2 * (world - 1) / world * ar_bytes / (ar_ms * 1e-3) / 1e9)
               if world > 1 and ar_ms > 0 else None}
        del qkv_p, kp, vp, qp, op, o_part, w_o

    # ---------------- ragged decode: Qwen3-14B geometry, 64 requests of mixed length ----------------
    rag = None
    if not args.skip_ragged and RAG_HKV % world == 0:
        torch.cuda.empty_cache()
        Hr, Hkvr = RAG_H // world, RAG_HKV // world   # kv-head groups per rank
        lens_np = ragged_lengths()
        Lmax = int(lens_np.max())
        kr = torch.empty(RAG_B, Hkvr, Lmax, D, dtype=torch.bfloat16, device=device)
        vr = torch.empty_like(kr)
        kr.normal_(generator=gen)
        vr.normal_(generator=gen)
        qr = torch.randn(RAG_B, Hr, D, device=device, generator=gen).bfloat16()
        orr = torch.empty(RAG_B, Hr * D, dtype=torch.bfloat16, device=device)
        lens_r = torch.from_numpy(lens_np.astype("int32")).to(device)
        ws_r_bytes = lib.mllm_decode_attention_workspace_size(RAG_B, Hr, Hkvr, D, Lmax)
        ws_r = torch.zeros(ws_r_bytes, dtype=torch.uint8, device=device)
        rsb, rsh, rst = kr.stride()[:3]

        def decode_r():
            # on torch's current stream: the stream being captured when the layer step is recorded
            st = lib.mllm_decode_attention_bf16(qr.data_ptr(), kr.data_ptr(), vr.data_ptr(), rsb, rsh, rst,
                                                lens_r.data_ptr(), RAG_B, Hr, Hkvr, D, Lmax, scale, orr.data_ptr(),
                                                ws_r.data_ptr(), ws_r_bytes, torch.cuda.current_stream().cuda_stream)
            assert st == 0, lib.mllm_attn_last_error()

        rsteps = max(3, min(args.steps, 50))
        for _ in range(args.warmup):
            decode_r()
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        r0.record(stream)
        for i in range(rsteps):
            decode_r()
        r1.record(stream)
        torch.cuda.synchronize()
        barrier()
        # The Qwen3-14B decode step as its 40 layers run it: per layer the decode over this rank's
        # kv heads, the o_proj of its q heads' outputs ([64, Hr*D] x [5120, Hr*D]^T, a partial
        # [64, 5120]) and the all-reduce of that partial (mllm_comm_all_reduce_bf16, NCCL) --
        # recorded as one CUDA graph of 40 layers and replayed.  Every layer reads the same
        # cache: its 4.4 GB (per GPU: / N) is far larger than L2, so each layer streams it anew.
        w_or = (0.02 * torch.randn(RAG_HIDDEN, Hr * D, device=device, generator=gen)).bfloat16()
        part_r = torch.empty(RAG_B, RAG_HIDDEN, dtype=torch.bfloat16, device=device)

        def exch_r():
            torch.matmul(orr, w_or.t(), out=part_r)
            if comm is not None:
                comm.all_reduce(part_r)

        def graph_ms(body, reps):
            side = torch.cuda.Stream(device=device)
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                body()
            stream.wait_stream(side)
            torch.cuda.synchronize()
            barrier()
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                for _ in range(RAG_LAYERS):
                    body()
            gr.replay()
            torch.cuda.synchronize()
            barrier()
            g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            g0.record(stream)
            for _ in range(reps):
                gr.replay()
            g1.record(stream)
            torch.cuda.synchronize()
            barrier()
            ms = max_over_ranks(g0.elapsed_time(g1) / reps)
            del gr   # holds NCCL work: released before the communicator
            torch.cuda.synchronize()
            return ms

        greps = max(3, min(args.steps, 10))
        step_ms = graph_ms(lambda: (decode_r(), exch_r()), greps)
        exch_ms = graph_ms(exch_r, greps)
        rag_layer = {"step_ms": step_ms, "oproj_exchange_ms": exch_ms, "reps": greps}
        del w_or, part_r
        rag = {"layer": rag_layer, "ms": max_over_ranks(r0.elapsed_time(r1) / rsteps), "steps": rsteps,
               "bytes_per_rank": int(lens_np.sum()) * 2 * Hkvr * D * 2, "sum_len": int(lens_np.sum()),
               "max_len": Lmax, "contiguous_cache_bytes": 2 * kr.numel() * 2}
        del kr, vr
        # the same batch over a paged cache: blocks of 256 rows handed out in a shuffled order,
        # the pool holding exactly the blocks the sequences need (no padding to the longest)
        import random
        from mllm_b200.runtime import PagedKVCache
        torch.cuda.empty_cache()
        bs = 256
        nblk = int(sum(-(-int(x) // bs) for x in lens_np))
        pk = PagedKVCache(num_blocks=nblk, num_kv_heads=Hkvr, head_dim=D, block_size=bs, max_seqs=RAG_B,
                          max_blocks_per_seq=-(-Lmax // bs), device=device)
        random.Random(RAG_SEED).shuffle(pk._free)
        pk.set_lengths([int(x) for x in lens_np])
        pk.k_pool.normal_(generator=gen)
        pk.v_pool.normal_(generator=gen)
        kvd = pk.descriptor()

        def decode_p():
            st = lib.mllm_decode_attention_paged_bf16(qr.data_ptr(), C.byref(kvd), pk.lengths.data_ptr(), RAG_B, Hr,
                                                      Hkvr, D, Lmax, scale, orr.data_ptr(), ws_r.data_ptr(),
                                                      ws_r_bytes, sh)
            assert st == 0, lib.mllm_attn_last_error()

        for _ in range(args.warmup):
            decode_p()
        barrier()
        torch.cuda.synchronize()
        r0.record(stream)
        for i in range(rsteps):
            decode_p()
        r1.record(stream)
        torch.cuda.synchronize()
        barrier()
        rag["paged_ms"] = max_over_ranks(r0.elapsed_time(r1) / rsteps)
        rag["paged_pool_bytes"] = 2 * pk.k_pool.numel() * 2
        rag["paged_block_size"] = bs
        del pk, qr, orr, ws_r

    clocks = sampler.stop() if rank == 0 else None
    if comm is not None:
        torch.cuda.synchronize()
        comm.close()
    return {"tp_parity": tp_parity, "elapsed_ms": elapsed_ms, "dec_ms": dec_ms, "unfused_ms": unfused_ms, "e2e_ms": e2e_ms, "pre": pre,
            "proj": proj,
            "rag": rag, "clocks": clocks,
            "launches_per_step": launches_per_step, "plan": (plan_rows.value, plan_chunks.value),
            "h2d": qkv.numel() * 2, "d2h": out.numel() * 2}


TP_B, TP_S, TP_STEPS = 2, 384, 2


def tp_parity_leg(rank, world, device, comm, barrier):
    """The head-sharded attention layer against the unsharded one, on every rank, for every
    o_proj exchange: a Qwen3-8B-shaped layer (hidden 4096, 32 q / 8 kv heads, head_dim 128,
    QK-norm, theta 1e6), batch 2, prefill of 384 rows then two decode steps, weights and inputs
    from one seed on every rank.  Each rank runs its kv-head group through mllm_b200.tp and its
    full output must lie within rtol = atol = 2e-2 of runtime.attention_block over all heads
    (the same path on one GPU).  Returns {"max_excess": ..., "ok": ..., "modes": {...}}; the
    excess is max(|got - ref| - (atol + rtol |ref|)) over ranks, steps and elements."""
    import torch
    import torch.distributed as dist
    from mllm_b200 import runtime as rt, tp
    g = torch.Generator(device=device).manual_seed(2024)
    r = lambda *shape, s=0.02: (s * torch.randn(*shape, device=device, generator=g)).bfloat16()
    w = {"w_q": r(H * D, HIDDEN), "w_k": r(HKV * D, HIDDEN), "w_v": r(HKV * D, HIDDEN), "w_o": r(HIDDEN, H * D)}
    gq = (1 + 0.1 * torch.randn(D, device=device, generator=g)).bfloat16()
    gk = (1 + 0.1 * torch.randn(D, device=device, generator=g)).bfloat16()
    xs = [r(TP_B, TP_S, HIDDEN, s=1.0)] + [r(TP_B, 1, HIDDEN, s=1.0) for _ in range(TP_STEPS)]
    pos = lambda i: torch.arange(TP_S, device=device) if i == 0 else torch.tensor([TP_S + i - 1], device=device)
    cache = rt.KVCache(TP_B, HKV, D, TP_S + TP_STEPS)
    ref = [rt.attention_block(x, w["w_q"], w["w_k"], w["w_v"], w["w_o"], H, HKV, D, THETA, pos(i), cache, gq, gk,
                              EPS).float() for i, x in enumerate(xs)]
    shard = tp.shard_heads(H, HKV, world, rank)
    wq, wk, wv, wo = tp.shard_weights(shard, D, w["w_q"], w["w_k"], w["w_v"], w["w_o"])
    modes = {}
    # Ulysses layout (tp.UlyssesLayout): this rank's token rows projected with the whole weights,
    # q/k/v to the head owners, attention on this rank's heads, rows back to their owners, o_proj
    # with the whole w_o; this rank's output rows against the same rows of the unsharded layer.
    # The decode steps (2 rows) run head-sharded with the all-reduce.
    lay = tp.UlyssesLayout(shard, H, HKV, D)
    c = rt.KVCache(TP_B, shard.num_kv_heads, D, TP_S + TP_STEPS)
    T = TP_B * TP_S
    Tn = T // world
    rows = slice(rank * Tn, (rank + 1) * Tn)
    w_packed = lay.pack_qkv_weights(w["w_q"], w["w_k"], w["w_v"])
    qkv_h = lay.heads_from_tokens_packed(lay.project(xs[0].view(T, HIDDEN)[rows], w_packed))
    Hr, Hkvr = shard.num_heads, shard.num_kv_heads
    qh = qkv_h[:, :Hr * D].view(TP_B, TP_S, Hr, D).transpose(1, 2)
    kh = qkv_h[:, Hr * D:(Hr + Hkvr) * D].view(TP_B, TP_S, Hkvr, D).transpose(1, 2)
    vh = qkv_h[:, (Hr + Hkvr) * D:].view(TP_B, TP_S, Hkvr, D).transpose(1, 2)
    att = rt.Attention.forward_projected(qh, kh, vh, None, Hr, Hkvr, D, THETA, pos(0), c, gq, gk, EPS)
    out_rows = torch.nn.functional.linear(lay.tokens_from_heads(att.reshape(T, Hr * D)), w["w_o"]).float()
    ref_rows = ref[0].view(T, HIDDEN)[rows]
    excess = float((out_rows - ref_rows).abs().sub(2e-2 + 2e-2 * ref_rows.abs()).max())
    for i in range(1, len(xs)):
        out = tp.tp_attention_block(xs[i], shard, D, THETA, pos(i), c, wq, wk, wv, wo, gq, gk, EPS,
                                    comm=comm).float()
        excess = max(excess, float((out - ref[i]).abs().sub(2e-2 + 2e-2 * ref[i].abs()).max()))
    torch.cuda.synchronize()
    t = torch.tensor([excess], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    modes["ulysses"] = {"max_excess": float(t.item()), "ok": float(t.item()) <= 0.0}
    barrier()
    # the same layout one sequence at a time (UlyssesLayout.run_sequences on a side stream): rank r
    # owns rows [r S/N, (r+1) S/N) of every sequence; its prefill rows against the same rows of
    # the unsharded layer
    Sn = TP_S // world
    out_seq = torch.empty(TP_B, Sn, HIDDEN, dtype=torch.bfloat16, device=device)
    seq_caches = [rt.KVCache(1, Hkvr, D, TP_S) for _ in range(TP_B)]

    def attend_p(b, qkv):
        qs = qkv[:, :Hr * D].view(1, TP_S, Hr, D).transpose(1, 2)
        ks = qkv[:, Hr * D:(Hr + Hkvr) * D].view(1, TP_S, Hkvr, D).transpose(1, 2)
        vs = qkv[:, (Hr + Hkvr) * D:].view(1, TP_S, Hkvr, D).transpose(1, 2)
        return rt.Attention.forward_projected(qs, ks, vs, None, Hr, Hkvr, D, THETA, pos(0), seq_caches[b], gq, gk,
                                              EPS).reshape(TP_S, Hr * D)

    def finish_p(b, rows):
        out_seq[b] = torch.nn.functional.linear(rows, w["w_o"])

    lay.run_sequences(lambda b: lay.project(xs[0][b, rank * Sn:(rank + 1) * Sn], w_packed), attend_p, finish_p,
                      TP_B, torch.cuda.Stream(device=device, priority=-1))
    torch.cuda.synchronize()
    ref_seq = ref[0][:, rank * Sn:(rank + 1) * Sn]
    t = torch.tensor([float((out_seq.float() - ref_seq).abs().sub(2e-2 + 2e-2 * ref_seq.abs()).max())],
                     dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    modes["ulysses_seq"] = {"max_excess": float(t.item()), "ok": float(t.item()) <= 0.0}
    barrier()
    for mode in ("nccl_chunked", "comm", "peer", "seqpar"):
        ex = {}
        if mode == "peer":
            ex = {TP_B * TP_S: tp.PeerExchange(TP_B * TP_S, HIDDEN), TP_B: tp.PeerExchange(TP_B, HIDDEN, sub=1)}
        elif mode == "seqpar":
            ex = {TP_B * TP_S: tp.SeqParallelOProj(TP_B * TP_S, HIDDEN, comm=comm)}
        c = rt.KVCache(TP_B, shard.num_kv_heads, D, TP_S + TP_STEPS)
        excess = -1e30
        for i, x in enumerate(xs):
            e = ex.get(x.shape[0] * x.shape[1])
            w_o_use = w["w_o"] if isinstance(e, tp.SeqParallelOProj) else wo
            out = tp.tp_attention_block(x, shard, D, THETA, pos(i), c, wq, wk, wv, w_o_use, gq, gk, EPS,
                                        overlap_chunks=3, exchange=e,
                                        comm=comm if mode in ("comm", "seqpar") else None).float()
            excess = max(excess, float((out - ref[i]).abs().sub(2e-2 + 2e-2 * ref[i].abs()).max()))
        torch.cuda.synchronize()
        for e in ex.values():
            if hasattr(e, "close"):
                e.close()
        t = torch.tensor([excess], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        modes[mode] = {"max_excess": float(t.item()), "ok": float(t.item()) <= 0.0}
        barrier()
    worst = max(m["max_excess"] for m in modes.values())
    return {"case": f"Qwen3-8B-shaped layer, batch {TP_B}, prefill {TP_S} rows + {TP_STEPS} decode steps, "
                    f"kv-head groups over {world} GPUs, vs the unsharded layer at rtol = atol = 2e-2",
            "max_excess": worst, "ok": worst <= 0.0, "modes": modes}


VAR_B, VAR_LMIN, VAR_LMAX, VAR_SEED = 32, 512, 8192, 77


def prefill_varlen_leg(args, lib, device, gen, Hr, Hkvr, scale, sh, stream, barrier, max_over_ranks, ksteps):
    """Packed prefill of 32 prompts of U[512, 8192] rows (seeded) over a paged cache, one
    mllm_prefill_attention_varlen_paged_bf16 launch, against one mllm_prefill_attention_paged_bf16
    launch per prompt on the same rows.  FLOPs = sum_b 4 H D S_b (S_b + 1) / 2."""
    import ctypes as C
    import numpy as np
    import torch
    from mllm_b200 import abi
    lens = np.random.default_rng(VAR_SEED).integers(VAR_LMIN, VAR_LMAX + 1, VAR_B).tolist()
    T, blk = sum(lens), 256
    nblk = [-(-L // blk) for L in lens]
    pool = torch.randn(sum(nblk), Hkvr, blk, D, device=device, generator=gen).bfloat16()
    vpool = torch.randn_like(pool)
    perm = torch.randperm(sum(nblk), generator=torch.Generator().manual_seed(VAR_SEED)).tolist()
    table = torch.zeros(VAR_B, max(nblk), dtype=torch.int32)
    k = 0
    for b, nb in enumerate(nblk):
        table[b, :nb] = torch.tensor(perm[k:k + nb], dtype=torch.int32)
        k += nb
    table = table.to(device)
    ps = pool.stride()
    kv = abi.PagedKV(pool.data_ptr(), vpool.data_ptr(), ps[0], ps[1], ps[2], sum(nblk), blk, table.data_ptr(),
                     table.stride(0), max(nblk))
    q = torch.randn(Hr, T, D, device=device, generator=gen).bfloat16()
    out = torch.empty(T, Hr * D, dtype=torch.bfloat16, device=device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=device)
    kvl = torch.tensor(lens, dtype=torch.int32, device=device)
    # the same prompts one launch each: Q [1, H, S, D] per prompt, the table row of that prompt
    q1 = [q[:, int(cu[b]):int(cu[b]) + L].unsqueeze(0).contiguous() for b, L in enumerate(lens)]
    o1 = [torch.empty(1, L, Hr * D, dtype=torch.bfloat16, device=device) for L in lens]
    kv1 = [abi.PagedKV(pool.data_ptr(), vpool.data_ptr(), ps[0], ps[1], ps[2], sum(nblk), blk,
                       table.data_ptr() + b * table.stride(0) * 4, table.stride(0), max(nblk)) for b in range(VAR_B)]

    def packed():
        st = lib.mllm_prefill_attention_varlen_paged_bf16(q.data_ptr(), C.byref(kv), cu.data_ptr(), kvl.data_ptr(),
                                                          VAR_B, Hr, Hkvr, D, T, max(lens), scale, out.data_ptr(), sh)
        assert st == 0, lib.mllm_attn_last_error()

    def one_each():
        for b, L in enumerate(lens):
            st = lib.mllm_prefill_attention_paged_bf16(q1[b].data_ptr(), C.byref(kv1[b]), 1, Hr, Hkvr, D, L, L,
                                                       scale, o1[b].data_ptr(), sh)
            assert st == 0, lib.mllm_attn_last_error()

    def timed(fn):
        for _ in range(2):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(ksteps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(e0.elapsed_time(e1)) / ksteps

    ms_packed, ms_each = timed(packed), timed(one_each)
    same = all(torch.equal(out[int(cu[b]):int(cu[b]) + L].view(torch.int16), o1[b][0].view(torch.int16))
               for b, L in enumerate(lens))
    fl = sum(4.0 * Hr * D * L * (L + 1) / 2 for L in lens)
    _, tf_peak, peak_src = load_peaks()
    tf = fl / (ms_packed * 1e-3) / 1e12
    return {"workload": f"{VAR_B} prompts of U[{VAR_LMIN}, {VAR_LMAX}] rows (seed {VAR_SEED}, {T} rows), "
                        f"{Hr} q / {Hkvr} kv heads, paged cache (256-row blocks, shuffled)",
            "value": tf, "unit": "TFLOP/s", "ms": ms_packed, "one_launch_per_prompt_ms": ms_each,
            "speedup": ms_each / ms_packed, "bit_identical_to_one_launch_per_prompt": same,
            "roofline": {"bound": "tensor", "kernel": "prefill_kernel<128> (packed)", "achieved": tf,
                         "peak": tf_peak, "unit": "TFLOP/s", "frac": tf / tf_peak, "peak_source": peak_src}}


def run_serve(args):
    """Continuous batching (mllm_b200.serving) against one request at a time, the way the
    reference's batch-1 Generate serves a queue (QwenRunner.cpp:420-545, Scheduler.cpp:45-77).
    Qwen3-8B geometry (36 layers, hidden 4096, 32/8 heads, SwiGLU 12288, vocab 151936), random
    bf16 weights; requests with prompt lengths U[64, 512] (seeded) and 32 new tokens each."""
    import numpy as np
    import torch
    from mllm_b200 import build
    from mllm_b200.serving import ContinuousBatcher, DecoderModel, DecoderShape
    build.build()
    shape = DecoderShape(vocab=151936, hidden=4096, layers=36, heads=32, kv_heads=8, head_dim=128,
                         intermediate=12288)
    model = DecoderModel(shape, seed=11)
    rng = np.random.default_rng(12)
    n_req, new_tok, serial_sample = args.serve_requests, 32, 4
    prompts = [rng.integers(0, shape.vocab, int(n)).tolist() for n in rng.integers(64, 513, n_req)]

    def serve(batch, reqs, graphs=True):
        bat = ContinuousBatcher(model, max_batch=batch, num_blocks=batch * 5 + 8, block_size=128, graphs=graphs)
        for p in reqs:
            bat.submit(p, new_tok)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        out = bat.run()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        serve.graph_steps, serve.steps = bat.graph_steps, bat.steps
        del bat
        torch.cuda.empty_cache()
        return dt, sum(len(t) for t in out.values()), sum(len(p) for p in reqs)

    def admit_ms(k, packed, reps=3):
        """Prefill of k prompts into an empty batch, as one packed pass (varlen epilogue and
        attention) or one forward per prompt; best of `reps` after one untimed pass."""
        reqs = prompts[:k]
        caches = model.new_caches(num_blocks=k * 5 + 8, block_size=128, max_seqs=k)
        best = None
        for rep in range(reps + 1):
            for c in caches:
                for i, p in enumerate(reqs):
                    c.release(i)
                    c.reserve(i, len(p) + new_tok)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            if packed:
                ids = torch.tensor([t for p in reqs for t in p], dtype=torch.int64, device="cuda")
                model.forward_packed(ids, [len(p) for p in reqs], [c.slot(0, k) for c in caches])
            else:
                for i, p in enumerate(reqs):
                    ids = torch.tensor([p], dtype=torch.int64, device="cuda")
                    model.forward(ids, torch.arange(len(p), device="cuda"), [c.slot(i) for c in caches])
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            if rep > 0:
                best = dt if best is None else min(best, dt)
        del caches
        torch.cuda.empty_cache()
        return best * 1e3, sum(len(p) for p in reqs)

    def step_ms(rows, graphs, steps=10):
        """Median wall-clock time of one steady decode step of `rows` live requests (sampling
        and the host read included), after admission and the step that records the graph."""
        bat = ContinuousBatcher(model, max_batch=rows, num_blocks=rows * 5 + 8, block_size=128, graphs=graphs)
        for p in prompts[:rows]:
            bat.submit(p, new_tok)
        bat.step()
        bat.step()
        times = []
        for _ in range(steps):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            bat.step()
            torch.cuda.synchronize()
            times.append((time.perf_counter() - t0) * 1e3)
        assert len(bat.live) == rows
        del bat
        torch.cuda.empty_cache()
        return statistics.median(times)

    serve(4, prompts[:4])     # warm-up: library set-up, cuBLAS handles, allocator
    n_admit = min(16, n_req)
    packed_ms, admit_tok = admit_ms(n_admit, True)
    single_ms, _ = admit_ms(n_admit, False)
    serve(args.serve_batch, prompts)   # warm-up at full size: the large packed prefill's allocations
    dt_e, tok_e, _ = serve(args.serve_batch, prompts, graphs=False)
    dt_b, tok_b, ptok_b = serve(args.serve_batch, prompts)
    steps_b, graph_b = serve.steps, serve.graph_steps
    dt_s, tok_s, ptok_s = serve(1, prompts[:serial_sample])
    rows = min(64, n_req)
    step_graph, step_eager = step_ms(rows, True), step_ms(rows, False)
    line = {"metric": "batched greedy serving through mllm_b200.serving (continuous batching over the paged KV cache)",
            "workload": f"Qwen3-8B geometry, random bf16 weights; {n_req} requests, prompts U[64, 512] tokens, "
                        f"{new_tok} new tokens each",
            "batched": {"max_batch": args.serve_batch, "seconds": dt_b, "new_tokens": tok_b, "prompt_tokens": ptok_b,
                        "new_tokens_per_s": tok_b / dt_b, "decode_steps": steps_b,
                        "decode_steps_from_graphs": graph_b},
            "batched_eager": {"seconds": dt_e, "new_tokens_per_s": tok_e / dt_e,
                              "note": "the same run with every decode step launched kernel by kernel"},
            "one_at_a_time": {"requests": serial_sample, "seconds": dt_s, "new_tokens": tok_s,
                              "prompt_tokens": ptok_s, "new_tokens_per_s": tok_s / dt_s},
            "speedup_new_tokens_per_s": (tok_b / dt_b) / (tok_s / dt_s),
            "decode_step_ms": {"rows": rows, "graph": step_graph, "eager": step_eager,
                               "timing": "wall clock per steady step, median of 10, sampling and host read included"},
            "prefill_admission": {"prompts": n_admit, "prompt_tokens": admit_tok, "packed_ms": packed_ms,
                                  "one_per_prompt_ms": single_ms, "speedup": single_ms / packed_ms,
                                  "timing": "wall clock, best of 3, 36 layers + final norm + lm_head"},
            "timing": "wall clock around ContinuousBatcher.run (prefills, decode steps, sampling, host reads)"}
    print(json.dumps(line))


def run_generate(args):
    """Full random-init Qwen3-8B (36 layers) through the reference's UNCHANGED QwenRunner, twice:
    built on the reference's own runtime headers and on the drop-in headers.  Batch 8 prompts
    of 2048 uniform-random ids, then greedy decode steps through IModelRunner::Forward (the runner
    picks prefill vs decode).  Reports tokens/s of both and greedy-token parity: per sequence the
    first step where the tokens differ and the reference's top-1/top-2 logit margin there."""
    import importlib.util
    import tempfile

    import numpy as np
    import torch
    from tests.qwen_model import QWEN3_8B, write_random_qwen3
    from mllm_b200.dropin.build_facade import runner_module_path

    def load(flavor):
        path = runner_module_path(flavor)
        spec = importlib.util.spec_from_file_location(os.path.basename(path).split(".")[0], path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod

    B, S, steps = 8, 2048, args.gen_steps
    rng = np.random.default_rng(2048)
    prompt = torch.from_numpy(rng.integers(0, QWEN3_8B.vocab, size=(B, S))).long()
    results = {}
    with tempfile.TemporaryDirectory(dir=args.model_dir) as d:
        t0 = time.time()
        write_random_qwen3(d, QWEN3_8B, seed=8)
        t_write = time.time() - t0
        ref_tokens = ref_margins = None
        ref_logits = []       # reference last-position logits per step (bf16, host)
        dropin_tf_logits = []  # drop-in logits under teacher forcing (bf16, host)
        tf = {}
        mods = {}
        graph_tokens = None
        for flavor in ("reference", "dropin", "dropin_graphs"):
            kind = "dropin" if flavor == "dropin_graphs" else flavor
            if kind not in mods:
                mods[kind] = load(kind)
            mod = mods[kind]
            if flavor == "dropin_graphs":
                # a fresh drop-in runner with its decode layers replayed as CUDA graphs: the timed
                # decode includes recording every layer (steps 2 and 3)
                os.environ["MLLM_B200_DECODE_GRAPHS"] = "1"
            runner = mod.Runner(d)
            if flavor == "dropin":
                # teacher forcing: the reference's own greedy tokens fed to the drop-in runner
                last = runner.forward(prompt)[:, -1].float()
                agree, diffs = [], []
                dropin_tf_logits.clear()
                for k in range(steps):
                    dropin_tf_logits.append(last.to(torch.bfloat16).cpu())
                    r = ref_logits[k].to(last.device).float()
                    diffs.append((last - r).abs().max(-1).values.cpu())
                    agree.append((last.argmax(-1).cpu() == ref_tokens[:, k]))
                    last = runner.forward(ref_tokens[:, k:k + 1])[:, -1].float()
                agree = torch.stack(agree, 1)
                diffs = torch.stack(diffs, 1)
                tf = {"argmax_agreement": float(agree.float().mean()),
                      "max_abs_logit_diff": float(diffs.max()), "mean_max_abs_logit_diff": float(diffs.mean())}
                for thr in (0.1, 0.25, 0.5):
                    sel = ref_margins > thr
                    tf[f"argmax_agreement_margin_gt_{thr}"] = (float(agree[sel].float().mean()) if sel.any() else None)
                    tf[f"steps_margin_gt_{thr}"] = int(sel.sum())
                runner.reset_cache()
            toks, margins = [], []
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            logits = runner.forward(prompt)
            last = logits[:, -1].float()
            del logits
            torch.cuda.synchronize()
            t_pre = time.perf_counter() - t0
            t0 = time.perf_counter()
            for _ in range(steps):
                if flavor == "reference":
                    ref_logits.append(last.to(torch.bfloat16).cpu())
                top2 = torch.topk(last, 2, dim=-1).values
                margins.append((top2[:, 0] - top2[:, 1]).cpu())
                nxt = last.argmax(-1, keepdim=True)          # greedy: first max wins
                toks.append(nxt.cpu())
                last = runner.forward(nxt.cpu())[:, -1].float()
            torch.cuda.synchronize()
            t_dec = time.perf_counter() - t0
            results[flavor] = {"prefill_s": t_pre, "decode_s": t_dec,
                               "prefill_tok_s": B * S / t_pre, "decode_tok_s": B * steps / t_dec}
            tokens = torch.cat(toks, 1)
            if flavor == "reference":
                ref_tokens, ref_margins = tokens, torch.stack(margins, 1)
            elif flavor == "dropin":
                new_tokens = tokens
            else:
                graph_tokens = tokens
            del runner
            torch.cuda.empty_cache()
            os.environ.pop("MLLM_B200_DECODE_GRAPHS", None)
    # fp32 floor: the same (bf16-valued) weights in fp32 through the reference runner, fed the
    # same tokens -- how far each bf16 runner's logits are from a higher-precision run.
    if args.fp32_floor:
        with tempfile.TemporaryDirectory(dir=args.model_dir) as d32:
            write_random_qwen3(d32, QWEN3_8B, seed=8, dtype="f32")
            runner = load("reference").Runner(d32)
            last = runner.forward(prompt)[:, -1].float()
            e_ref, e_new = [], []
            for k in range(steps):
                e_ref.append((ref_logits[k].to(last.device).float() - last).abs().max(-1).values.cpu())
                e_new.append((dropin_tf_logits[k].to(last.device).float() - last).abs().max(-1).values.cpu())
                last = runner.forward(ref_tokens[:, k:k + 1])[:, -1].float()
            del runner
            torch.cuda.empty_cache()
        e_ref = torch.stack(e_ref)
        e_new = torch.stack(e_new)
        tf["fp32_floor"] = {"reference_bf16_max_abs_vs_fp32": float(e_ref.max()),
                            "reference_bf16_mean_max_abs_vs_fp32": float(e_ref.mean()),
                            "dropin_bf16_max_abs_vs_fp32": float(e_new.max()),
                            "dropin_bf16_mean_max_abs_vs_fp32": float(e_new.mean())}
    same = (new_tokens == ref_tokens)
    first_div = []
    for b in range(B):
        bad = (~same[b]).nonzero()
        if len(bad) == 0:
            first_div.append({"seq": b, "diverged": False})
        else:
            k = int(bad[0])
            first_div.append({"seq": b, "diverged": True, "step": k,
                              "ref_top2_margin": float(ref_margins[b, k])})
    line = {"metric": "Qwen3-8B random-init greedy generation through the unchanged QwenRunner",
            "workload": f"batch {B} x {S}-token prompts + {steps} greedy steps, 36 layers, bf16",
            "reference_runner": results["reference"], "dropin_runner": results["dropin"],
            "speedup_prefill": results["reference"]["prefill_s"] / results["dropin"]["prefill_s"],
            "speedup_decode": results["reference"]["decode_s"] / results["dropin"]["decode_s"],
            "dropin_runner_decode_graphs": dict(
                results["dropin_graphs"],
                speedup_decode=results["reference"]["decode_s"] / results["dropin_graphs"]["decode_s"],
                tokens_identical_to_eager_dropin=float((graph_tokens == new_tokens).float().mean()),
                note="MLLM_B200_DECODE_GRAPHS=1 on a fresh runner; the timed decode includes recording "
                     "every layer"),
            "tokens_identical_fraction": float(same.float().mean()),
            "sequences_fully_identical": int(sum(1 for f in first_div if not f["diverged"])),
            "first_divergence": first_div, "teacher_forced": tf,
            "note": "reference decode steps include copying its per-step logits to the host (parity record)",
            "checkpoint_write_s": t_write}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--skip-prefill", action="store_true")
    ap.add_argument("--skip-ragged", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true", help="omit the CPU baseline leg (profiling runs)")
    ap.add_argument("--workload", default="decode", choices=["decode", "qwen3-8b-generate", "serve"],
                    help="decode: the headline line; qwen3-8b-generate: full-model runner parity + speed; "
                         "serve: continuous batching vs one request at a time")
    ap.add_argument("--serve-requests", type=int, default=64)
    ap.add_argument("--serve-batch", type=int, default=64)
    ap.add_argument("--gen-steps", type=int, default=128)
    ap.add_argument("--fp32-floor", action="store_true",
                    help="also run the reference runner on fp32 weights as the precision floor")
    ap.add_argument("--model-dir", default=None, help="where to write the random checkpoint (default: tmp)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "qwen3-8b-generate":
        run_generate(args)
        return
    if args.workload == "serve":
        run_serve(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n = max(args.gpus, world)
    config = {"workload": f"Qwen3-8B decode attention: batch {DEC_B} x 1 new token, bf16 KV cache "
                          f"{DEC_L} rows/seq, H={H} Hkv={HKV} D={D}, QK-norm, theta 1e6 (per rank)",
              "batch": DEC_B, "kv_len": DEC_L, "num_heads": H, "num_kv_heads": HKV, "head_dim": D,
              "parallelism": f"request-batch replicas x{n} (decode); kv-head groups /{n} (prefill)",
              "l2": "inputs larger than L2 (537 MB KV cache per rank > 126 MB)"}

    if args.impl == "reference":
        if rank != 0:
            return
        r = cpu_reference_decode(args.steps, args.warmup)
        line = {"metric": METRIC, "value": r["value"], "unit": "GB/s", "n_gpus": n, "steps": r["steps_timed"],
                "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "impl": "reference", "config": config,
                "cpu_baseline": {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the attention path has no CPU fallback)")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    res = run_gpu(args, rank, world, device)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    if rank != 0:
        return

    hbm_peak, tf_peak, peak_src = load_peaks()
    kv_bytes = decode_kv_bytes(DEC_B, HKV, DEC_L, D)
    ms = res["elapsed_ms"] / args.steps
    value = kv_bytes * n / (ms * 1e-3) / 1e9
    achieved = kv_bytes / (ms * 1e-3) / 1e9
    e2e_ms = res["e2e_ms"] / args.steps
    cpu = None
    if n == 1 and not args.skip_cpu:
        r = cpu_reference_decode(5, 1, budget_s=20.0)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    line = {"metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": n, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": config,
            "e2e": {"value": kv_bytes * n / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                    "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                    "ms_per_step": e2e_ms},
            "gpu_launches": res["launches_per_step"] * args.steps,
            "decode_plan": {"chunk_rows": res["plan"][0], "chunks_per_sequence": res["plan"][1],
                            "launches_per_step": res["launches_per_step"]},
            "unfused": {"ms_per_step": res["unfused_ms"], "decode_only_ms": res["dec_ms"],
                        "value": kv_bytes * n / (res["unfused_ms"] * 1e-3) / 1e9, "unit": "GB/s",
                        "note": "the same step as mllm_qkv_epilogue_bf16 + mllm_decode_attention_bf16"},
            "roofline": {"bound": "hbm",
                         "kernel": "decode_split_kernel<128, fused>" +
                                   (" + decode_combine_kernel" if res["launches_per_step"] > 1 else ""),
                         "timing": "K back-to-back fused decode steps between two CUDA events",
                         "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
                         "peak_source": peak_src, "traffic": profile_traffic("decode_qwen3_8b_b32_l4096")},
            "cpu_baseline": cpu, "clocks": res["clocks"]}
    if res["tp_parity"] is not None:
        line["tp_parity"] = res["tp_parity"]
    if res["proj"] is not None:
        pj = res["proj"]
        q_gbs = pj["bytes"] / (pj["ours_us"] * 1e-6) / 1e9
        line["qkv_projection"] = {
            "workload": f"Qwen3-8B q|k|v projections at decode, {DEC_B} tokens: [{DEC_B}x{HIDDEN}] x "
                        f"[{HIDDEN}x{(H + 2 * HKV) * D}] (three weights, one launch)",
            "timing": "per launch, 40 launches in a CUDA graph over a ring of 4 weight sets (192 MB > L2)",
            "us": pj["ours_us"], "cublas_three_gemms_us": pj["cublas_three_us"],
            "cublas_concatenated_us": pj["cublas_concat_us"],
            "speedup_vs_three_gemms": pj["cublas_three_us"] / pj["ours_us"],
            "roofline": {"bound": "hbm", "kernel": "linear_kernel<32>", "achieved": q_gbs, "peak": hbm_peak,
                         "unit": "GB/s", "frac": q_gbs / hbm_peak, "peak_source": peak_src,
                         "algorithmic_bytes": pj["bytes"]}}
        f8 = pj["fp8"]
        f8_gbs = f8["bytes"] / (f8["ours_us"] * 1e-6) / 1e9
        line["fp8_projection"] = {
            "workload": f"Qwen3-8B gate projection with FP8 weights, {DEC_B} tokens: [{DEC_B}x{HIDDEN}] x "
                        f"[{HIDDEN}x{f8['out_features']}] e4m3, 128 x 128 block scales",
            "timing": "per launch, 40 launches in a CUDA graph over a ring of 4 weight sets (201 MB of fp8 > L2)",
            "us": f8["ours_us"], "reference_route_us": f8["reference_route_us"],
            "cublas_bf16_weights_us": f8["cublas_bf16_weights_us"],
            "speedup_vs_reference_route": f8["reference_route_us"] / f8["ours_us"],
            "note": "reference_route: DequantizeFP8 (w.to(bf16) * scale.to(bf16)) then a cuBLAS GEMM, what "
                    "QwenRunner runs per layer per step; the outputs are the same bf16 GEMM of the same "
                    "dequantized weight",
            "roofline": {"bound": "hbm", "kernel": "linear_fp8_kernel<32>", "achieved": f8_gbs, "peak": hbm_peak,
                         "unit": "GB/s", "frac": f8_gbs / hbm_peak, "peak_source": peak_src,
                         "algorithmic_bytes": f8["bytes"]}}
    if res["pre"] is not None:
        p = res["pre"]
        fl = prefill_flops(PRE_B, H, D, PRE_S)
        line["prefill"] = {
            "workload": f"Qwen3-8B causal prefill attention, batch {PRE_B} x {PRE_S}, heads split over {n} GPU(s)",
            "value": fl / (p["pre_ms"] * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": p["pre_ms"],
            "steps": p["steps"],
            "tp_exchange": {"o_proj_ms": p["oproj_ms"], "allreduce_ms": p["allreduce_ms"],
                            "overlapped_ms": p["overlap_ms"], "peer_exchange_ms": p["peer_ms"],
                            "allreduce_bytes": p["allreduce_bytes"], "allreduce_busbw_gbs": p["allreduce_busbw_gbs"],
                            "note": "column-sharded o_proj GEMM + NCCL all-reduce of the [B*S, hidden] partials; "
                                    "overlapped_ms: GEMM in 4 pieces, each piece's all-reduce overlapping the "
                                    "next GEMM; peer_exchange_ms: GEMM pieces written to a buffer every rank "
                                    "can read; each owner's kernel pulls its rows from all ranks over NVLink, "
                                    "sums them and stores the result into every rank (no NCCL)"},
            "roofline": {"bound": "tensor", "kernel": "prefill_kernel<128>",
                         "achieved": fl / n / (p["attn_ms"] * 1e-3) / 1e12, "peak": tf_peak, "unit": "TFLOP/s",
                         "frac": fl / n / (p["attn_ms"] * 1e-3) / 1e12 / tf_peak, "peak_source": peak_src,
                         "traffic": profile_traffic("prefill_qwen3_8b_b4_s8192")},
            "varlen": p["varlen"]}
        epi_gbs = p["epi_bytes"] / (p["epi_ms"] * 1e-3) / 1e9
        line["prefill"]["qkv_epilogue"] = {
            "ms": p["epi_ms"], "tokens": PRE_B * PRE_S,
            "roofline": {"bound": "hbm", "kernel": "qkv_epilogue_tma_kernel<128, 1>", "achieved": epi_gbs,
                         "peak": hbm_peak, "unit": "GB/s", "frac": epi_gbs / hbm_peak, "peak_source": peak_src,
                         "algorithmic_bytes": p["epi_bytes"],
                         "note": "q/k/v head rows read once, q rows and the K/V cache rows written once"}}
        lm = p["layer_ms"]
        best = min(lm, key=lm.get)
        line["layer"] = {
            "workload": f"the whole attention layer of the Qwen3-8B prefill step (batch {PRE_B} x {PRE_S}): QKV "
                        f"epilogue + causal attention + o_proj + the o_proj exchange, heads split over {n} GPU(s)",
            "scaling": "strong", "ms": lm[best], "exchange": best, "ms_by_exchange": lm,
            "note": "single_gpu: o_proj GEMM with the whole w_o; gemm_then_*_allreduce: column-slice GEMM, then "
                    "the all-reduce of the [B*S, hidden] partial (torch NCCL, or the library's mllm_comm); "
                    "chunked_overlap: the GEMM in 4 pieces overlapping their all-reduces; seqpar_*: attention "
                    "rows all-to-all to their row's owner, full-K o_proj there, all-gather of the output rows "
                    "(torch NCCL, or mllm_comm for the all-gather); peer_exchange: pull-sum-push over peer memory; "
                    "microM_*: the 4 sequences in M micro-batches, each micro-batch's o_proj + exchange on a "
                    "high-priority stream while the next micro-batch's epilogue + attention runs; "
                    "micro1_ulysses_token_rows_io: the layer's input and output sharded by token rows "
                    "(mllm_b200.tp.UlyssesLayout: q/k/v all-to-all to the head owners, attention, all-to-all "
                    "back, o_proj of the rank's rows with the whole w_o) -- no output is replicated; "
                    "micro4_ulysses_per_sequence: the same layout one sequence at a time (rank r owns rows "
                    "[r S/N, (r+1) S/N) of every sequence), sequence b+1's input all-to-all and sequence "
                    "b-1's output all-to-all + o_proj on a side stream under sequence b's attention "
                    "(UlyssesLayout.run_sequences)"}
    if res["rag"] is not None:
        r = res["rag"]
        ach = r["bytes_per_rank"] / (r["ms"] * 1e-3) / 1e9
        line["ragged_decode"] = {
            "workload": f"Qwen3-14B decode over a ragged batch: {RAG_B} requests, cache lengths U[{RAG_LMIN}, "
                        f"{RAG_LMAX}] (seed {RAG_SEED}, sum {r['sum_len']}, max {r['max_len']}), H={RAG_H} "
                        f"Hkv={RAG_HKV} D={D}; one layer per call, kv-head groups /{n}",
            "value": ach * n, "unit": "GB/s", "ms_per_layer": r["ms"],
            "ms_per_step_all_layers": r["ms"] * RAG_LAYERS, "layers": RAG_LAYERS, "steps": r["steps"],
            "scaling": "strong", "higher_is_better": True,
            "roofline": {"bound": "hbm", "kernel": "decode_split_kernel<128> + decode_combine_kernel",
                         "achieved": ach, "peak": hbm_peak, "unit": "GB/s", "frac": ach / hbm_peak,
                         "peak_source": peak_src},
            "layer_step": {
                "ms_per_step_all_layers": r["layer"]["step_ms"],
                "ms_per_layer": r["layer"]["step_ms"] / RAG_LAYERS,
                "oproj_and_allreduce_ms_per_step": r["layer"]["oproj_exchange_ms"],
                "collective_share": r["layer"]["oproj_exchange_ms"] / r["layer"]["step_ms"],
                "timing": f"{RAG_LAYERS} layers recorded in one CUDA graph, replayed {r['layer']['reps']} times",
                "note": "per layer: decode over this rank's kv heads, o_proj of its q heads ([64, Hr*D] x "
                        "[5120, Hr*D]^T) and mllm_comm_all_reduce_bf16 of the [64, 5120] partial (no collective "
                        "at one GPU); oproj_and_allreduce_ms_per_step times those two alone"},
            "paged": {"value": r["bytes_per_rank"] * n / (r["paged_ms"] * 1e-3) / 1e9, "unit": "GB/s",
                      "ms_per_layer": r["paged_ms"], "block_size": r["paged_block_size"],
                      "cache_bytes_per_rank": r["paged_pool_bytes"],
                      "contiguous_cache_bytes_per_rank": r["contiguous_cache_bytes"],
                      "note": "mllm_decode_attention_paged_bf16 over a pool holding exactly the blocks the "
                              "sequences need, handed out in a shuffled order"}}
    print(json.dumps(line))


if __name__ == "__main__":
    main()
