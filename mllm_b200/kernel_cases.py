"""One hot kernel on one fixed workload, launched back to back: the command to time a kernel alone
with CUDA events, or to hand to a profiler (`ncu -k regex:<kernel> -s <warmup> -c 1 python -m
mllm_b200.kernel_cases <case>`).

Cases (Qwen3-8B attention geometry: 32 q heads, 8 kv heads, head_dim 128, hidden 4096):
  epilogue   QK-RMSNorm + RoPE + cache append of B x S prefill tokens (qkv_epilogue_tma_kernel)
  prefill    causal attention of B x S rows over a cache of S rows (prefill_kernel)
  decode     one query row per sequence over L cache rows, B sequences (decode_split_kernel)
  ragged     Qwen3-14B decode over 64 sequences of seeded lengths U[256, 32768], --kv-heads kv heads
             (5 q heads each): 8 is one GPU's share at 1 GPU, 1 at 8 GPUs
  linear     q|k|v projection of T tokens, bf16 weights (linear_kernel)
  linear_fp8 the same with e4m3 weights and 128 x 128 block scales (linear_fp8_kernel)

Prints one line: the case, its sizes and the mean milliseconds per launch over --iters launches
(after --warmup).  Inputs are seeded random data; every launch goes through the C-ABI.  With --graph
(the default for the projections, whose launches last about as long as a host call) the --iters
launches are recorded once in a CUDA graph and the graph is timed."""
import argparse
import json

import torch

from mllm_b200 import abi
from mllm_b200 import runtime as rt

H, HKV, D, HIDDEN = 32, 8, 128, 4096


def _epilogue(args, dev, g):
    B, S = args.batch, args.seq
    H, HKV = (args.heads, args.kv_heads) if args.heads else (32, 8)   # --heads: one GPU's share
    row = (H + 2 * HKV) * D
    qkv = (torch.randn(B, S, row, device=dev, generator=g) * 0.5).bfloat16()
    q = qkv[..., : H * D].view(B, S, H, D).transpose(1, 2)
    k = qkv[..., H * D:(H + HKV) * D].view(B, S, HKV, D).transpose(1, 2)
    v = qkv[..., (H + HKV) * D:].view(B, S, HKV, D).transpose(1, 2)
    gq = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).bfloat16()
    gk = (1 + 0.1 * torch.randn(D, device=dev, generator=g)).bfloat16()
    pos = torch.arange(S, dtype=torch.int64, device=dev)
    cache = rt.KVCache(B, HKV, D, S, device=dev)
    q_out = torch.empty(B, H, S, D, dtype=torch.bfloat16, device=dev)
    start = torch.zeros(B, dtype=torch.int32, device=dev)
    csb, csh, cst = cache.strides

    def launch():
        abi.call("mllm_qkv_epilogue_bf16", q.data_ptr(), q.stride(0), q.stride(2), q.stride(1),
                 k.data_ptr(), k.stride(0), k.stride(2), k.stride(1), v.data_ptr(), v.stride(0), v.stride(2),
                 v.stride(1), B, S, H, HKV, D, pos.data_ptr(), 0, 1, 1e6, None, None, 0, 0, gq.data_ptr(),
                 gk.data_ptr(), 1e-6, q_out.data_ptr(), cache.key_buf.data_ptr(), cache.value_buf.data_ptr(),
                 csb, csh, cst, S, start.data_ptr(), 0, abi.stream_handle())
    return launch, {"batch": B, "seq": S, "heads": H, "kv_heads": HKV, "bytes": 2 * B * S * row * 2}


def _prefill(args, dev, g):
    B, S = args.batch, args.seq
    cache = rt.KVCache(B, HKV, D, S, device=dev)
    cache.key_buf.normal_(generator=g)
    cache.value_buf.normal_(generator=g)
    cache.set_lengths([S] * B)
    q = torch.randn(B, H, S, D, device=dev, generator=g).bfloat16()

    def launch():
        rt.prefill_attention(q, cache, HKV)
    return launch, {"batch": B, "seq": S, "flop": 4 * B * H * D * S * (S + 1) // 2}


def _decode(args, dev, g):
    B, L = args.batch, args.kv_len
    cache = rt.KVCache(B, HKV, D, L, device=dev)
    cache.key_buf.normal_(generator=g)
    cache.value_buf.normal_(generator=g)
    cache.set_lengths([L] * B)
    q = torch.randn(B, H, 1, D, device=dev, generator=g).bfloat16()

    def launch():
        rt.decode_attention(q, cache, HKV, max_kv_len=L)
    return launch, {"batch": B, "kv_len": L, "bytes": 2 * B * HKV * L * D * 2}


def _ragged(args, dev, g):
    import numpy as np
    B, rep = 64, 5
    lens = np.random.default_rng(14).integers(256, 32768 + 1, size=B)
    hkv = args.kv_heads
    L = int(lens.max())
    cache = rt.KVCache(B, hkv, D, L, device=dev)
    cache.key_buf.normal_(generator=g)
    cache.value_buf.normal_(generator=g)
    cache.set_lengths([int(x) for x in lens])
    q = torch.randn(B, hkv * rep, 1, D, device=dev, generator=g).bfloat16()

    def launch():
        rt.decode_attention(q, cache, hkv, max_kv_len=L)
    return launch, {"kv_heads": hkv, "batch": B, "bytes": int(lens.sum()) * hkv * D * 2 * 2}


def _linear(args, dev, g, fp8):
    """Launches cycle through a ring of weight sets larger than L2 (126 MB), so that every launch
    streams its weights from HBM."""
    T = args.tokens
    x = torch.randn(T, HIDDEN, device=dev, generator=g).bfloat16()
    ws = [torch.randn(n, HIDDEN, device=dev, generator=g).mul_(0.02).bfloat16() for n in (H * D, HKV * D, HKV * D)]
    count = [0]
    if fp8:
        w0 = rt.Fp8Weight.quantize(torch.cat(ws))
        nbytes = w0.w.numel() + w0.scale_inv.numel() * 4
        ring = [w0] + [rt.Fp8Weight(w0.w.clone(), w0.scale_inv.clone()) for _ in range(-(-256 * 2**20 // nbytes) - 1)]

        def launch():
            rt.linear_fp8(x, ring[count[0] % len(ring)])
            count[0] += 1
        return launch, {"tokens": T, "bytes": nbytes, "ring": len(ring)}
    nbytes = sum(t.numel() for t in ws) * 2
    ring = [ws] + [[t.clone() for t in ws] for _ in range(-(-256 * 2**20 // nbytes) - 1)]

    def launch():
        rt.linear(x, ring[count[0] % len(ring)])
        count[0] += 1
    return launch, {"tokens": T, "bytes": nbytes, "ring": len(ring)}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("case", choices=["epilogue", "prefill", "decode", "ragged", "linear", "linear_fp8"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--kv-len", type=int, default=4096)
    ap.add_argument("--tokens", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=1,
                    help="ragged: kv heads (Qwen3-14B has 8); epilogue: kv heads with --heads")
    ap.add_argument("--heads", type=int, default=0,
                    help="epilogue: q heads (0: the whole Qwen3-8B, 32 q / 8 kv heads; 4 with --kv-heads 1 is "
                         "one GPU's share at 8 GPUs)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--graph", action=argparse.BooleanOptionalAction, default=None,
                    help="time the launches as one CUDA graph (default: on for linear and linear_fp8)")
    args = ap.parse_args(argv)
    if args.graph is None:
        args.graph = args.case in ("linear", "linear_fp8", "ragged")
    if args.batch is None:
        args.batch = 32 if args.case == "decode" else 4
    if not torch.cuda.is_available():
        raise SystemExit("kernel_cases: needs a CUDA device")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1)
    if args.case == "epilogue":
        launch, info = _epilogue(args, dev, g)
    elif args.case == "prefill":
        launch, info = _prefill(args, dev, g)
    elif args.case == "decode":
        launch, info = _decode(args, dev, g)
    elif args.case == "ragged":
        launch, info = _ragged(args, dev, g)
    else:
        launch, info = _linear(args, dev, g, args.case == "linear_fp8")
    for _ in range(args.warmup):
        launch()
    torch.cuda.synchronize()
    run = lambda: [launch() for _ in range(args.iters)]
    if args.graph:
        graph = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        scratch = rt.GraphScratch()   # the graph's workspaces: alive as long as the graph
        with torch.cuda.stream(stream):
            with rt.graph_scratch(scratch):
                graph.capture_begin()
                run()
                graph.capture_end()
        torch.cuda.current_stream().wait_stream(stream)
        graph.replay()
        torch.cuda.synchronize()
        run = graph.replay
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.iters
    info.update(case=args.case, ms=ms, graph=args.graph)
    if "bytes" in info:
        info["gb_s"] = info["bytes"] / ms / 1e6
    if "flop" in info:
        info["tflop_s"] = info["flop"] / ms / 1e9
    print(json.dumps(info))


if __name__ == "__main__":
    main()
