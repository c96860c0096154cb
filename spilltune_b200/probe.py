"""Run one frozen-linear op at a given shape, for profiling and quick timing.

    python -m spilltune_b200.probe --op fwd --M 8192 --N 14336 --K 4096 [--iters 3] [--time]

With --experts E > 1, fwd/bwd run the grouped (MoE) kernels over M routed
rows: M / top_k tokens routed uniformly at random to `top_k` of E experts of
a stacked [E, N, K] record, and --rank gives every expert its own LoRA pair.

Each call is preceded by two warm-up calls, so an `ncu -s 2 -c 1` capture
selects the first measured launch.  --time prints CUDA-event timings instead.

    python -m spilltune_b200.probe --sweep

runs the kernel sweep of the benchmark plan instead: forward and backward
(LoRA rank 16, s = 2) of NF4-g128 weights N x K in {4096x4096, 1024x4096,
14336x4096, 4096x14336} at M in {1, 16, 256, 2048, 8192} tokens, one JSON line
each.  Each timing replays a CUDA graph of ten (256 MB buffer write + call)
pairs and subtracts a graph of the ten buffer writes alone, so the weights
come from HBM and host launch overhead is excluded.
"""
import argparse
import json

import torch

from . import codec, moe, ops


def _graph_us(fn, flush, reps=10):
    """Device time of fn() per call: graph of (flush, fn) pairs minus graph of flushes."""
    def timed(body):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(reps):
                body()
        g.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            g.replay()
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e) * 1e3)
        return best

    both = timed(lambda: (flush.add_(1), fn()))
    alone = timed(lambda: flush.add_(1))
    return (both - alone) / reps


def sweep():
    dev = torch.device("cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    r = 16
    for (N, K) in [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]:
        g = torch.Generator(device=dev).manual_seed(1)
        w = codec.encode(torch.randn(N, K, generator=g, device=dev) * 0.02, "nf4-g128")
        A = torch.randn(r, K, generator=g, device=dev) * 0.01
        B = torch.randn(N, r, generator=g, device=dev) * 0.01
        for M in (1, 16, 256, 2048, 8192):
            x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
            dy = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
            f = lambda: ops.fwd(x, w, A, B, 2.0)
            b = lambda: ops.bwd(dy, x, w, A, B, 2.0)
            for _ in range(2):
                f()
                b()
            torch.cuda.synchronize()
            tf, tb = _graph_us(f, flush), _graph_us(b, flush)
            wbytes = N * K // 2 + 4 * N * K // 128
            fl_f = 2 * M * N * K + 2 * M * K * r + 2 * M * r * N
            fl_b = 2 * M * N * K + 4 * M * N * r + 6 * M * K * r
            print(json.dumps({"N": N, "K": K, "M": M, "fwd_us": round(tf, 1), "bwd_us": round(tb, 1),
                              "fwd_tflops": round(fl_f / tf / 1e6, 1), "bwd_tflops": round(fl_b / tb / 1e6, 1),
                              "fwd_weight_tbs": round(wbytes / tf / 1e6, 3),
                              "bwd_weight_tbs": round(wbytes / tb / 1e6, 3)}), flush=True)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--op", choices=["fwd", "bwd", "dequant"], default="fwd")
    p.add_argument("--M", type=int, default=8192)
    p.add_argument("--N", type=int, default=14336)
    p.add_argument("--K", type=int, default=4096)
    p.add_argument("--rank", type=int, default=16)
    p.add_argument("--codec", default="nf4-g128")
    p.add_argument("--iters", type=int, default=1)
    p.add_argument("--time", action="store_true")
    p.add_argument("--experts", type=int, default=1)
    p.add_argument("--top-k", type=int, default=8)
    p.add_argument("--sweep", action="store_true")
    a = p.parse_args()
    if a.sweep:
        sweep()
        return
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    E = a.experts
    lead = (E,) if E > 1 else ()
    w = codec.encode(torch.randn(*lead, a.N, a.K, generator=g, device=dev) * 0.02, a.codec)
    x = torch.randn(a.M, a.K, generator=g, device=dev).to(torch.bfloat16)
    dy = torch.randn(a.M, a.N, generator=g, device=dev).to(torch.bfloat16)
    A = torch.randn(*lead, a.rank, a.K, generator=g, device=dev) * 0.01 if a.rank else None
    B = torch.randn(*lead, a.N, a.rank, generator=g, device=dev) * 0.01 if a.rank else None
    if E > 1:
        if a.op == "dequant" or a.M % a.top_k:
            raise SystemExit("--experts needs --op fwd|bwd and M divisible by --top-k")
        scores = torch.rand(a.M // a.top_k, E, generator=g, device=dev)
        segs = moe.expert_segments(scores.topk(a.top_k, dim=-1)[1], E)
        fn = {
            "fwd": lambda: moe.grouped_fwd(x, segs, w, A, B, 2.0),
            "bwd": lambda: moe.grouped_bwd(dy, x, segs, w, A, B, 2.0),
        }[a.op]
    else:
        out = torch.empty(a.N, a.K, dtype=torch.bfloat16, device=dev)
        fn = {
            "fwd": lambda: ops.fwd(x, w, A, B, 2.0),
            "bwd": lambda: ops.bwd(dy, x, w, A, B, 2.0),
            "dequant": lambda: ops.dequant(w, out=out),
        }[a.op]
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    if not a.time:
        for _ in range(a.iters):
            fn()
        torch.cuda.synchronize()
        return
    iters = max(a.iters, 10)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) / iters * 1e3
    flops = 2.0 * a.M * a.N * a.K * (1 if a.op != "dequant" else 0)
    print(json.dumps({"op": a.op, "M": a.M, "N": a.N, "K": a.K, "experts": E, "us": us,
                      "tflops": flops / us / 1e6 if flops else None}))


if __name__ == "__main__":
    main()
