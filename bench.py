#!/usr/bin/env python
"""Throughput of the frozen-linear hot path of Llama-3-8B NF4 LoRA streaming training.

One step = one training pass of the 32-layer frozen-linear stack over one
micro-batch (micro-batch 4 x seq 2048 = 8192 tokens per GPU):
  forward        : for each layer, q,k,v,o,gate,up,down  Y = X.W^T + s.(X.A^T).B^T, as five
                   calls: q/k/v fused (they share their input and sit back to back
                   in the layer image), o, gate, up, down
  recompute+bwd  : for each layer in reverse, the recomputed forward of every
                   projection (StreamingBlockFunction.backward reruns the block,
                   ram_vram_finetune/training/recompute.py:85-105) and its
                   backward dX, dA, dB (recompute.py:102-127)
  data parallel  : NCCL all-reduce of each layer's LoRA gradients (N > 1)
  optimizer      : fused AdamW (lr 1e-4) over every LoRA A/B.
Weights are NF4 group-128 (the reference's group-128 byte layout) drawn from
N(0, 0.02) and encoded on the GPU; LoRA rank 16, alpha 32 on all seven targets;
activations and upstream gradients are synthetic N(0,1) bf16 tensors in two
alternating per-layer buffer sets (each layer touches ~2 GB, far above L2).

`value`  : tokens/s with every packed layer resident in HBM.
`e2e`    : tokens/s through the public API with host buffers: packed layers in
           pinned host memory streamed by PackedSlotSession (2 VRAM slots,
           one-layer prefetch on a copy stream, reloaded for the backward like
           the reference; with N > 1 each rank copies 1/N of every layer and the
           slot is all-gathered over NVLink), the stack input copied H2D and the
           step's gradient norm read back D2H every step.
"""
import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, KV = 4096, 14336, 1024
# name, out_features N, in_features K, input buffer
PROJ = [("q_proj", HIDDEN, HIDDEN, "attn"), ("k_proj", KV, HIDDEN, "attn"), ("v_proj", KV, HIDDEN, "attn"),
        ("o_proj", HIDDEN, HIDDEN, "o"), ("gate_proj", INTER, HIDDEN, "mlp"), ("up_proj", INTER, HIDDEN, "mlp"),
        ("down_proj", HIDDEN, INTER, "down")]
INPUT_WIDTH = {"attn": HIDDEN, "o": HIDDEN, "mlp": HIDDEN, "down": INTER}
RANK, ALPHA = 16, 32.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["llama3-8b", "qwen3-30b-a3b", "deepseek-v3-6l"], default="llama3-8b",
                   help="llama3-8b: the headline step (Llama-3-8B stack, 32 layers); qwen3-30b-a3b: the Qwen3-MoE "
                        "30B-A3B stack; deepseek-v3-6l: DeepSeek-V3 truncated to 6 layers (3 dense, 3 MoE)")
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--tokens", type=int, default=8192, help="tokens per GPU per step (micro-batch 4 x seq 2048)")
    p.add_argument("--codec", default="nf4-g128")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--cpu-passes", type=int, default=2,
                   help="timed one-layer passes of the reference CPU path for this arm's cpu_baseline")
    p.add_argument("--no-ref-gpu", action="store_true", help="reference arm: skip the reference's GPU path")
    # single-op and sweep modes (for profiling; no JSON bench line)
    p.add_argument("--op", choices=["fwd", "bwd", "dequant"], default=None,
                   help="run one frozen-linear call at --M/--N/--K instead of the training step")
    p.add_argument("--M", type=int, default=8192)
    p.add_argument("--N", type=int, default=14336)
    p.add_argument("--K", type=int, default=4096)
    p.add_argument("--rank", type=int, default=16)
    p.add_argument("--iters", type=int, default=1)
    p.add_argument("--time", action="store_true")
    p.add_argument("--experts", type=int, default=1)
    p.add_argument("--ts", action="store_true", help="--op bwd: pass the forward's Ts (fl_bwd_ts, the step's path)")
    p.add_argument("--top-k", type=int, default=8)
    p.add_argument("--sweep", action="store_true", help="kernel sweep: 4 Llama-3-8B shapes x M in {1..8192}")
    p.add_argument("--sweep-m", default="1,16,256,2048,8192", help="--sweep: token counts, comma separated")
    p.add_argument("--no-split", action="store_true",
                   help="--op/--sweep: calls never split their reduction (the one-pass-per-tile order)")
    return p.parse_args()


# ---------------------------------------------------------------- distributed
def init_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def host_link_gbs(dev, nbytes, reps=5):
    """Pinned host -> device copy bandwidth for one buffer of nbytes (best of reps, CUDA
    events on a stream of its own): the link the slot session's copies use."""
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    best = float("inf")
    with torch.cuda.stream(stream):
        for _ in range(reps + 1):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            dst.copy_(src, non_blocking=True)
            e.record(stream)
            e.synchronize()
            best = min(best, s.elapsed_time(e) / 1e3)
    del src, dst
    return nbytes / best / 1e9


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = str(gpu_index)
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9 or f[0] != self.gpu:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- model
# Calls per layer: q, k and v share their input and run as one fused call over
# their adjacent records (one weight pass and one read of X instead of three,
# and the narrow k/v GEMMs no longer leave most SMs idle); gate and up are
# measured faster as two calls (the wide fused GEMM gains nothing, the
# low-rank kernels of a rank-32 branch cost more).  Name, members, input.
GROUPS = [("qkv", ("q_proj", "k_proj", "v_proj"), "attn"), ("o", ("o_proj",), "o"),
          ("gate", ("gate_proj",), "mlp"), ("up", ("up_proj",), "mlp"), ("down", ("down_proj",), "down")]
SHAPE = {name: (N, K) for name, N, K, _src in PROJ}
DOMINANT_GROUP = "gate"


class GroupLoRA:
    """The LoRA factors of one fused group as one branch: A = [A_1; A_2; ...]
    ([n r, K]) and B = blockdiag(B_1, B_2, ...) ([sum N_i, n r]); every member
    keeps its own rank-16 factors (views of the diagonal blocks).  The
    off-diagonal blocks of B start at zero and their gradient is masked to zero
    after every backward, so AdamW (element-wise) keeps them at zero: the same
    update as separate per-projection factors."""

    def __init__(self, members, g, device):
        K = SHAPE[members[0]][1]
        Ns = [SHAPE[m][0] for m in members]
        n = len(members)
        self.A = (torch.randn(n * RANK, K, generator=g, device=device) * 0.01).requires_grad_(True)
        B = torch.zeros(sum(Ns), n * RANK, device=device)
        self.mask = torch.zeros_like(B) if n > 1 else None
        row = 0
        for i, N in enumerate(Ns):
            B[row:row + N, i * RANK:(i + 1) * RANK] = torch.randn(N, RANK, generator=g, device=device) * 0.01
            if self.mask is not None:
                self.mask[row:row + N, i * RANK:(i + 1) * RANK] = 1.0
            row += N
        self.B = B.requires_grad_(True)
        self.A.grad = torch.zeros_like(self.A)
        self.B.grad = torch.zeros_like(self.B)

    def params(self):
        return (self.A, self.B)


def build_model(layers, codec_name, device, seed):
    """Per layer: the seven records packed into one device buffer laid out like
    a slot image (so q/k/v and gate/up are adjacent), and one GroupLoRA per
    group.  Returns (buffers, host-order records {name: PackedWeight view}, loras)."""
    from spilltune_b200 import codec, streaming
    g = torch.Generator(device=device).manual_seed(seed)
    bufs, weights, loras = [], [], []
    for _ in range(layers):
        layer = {}
        for name, N, K, _src in PROJ:
            w = torch.randn(N, K, generator=g, device=device) * 0.02
            layer[name] = codec.encode(w, codec_name)
            del w
        buf, views = streaming.pack_layer(layer, device)
        del layer
        bufs.append(buf)
        weights.append(views)
        loras.append({gname: GroupLoRA(members, g, device) for gname, members, _src in GROUPS})
    return bufs, weights, loras


def make_buffers(tokens, device, seed):
    g = torch.Generator(device=device).manual_seed(seed + 1)
    sets = []
    for _ in range(2):
        x = {k: torch.randn(tokens, w, generator=g, device=device).to(torch.bfloat16) for k, w in INPUT_WIDTH.items()}
        dy = {gname: torch.randn(tokens, sum(SHAPE[m][0] for m in members), generator=g,
                                 device=device).to(torch.bfloat16) for gname, members, _s in GROUPS}
        sets.append((x, dy))
    return sets


class Step:
    """One training step of the frozen-linear stack (see module docstring):
    per layer five calls (q/k/v fused, o, gate, up, down), forward, then
    recompute + backward in reverse layer order, then AdamW."""

    def __init__(self, weights_for, loras, bufs, world, optimizer, timed_name=DOMINANT_GROUP):
        from spilltune_b200 import ops
        self.ops = ops
        self.weights_for = weights_for
        self.loras = loras
        self.bufs = bufs
        self.world = world
        self.opt = optimizer
        self.scale = ALPHA / RANK
        self.timed_name = timed_name
        self.record = False
        self.events = []
        self.launches = 0

    def _record(self, W, members):
        if len(members) == 1:
            return W[members[0]]
        cat = self.ops.concat_records([W[m] for m in members])
        if cat is None:
            raise RuntimeError("fused group records are not adjacent in the layer image")
        return cat

    def _fwd(self, x, w, lora, name, return_ts=False):
        if self.record and name == self.timed_name:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = self.ops.fwd(x, w, lora.A, lora.B, self.scale, return_ts=return_ts)
            e.record()
            self.events.append((s, e))
        else:
            out = self.ops.fwd(x, w, lora.A, lora.B, self.scale, return_ts=return_ts)
        # Kernels of one fl_fwd call at these sizes: factor prepass, lora_down, GEMM.
        self.launches += 3
        return out

    def __call__(self):
        L = len(self.loras)
        for l in range(L):
            x, _ = self.bufs[l % 2]
            with self.weights_for(l, "forward") as W:
                for gname, members, src in GROUPS:
                    self._fwd(x[src], self._record(W, members), self.loras[l][gname], gname)
        from spilltune_b200.dp import LoRAGradReducer
        reducer = LoRAGradReducer(average=True)
        for l in reversed(range(L)):
            x, dy = self.bufs[l % 2]
            with self.weights_for(l, "backward") as W:
                for gname, members, src in reversed(GROUPS):
                    lora = self.loras[l][gname]
                    w = self._record(W, members)
                    # Recompute; the backward reuses its Ts = bf16(s * x . A^T)
                    # as the reference's autograd reuses F.linear(x, A).
                    _y, ts = self._fwd(x[src], w, lora, gname, return_ts=True)
                    self.ops.bwd(dy[gname], x[src], w, lora.A, lora.B, self.scale, dA=lora.A.grad,
                                 dB=lora.B.grad, accumulate=False, ts=ts)
                    # prepass(B), lora_down(Us; with rank <= 16 also dB), backward GEMM,
                    # lora_grad(dA) [, lora_grad(dB) above rank 16]
                    self.launches += 4 if lora.A.shape[0] <= 16 else 5
                    if lora.mask is not None:
                        lora.B.grad.mul_(lora.mask)  # no gradient for the zero blocks
            # Data parallel: this layer's LoRA gradients are final; all-reduce
            # them on a side stream while the next layer recomputes.
            reducer.reduce([t.grad for gname, _m, _s in GROUPS for t in self.loras[l][gname].params()])
        reducer.finish()
        self.opt.step()


def algorithmic_fwd_flops(M, N, K, r):
    return 2.0 * M * N * K + 2.0 * M * K * r + 2.0 * M * r * N


def step_flops(M, layers):
    f = b = 0.0
    for _name, N, K, _s in PROJ:
        f += algorithmic_fwd_flops(M, N, K, RANK)
        b += 2.0 * M * N * K + 4.0 * M * N * RANK + 4.0 * M * RANK * K + 2.0 * M * K * RANK
    return layers * (2 * f + b)


def load_profile_traffic():
    path = os.path.join(ROOT, "profiles", "fl_fwd_gate_8192x14336x4096.json")
    try:
        with open(path) as f:
            return json.load(f).get("dram_bytes_per_launch")
    except (OSError, ValueError):
        return None


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return d["bf16_tflops_sustained"], d["hbm_gbs"], "measured"
    except (OSError, ValueError, KeyError):
        return 1400.0, 6650.0, "fallback"


# ---------------------------------------------------------------- the reference's own path
class ReferenceLayerPass:
    """One layer of the step through the reference's own implementation of the
    path, restated by the oracle (test infrastructure; the reference itself is
    pure Python and does not travel to the GPU box):

    * ``SlotSession.load`` (memory.py:224-229) decodes every packed matrix of
      the layer into a BF16 slot with ``decode_into`` (quantization/codecs.py:
      158-170; ``oracle.codec.decode_torch``, bit-exact), once for the forward
      and again for the recompute;
    * ``LoRAProjection.forward`` (finetune/lora.py:205-220): BF16 ``F.linear``
      plus the two FP32 LoRA ``F.linear``s, for q, k, v, o, gate, up, down;
    * ``StreamingBlockFunction.backward`` (training/recompute.py:85-127): the
      recomputed forward and its autograd VJP (dX, dA, dB) per projection;
    * the FP32 AdamW update of the layer's LoRA factors (finetune/optimizer.py).

    On the CPU this is the reference's CPU path (torch with every host thread);
    on a CUDA device it is the reference's GPU path (torch elementwise decode +
    cuBLAS).  Weights are random packed records with the statistics of
    NF4/int4-encoded N(0, 0.02) weights, in two alternating layer sets."""

    def __init__(self, tokens, codec_name, device, seed=3, sets=2):
        import oracle.codec as oc
        import oracle.linear as ol
        from spilltune_b200 import codec
        self.oc, self.ol = oc, ol
        self.device = torch.device(device)
        self.tokens = tokens
        g = torch.Generator().manual_seed(seed)
        lut = (codec.NF4_LUT if codec_name == "nf4-g128" else codec.INT4_SYM_LUT).to(self.device)
        self.lut = lut
        self.sets = []
        for _ in range(sets):
            recs = {}
            for name, N, K, _src in PROJ:
                groups = N * K // 128
                payload = torch.randint(0, 256, (groups * 64,), dtype=torch.uint8, generator=g)
                scales = (0.02 * (2.5 + 0.3 * torch.rand(groups, generator=g))).float()
                recs[name] = (payload.to(self.device), scales.to(self.device), N, K)
            self.sets.append(recs)
        self.slot = {name: torch.empty(N, K, dtype=torch.bfloat16, device=self.device) for name, N, K, _s in PROJ}
        self.xs = {k: torch.randn(tokens, w, generator=g).to(torch.bfloat16).to(self.device)
                   for k, w in INPUT_WIDTH.items()}
        self.dys = {name: torch.randn(tokens, N, generator=g).to(torch.bfloat16).to(self.device)
                    for name, N, _K, _s in PROJ}
        self.lora = {}
        for name, N, K, _s in PROJ:
            A = (torch.randn(RANK, K, generator=g) * 0.01).to(self.device).requires_grad_(True)
            B = (torch.randn(N, RANK, generator=g) * 0.01).to(self.device).requires_grad_(True)
            self.lora[name] = (A, B, torch.zeros_like(A.detach()), torch.zeros_like(B.detach()))
        params = [t for A, B, _a, _b in self.lora.values() for t in (A, B)]
        self.opt = torch.optim.AdamW(params, lr=1e-4, foreach=False)

    def _load(self, recs):
        for name, (payload, scales, N, K) in recs.items():
            self.oc.decode_torch(payload, scales, N * K, self.lut, self.slot[name])

    def __call__(self, layer):
        s = ALPHA / RANK
        recs = self.sets[layer % len(self.sets)]
        self._load(recs)                                        # forward load
        with torch.no_grad():
            for name, _N, _K, src in PROJ:
                A, B, _ga, _gb = self.lora[name]
                self.ol.lora_forward_reference(self.xs[src], self.slot[name], A, B, s)
        self._load(recs)                                        # reload for the recompute
        for name, _N, _K, src in reversed(PROJ):
            A, B, ga, gb = self.lora[name]
            _y, _dx, da, db = self.ol.lora_backward_reference(self.xs[src], self.slot[name], A, B, s,
                                                              self.dys[name])
            ga.copy_(da)
            gb.copy_(db)
            A.grad, B.grad = ga, gb
        self.opt.step()


def reference_cpu_sample(tokens, codec_name, steps, warm=1, threads=None):
    """Time `steps` one-layer passes of the reference's CPU path (after `warm`
    untimed ones).  Every layer of the 32-layer stack has the same shapes and
    cost, so the stack's tokens/s is tokens / (32 x one layer pass)."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    run = ReferenceLayerPass(tokens, codec_name, "cpu")
    for i in range(warm):
        run(i)
    times = []
    for i in range(steps):
        t0 = time.perf_counter()
        run(i)
        times.append(time.perf_counter() - t0)
    layer_s = statistics.median(times)
    return {"value": tokens / (32 * layer_s), "unit": "tokens/s", "cores": threads, "kind": "port",
            "layer_seconds": times, "tokens": tokens,
            "sample": f"{steps} timed one-layer passes ({tokens} tokens, 7 projections, 2 decode_into loads, "
                      f"fwd + recompute + bwd + AdamW) of the 32-layer stack, median {layer_s:.2f} s; "
                      f"tokens/s = tokens / (32 x median layer pass)"}


def reference_gpu_torch(tokens, codec_name, steps, warmup, layers=32):
    """The reference's GPU path (torch decode_into on the device, cuBLAS BF16
    F.linear, FP32 LoRA F.linears, autograd VJP, AdamW) over the whole
    `layers`-layer step on cuda:0, timed with CUDA events: the comparator the
    fused kernels replace."""
    dev = torch.device("cuda", torch.cuda.current_device())
    run = ReferenceLayerPass(tokens, codec_name, dev)
    step = lambda: [run(l) for l in range(layers)]
    for _ in range(max(1, warmup)):
        step()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    return {"value": tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "what": f"reference GPU path restated (torch decode_into + cuBLAS + FP32 LoRA + autograd + AdamW), "
                    f"{layers} layers x 7 projections, {tokens} tokens, weights resident packed in HBM"}


def bench_config(args, world):
    """The workload both arms report (the reference arm times the same step on the host)."""
    return {"workload": "llama3-8b frozen-linear stack: 32 layers x (q,k,v,o,gate,up,down), "
                        "fwd + recompute + bwd(dX,dA,dB) + AdamW",
            "layers": args.layers, "tokens_per_gpu": args.tokens, "micro_batch": 4, "seq_len": 2048, "rank": RANK,
            "alpha": ALPHA, "codec": args.codec, "parallelism": f"dp{world}",
            "l2": "inputs > L2 (per-layer working set ~2 GB, alternating buffer sets)"}


def run_reference(args, world, rank):
    """The reference arm: each step is one measured one-layer pass of the
    reference's CPU path at the full config (8192 tokens, 7 projections);
    ms_per_step is that pass's wall time and value the stack's tokens/s
    (tokens / (32 x median pass)).  Adds the reference's GPU path on cuda:0
    (ref_gpu_torch) when a GPU is present."""
    if rank != 0:
        return 0
    steps = max(1, args.steps)
    info = reference_cpu_sample(args.tokens, args.codec, steps, warm=min(1, max(0, args.warmup)))
    value = info["value"]
    layer_ms = 1e3 * statistics.median(info["layer_seconds"])
    gpu = None
    if torch.cuda.is_available() and not args.no_ref_gpu:
        gpu = reference_gpu_torch(args.tokens, args.codec, steps=min(steps, 3), warmup=1)
    line = {"metric": "train tokens/s (8B NF4 LoRA frozen-linear stack)", "value": value, "unit": "tokens/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": steps, "warmup": args.warmup,
            "ms_per_step": layer_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": bench_config(args, world),
            "step_is": {"layers_timed_per_step": 1, "layers_in_model": 32, "tokens_per_step": args.tokens,
                        "timed_passes": steps,
                        "value_formula": "tokens_per_step / (32 x median one-layer pass seconds)"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": info["cores"], "kind": "port",
                             "sample": info["sample"]},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "ref_gpu_torch": gpu}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- single-op and sweep modes
# `python bench.py --op fwd|bwd|dequant --M .. --N .. --K ..` runs one frozen-linear
# call at a given shape (two warm-up calls first, so `ncu -s 2 -c 1` selects the
# first measured launch; --time prints CUDA-event timings).  With --experts E > 1,
# fwd/bwd run the grouped (MoE) kernels over M routed rows: M / top_k tokens routed
# uniformly at random to top_k of E experts of a stacked [E, N, K] record, with a
# LoRA pair per expert.  `python bench.py --sweep` runs the kernel sweep: forward
# and backward (LoRA rank 16, s = 2) of NF4-g128 weights N x K in {4096x4096,
# 1024x4096, 14336x4096, 4096x14336} at M in {1, 16, 256, 2048, 8192}, one JSON
# line each.  Each timing replays a CUDA graph of calls that rotate over C copies
# of the weights and activations, C chosen so the copies together exceed three
# L2s: every call reads cold weights from HBM, back to back as in a model step,
# and host launch overhead is excluded.  (Writing a 256 MB buffer between calls
# instead leaves dirty L2 lines whose write-back overlaps the next call; that
# added 1.5-4 us to a decode-step call.)
def _graph_us(fns, rounds=4):
    """Device time per call of a CUDA graph of `rounds` passes over fns."""
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(rounds):
            for fn in fns:
                fn()
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
    del g
    return best / (rounds * len(fns))


def probe_sweep(ms=(1, 16, 256, 2048, 8192), split=True):
    from spilltune_b200 import codec, ops
    dev = torch.device("cuda")
    r = 16
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    for (N, K) in [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)]:
        g = torch.Generator(device=dev).manual_seed(1)
        w0 = codec.encode(torch.randn(N, K, generator=g, device=dev) * 0.02, "nf4-g128")
        A = torch.randn(r, K, generator=g, device=dev) * 0.01
        B = torch.randn(N, r, generator=g, device=dev) * 0.01
        wbytes = N * K // 2 + 4 * N * K // 128
        for M in ms:
            footprint = wbytes + 4 * M * (N + K)  # weights, X, dY, Y, dX
            C = max(2, -(-3 * l2 // footprint))
            ws = [w0] + [codec.PackedWeight(w0.payload.clone(), w0.scales.clone(), w0.lut, w0.shape, w0.codec)
                         for _ in range(C - 1)]
            xs = [torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16) for _ in range(C)]
            dys = [torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16) for _ in range(C)]
            fs = [lambda x=x, w=w: ops.fwd(x, w, A, B, 2.0, split_reduction=split) for x, w in zip(xs, ws)]
            bs = [lambda x=x, w=w, dy=dy: ops.bwd(dy, x, w, A, B, 2.0, split_reduction=split)
                  for x, w, dy in zip(xs, ws, dys)]
            for f, b in zip(fs[:2], bs[:2]):
                f()
                b()
            torch.cuda.synchronize()
            rounds = max(1, 40 // C)
            tf, tb = _graph_us(fs, rounds), _graph_us(bs, rounds)
            fl_f = 2 * M * N * K + 2 * M * K * r + 2 * M * r * N
            fl_b = 2 * M * N * K + 4 * M * N * r + 6 * M * K * r
            print(json.dumps({"N": N, "K": K, "M": M, "copies": C, "fwd_us": round(tf, 1), "bwd_us": round(tb, 1),
                              "fwd_tflops": round(fl_f / tf / 1e6, 1), "bwd_tflops": round(fl_b / tb / 1e6, 1),
                              "fwd_weight_tbs": round(wbytes / tf / 1e6, 3),
                              "bwd_weight_tbs": round(wbytes / tb / 1e6, 3)}), flush=True)
            del ws, xs, dys, fs, bs
            torch.cuda.empty_cache()


def probe_op(a):
    from spilltune_b200 import codec, moe, ops
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
        ts = ops.fwd(x, w, A, B, 2.0, return_ts=True)[1] if a.ts and a.op == "bwd" and a.rank else None
        sp = not a.no_split
        fn = {
            "fwd": lambda: ops.fwd(x, w, A, B, 2.0, split_reduction=sp),
            "bwd": lambda: ops.bwd(dy, x, w, A, B, 2.0, ts=ts, split_reduction=sp),
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


# ---------------------------------------------------------------- Qwen3-30B-A3B MoE stack
MOE = {"layers": 48, "hidden": 2048, "q": 4096, "kv": 512, "experts": 128, "top_k": 8, "inter": 768, "rank": 8,
       "alpha": 16.0, "tokens": 8192}


def run_moe(args, world, rank, local):
    """The frozen-linear stack of a Qwen3-30B-A3B-shaped model (the MoE
    training configuration: 48 layers, hidden 2048, 32 x 128 query heads, 4 KV heads, 128
    experts top-8 with expert intermediate 768; NF4 group-128 records; LoRA
    rank 8 on the attention projections and per expert on gate_up / down;
    seq 4096 x micro-batch 2 = 8192 tokens per GPU).  Per layer: q/k/v fused
    (N = 4096 + 512 + 512), o, and the two grouped expert projections over
    the 65536 routed rows (fl_grouped_fwd / fl_grouped_bwd: expert
    gate_up [128, 1536, 2048], down [128, 2048, 768]); routing from random
    router weights (near-uniform load), sorted by expert on the device as
    moe.expert_segments does.  Step = forward, recomputed forward and backward
    of every call, then AdamW.  Inputs and upstream gradients are synthetic
    per-call buffers in two alternating sets (the router, gather, SiLU and
    combine are outside the frozen-linear stack, as attention is for the
    dense workload).  Weights resident in HBM (15.9 GB packed)."""
    from spilltune_b200 import build, codec, moe, ops, streaming
    build.build()
    dev = torch.device("cuda", local)
    c = MOE
    T, H, E, k, I, r = args.tokens, c["hidden"], c["experts"], c["top_k"], c["inter"], c["rank"]
    L = args.layers if args.layers != 32 else c["layers"]
    scale = c["alpha"] / r
    rows = T * k
    g = torch.Generator(device=dev).manual_seed(1234)

    def lora(n_experts, N, K, rk):
        shape_a = (n_experts, rk, K) if n_experts else (rk, K)
        shape_b = (n_experts, N, rk) if n_experts else (N, rk)
        A = (torch.randn(*shape_a, generator=g, device=dev) * 0.01).requires_grad_(True)
        B = (torch.randn(*shape_b, generator=g, device=dev) * 0.01).requires_grad_(True)
        A.grad, B.grad = torch.zeros_like(A), torch.zeros_like(B)
        return A, B

    layers = []
    for _ in range(L):
        attn = {n: codec.encode(torch.randn(N, K, generator=g, device=dev) * 0.02, args.codec)
                for n, N, K in (("q", c["q"], H), ("k", c["kv"], H), ("v", c["kv"], H), ("o", H, c["q"]))}
        buf, views = streaming.pack_layer(attn, dev)
        del attn
        qkv = ops.concat_records([views["q"], views["k"], views["v"]])
        gate_up = codec.encode(torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02, args.codec)
        down = codec.encode(torch.randn(E, H, I, generator=g, device=dev) * 0.02, args.codec)
        router = torch.randn(E, H, generator=g, device=dev) * 0.02
        logits = torch.randn(T, H, generator=g, device=dev) @ router.t()
        segs = moe.expert_segments(torch.topk(logits.softmax(-1), k, dim=-1)[1], E)
        A_qkv = (torch.randn(3 * r, H, generator=g, device=dev) * 0.01).requires_grad_(True)
        B_qkv = torch.zeros(c["q"] + 2 * c["kv"], 3 * r, device=dev)
        mask = torch.zeros_like(B_qkv)
        row = 0
        for i, N in enumerate((c["q"], c["kv"], c["kv"])):
            B_qkv[row:row + N, i * r:(i + 1) * r] = torch.randn(N, r, generator=g, device=dev) * 0.01
            mask[row:row + N, i * r:(i + 1) * r] = 1.0
            row += N
        B_qkv.requires_grad_(True)
        A_qkv.grad, B_qkv.grad = torch.zeros_like(A_qkv), torch.zeros_like(B_qkv)
        layers.append({"buf": buf, "qkv": qkv, "o": views["o"], "gate_up": gate_up, "down": down, "segs": segs,
                       "lora": {"qkv": (A_qkv, B_qkv), "o": lora(0, H, c["q"], r),
                                "gate_up": lora(E, 2 * I, H, r), "down": lora(E, H, I, r)},
                       "mask": mask})
    gi = torch.Generator(device=dev).manual_seed(100 + rank)
    rnd = lambda *shape: torch.randn(*shape, generator=gi, device=dev).to(torch.bfloat16)  # noqa: E731
    bufs = [{"attn": rnd(T, H), "o": rnd(T, c["q"]), "xs": rnd(rows, H), "act": rnd(rows, I),
             "d_qkv": rnd(T, c["q"] + 2 * c["kv"]), "d_o": rnd(T, H), "d_gu": rnd(rows, 2 * I), "d_dn": rnd(rows, H)}
            for _ in range(2)]
    params = [t for lay in layers for AB in lay["lora"].values() for t in AB]
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)
    counts = {"launches": 0}

    def step():
        for li, lay in enumerate(layers):
            b = bufs[li % 2]
            ops.fwd(b["attn"], lay["qkv"], *lay["lora"]["qkv"], scale)
            ops.fwd(b["o"], lay["o"], *lay["lora"]["o"], scale)
            moe.grouped_fwd(b["xs"], lay["segs"], lay["gate_up"], *lay["lora"]["gate_up"], scale)
            moe.grouped_fwd(b["act"], lay["segs"], lay["down"], *lay["lora"]["down"], scale)
        for li in reversed(range(len(layers))):
            lay, b = layers[li], bufs[li % 2]
            for name, x, d in (("down", b["act"], b["d_dn"]), ("gate_up", b["xs"], b["d_gu"])):
                A, B = lay["lora"][name]
                moe.grouped_fwd(x, lay["segs"], lay[name], A, B, scale)  # recompute
                moe.grouped_bwd(d, x, lay["segs"], lay[name], A, B, scale, dA=A.grad, dB=B.grad)
            for name, x, d in (("o", b["o"], b["d_o"]), ("qkv", b["attn"], b["d_qkv"])):
                A, B = lay["lora"][name]
                _y, ts = ops.fwd(x, lay[name], A, B, scale, return_ts=True)  # recompute
                ops.bwd(d, x, lay[name], A, B, scale, dA=A.grad, dB=B.grad, ts=ts)
            lay["lora"]["qkv"][1].grad.mul_(lay["mask"])
        opt.step()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    # Algorithmic work per token per layer: forward 2 x (attention weights + top_k expert weights),
    # backward (dX) the same, the recompute once more; LoRA terms are small and not counted here.
    w_tok = c["q"] * H + 2 * c["kv"] * H + H * c["q"] + k * (2 * I * H + H * I)
    step_flops = 3 * 2.0 * w_tok * T * L
    line = {"metric": "train tokens/s (Qwen3-30B-A3B NF4 LoRA frozen-linear stack)", "value": T / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"qwen3-30b-a3b frozen-linear stack: {L} layers x (q/k/v fused, o, grouped experts "
                                   "gate_up and down over 65536 routed rows), fwd + recompute + bwd + AdamW",
                       "layers": L, "tokens_per_gpu": T, "micro_batch": 2, "seq_len": 4096, "experts": E,
                       "top_k": k, "expert_inter": I, "rank": r, "alpha": c["alpha"], "codec": args.codec,
                       "parallelism": "dp1", "weights": "resident in HBM (no e2e streaming in this mode)"},
            "step_tflops": step_flops / (ms / 1e3) / 1e12, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


DSV3 = {"hidden": 7168, "heads": 128, "q_lora": 1536, "kv_lora": 512, "nope": 128, "rope": 64, "v_head": 128,
        "dense_inter": 18432, "dense_layers": 3, "moe_layers": 3, "experts": 256, "top_k": 8, "expert_inter": 2048,
        "groups": 8, "group_k": 4, "route_scale": 2.5, "rank": 16, "alpha": 32.0, "tokens": 4096}


def run_deepseek(args, world, rank, local):
    """The frozen-linear stack of DeepSeek-V3 truncated to 6 layers (3 dense with
    intermediate 18432, then 3 MoE with 256 routed experts top-8 of intermediate
    2048 plus one shared expert; hidden 7168; MLA attention with 128 heads,
    q_lora_rank 1536, kv_lora_rank 512, qk_nope 128, qk_rope 64, v_head 128;
    NF4 group-128 records; LoRA rank 16 on every projection, per expert for the
    routed ones; seq 4096 x micro-batch 1 = 4096 tokens per GPU).  Per layer:
    q_a_proj and kv_a_proj_with_mqa over the same input as one call (N = 1536 +
    576), q_b_proj (24576 x 1536), kv_b_proj (32768 x 512), o_proj (7168 x 16384);
    dense layers gate, up (18432 x 7168) and down (7168 x 18432); MoE layers the
    shared expert's gate/up as one call (4096 x 7168) and down (7168 x 2048), and
    the grouped routed experts gate_up [256, 4096, 7168] and down [256, 7168, 2048]
    over the 32768 routed rows, routed by DeepSeek-V3's group-limited sigmoid
    router (moe.deepseek_route) from random router weights.  Step = forward,
    recomputed forward and backward of every call, then AdamW.  The records hold
    random NF4 codes and scales (19 GB packed, resident in HBM): the kernels' work
    does not depend on the values, and encoding 11 B expert weights per layer from
    FP32 would need tens of GB of temporaries.  Inputs and upstream gradients are
    synthetic per-call buffers in two alternating sets; attention, norms, router,
    gather, SiLU and combine are outside the frozen-linear stack."""
    import math
    from spilltune_b200 import build, codec, moe, ops
    build.build()
    dev = torch.device("cuda", local)
    c = DSV3
    T = args.tokens if args.tokens != 8192 else c["tokens"]
    H, E, k, I, r = c["hidden"], c["experts"], c["top_k"], c["expert_inter"], c["rank"]
    qb_n = c["heads"] * (c["nope"] + c["rope"])
    kvb_n = c["heads"] * (c["nope"] + c["v_head"])
    o_k = c["heads"] * c["v_head"]
    kva_n = c["kv_lora"] + c["rope"]
    scale = c["alpha"] / r
    rows = T * k
    g = torch.Generator(device=dev).manual_seed(4321)
    lut = codec.NF4_LUT.to(dev)

    def record(*shape):
        groups = math.prod(shape) // 128
        payload = torch.randint(0, 256, (groups * 64,), generator=g, device=dev, dtype=torch.uint8)
        scales = torch.rand(groups, generator=g, device=dev) * 0.02 + 0.004
        return codec.PackedWeight(payload, scales, lut, shape, codec.NF4)

    def lora(n_experts, N, K, rk=r):
        shape_a = (n_experts, rk, K) if n_experts else (rk, K)
        shape_b = (n_experts, N, rk) if n_experts else (N, rk)
        A = (torch.randn(*shape_a, generator=g, device=dev) * 0.01).requires_grad_(True)
        B = (torch.randn(*shape_b, generator=g, device=dev) * 0.01).requires_grad_(True)
        A.grad, B.grad = torch.zeros_like(A), torch.zeros_like(B)
        return A, B

    layers = []
    for li in range(c["dense_layers"] + c["moe_layers"]):
        moe_layer = li >= c["dense_layers"]
        # q_a and kv_a as one call: A = [A_qa; A_kva], B block-diagonal (gradient masked).
        A_a = (torch.randn(2 * r, H, generator=g, device=dev) * 0.01).requires_grad_(True)
        B_a = torch.zeros(c["q_lora"] + kva_n, 2 * r, device=dev)
        mask = torch.zeros_like(B_a)
        B_a[:c["q_lora"], :r] = torch.randn(c["q_lora"], r, generator=g, device=dev) * 0.01
        B_a[c["q_lora"]:, r:] = torch.randn(kva_n, r, generator=g, device=dev) * 0.01
        mask[:c["q_lora"], :r] = 1.0
        mask[c["q_lora"]:, r:] = 1.0
        B_a.requires_grad_(True)
        A_a.grad, B_a.grad = torch.zeros_like(A_a), torch.zeros_like(B_a)
        lay = {"moe": moe_layer, "mask": mask,
               "w": {"a": record(c["q_lora"] + kva_n, H), "qb": record(qb_n, c["q_lora"]),
                     "kvb": record(kvb_n, c["kv_lora"]), "o": record(H, o_k)},
               "lora": {"a": (A_a, B_a), "qb": lora(0, qb_n, c["q_lora"]), "kvb": lora(0, kvb_n, c["kv_lora"]),
                        "o": lora(0, H, o_k)}}
        if moe_layer:
            lay["w"].update({"sgu": record(2 * I, H), "sdn": record(H, I)})
            lay["lora"].update({"sgu": lora(0, 2 * I, H), "sdn": lora(0, H, I)})
            lay["gate_up"], lay["down"] = record(E, 2 * I, H), record(E, H, I)
            lay["lora"].update({"gate_up": lora(E, 2 * I, H), "down": lora(E, H, I)})
            router = torch.randn(E, H, generator=g, device=dev) * 0.02
            bias = torch.randn(E, generator=g, device=dev) * 0.01
            _w, idx = moe.deepseek_route(torch.randn(T, H, generator=g, device=dev), router, bias, groups=c["groups"],
                                         group_k=c["group_k"], top_k=k, normalize=True, scale=c["route_scale"])
            lay["segs"] = moe.expert_segments(idx, E)
        else:
            DI = c["dense_inter"]
            lay["w"].update({"gate": record(DI, H), "up": record(DI, H), "down_d": record(H, DI)})
            lay["lora"].update({"gate": lora(0, DI, H), "up": lora(0, DI, H), "down_d": lora(0, H, DI)})
        layers.append(lay)
    gi = torch.Generator(device=dev).manual_seed(100 + rank)
    rnd = lambda *shape: torch.randn(*shape, generator=gi, device=dev).to(torch.bfloat16)  # noqa: E731
    # Inputs of each dense call (name -> [T, K]) and their upstream gradients ([T, N]).
    dense_in = {"a": H, "qb": c["q_lora"], "kvb": c["kv_lora"], "o": o_k, "gate": H, "up": H,
                "down_d": c["dense_inter"], "sgu": H, "sdn": I}
    dense_out = {"a": c["q_lora"] + kva_n, "qb": qb_n, "kvb": kvb_n, "o": H, "gate": c["dense_inter"],
                 "up": c["dense_inter"], "down_d": H, "sgu": 2 * I, "sdn": H}
    bufs = []
    for _ in range(2):
        b = {("x", n): rnd(T, K) for n, K in dense_in.items()}
        b.update({("d", n): rnd(T, N) for n, N in dense_out.items()})
        b.update({"xs": rnd(rows, H), "act": rnd(rows, I), "d_gu": rnd(rows, 2 * I), "d_dn": rnd(rows, H)})
        bufs.append(b)
    params = [t for lay in layers for AB in lay["lora"].values() for t in AB]
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)

    def names(lay):
        return ["a", "qb", "kvb", "o"] + (["sgu", "sdn"] if lay["moe"] else ["gate", "up", "down_d"])

    def step():
        for li, lay in enumerate(layers):
            b = bufs[li % 2]
            for n in names(lay):
                ops.fwd(b[("x", n)], lay["w"][n], *lay["lora"][n], scale)
            if lay["moe"]:
                moe.grouped_fwd(b["xs"], lay["segs"], lay["gate_up"], *lay["lora"]["gate_up"], scale)
                moe.grouped_fwd(b["act"], lay["segs"], lay["down"], *lay["lora"]["down"], scale)
        for li in reversed(range(len(layers))):
            lay, b = layers[li], bufs[li % 2]
            if lay["moe"]:
                for name, x, d in (("down", b["act"], b["d_dn"]), ("gate_up", b["xs"], b["d_gu"])):
                    A, B = lay["lora"][name]
                    moe.grouped_fwd(x, lay["segs"], lay[name], A, B, scale)  # recompute
                    moe.grouped_bwd(d, x, lay["segs"], lay[name], A, B, scale, dA=A.grad, dB=B.grad)
            for n in reversed(names(lay)):
                A, B = lay["lora"][n]
                x = b[("x", n)]
                _y, ts = ops.fwd(x, lay["w"][n], A, B, scale, return_ts=True)  # recompute
                ops.bwd(b[("d", n)], x, lay["w"][n], A, B, scale, dA=A.grad, dB=B.grad, ts=ts)
            lay["lora"]["a"][1].grad.mul_(lay["mask"])
        opt.step()

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        torch.cuda.nvtx.range_push("timed_step")
        for _ in range(args.steps):
            step()
        torch.cuda.nvtx.range_pop()
        t1.record()
        torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / args.steps
    # Weights each token passes per layer (LoRA terms are small and not counted): forward,
    # recompute and backward (dX) each 2 FLOPs per weight per token.
    attn = (c["q_lora"] + kva_n) * H + qb_n * c["q_lora"] + kvb_n * c["kv_lora"] + H * o_k
    w_dense = attn + 3 * c["dense_inter"] * H
    w_moe = attn + 3 * I * H + k * 3 * I * H
    step_flops = 3 * 2.0 * T * (c["dense_layers"] * w_dense + c["moe_layers"] * w_moe)
    packed = sum(w.payload.numel() + 4 * w.scales.numel() for lay in layers
                 for w in list(lay["w"].values()) + ([lay["gate_up"], lay["down"]] if lay["moe"] else []))
    line = {"metric": "train tokens/s (DeepSeek-V3-6L NF4 LoRA frozen-linear stack)", "value": T / (ms / 1e3),
            "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "deepseek-v3-6l frozen-linear stack: 3 dense + 3 MoE layers x (q_a/kv_a fused, "
                                   "q_b, kv_b, o; dense gate, up, down | shared gate_up, down + grouped routed experts "
                                   f"gate_up and down over {rows} routed rows), fwd + recompute + bwd + AdamW",
                       "layers": len(layers), "tokens_per_gpu": T, "micro_batch": 1, "seq_len": 4096, "experts": E,
                       "top_k": k, "expert_inter": I, "rank": r, "alpha": c["alpha"], "codec": "nf4-g128",
                       "parallelism": "dp1", "packed_gb": round(packed / 1e9, 2),
                       "weights": "random NF4 codes and scales, resident in HBM (no e2e streaming in this mode)"},
            "step_tflops": step_flops / (ms / 1e3) / 1e12, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- main
def main():
    args = parse()
    if args.workload in ("qwen3-30b-a3b", "deepseek-v3-6l"):
        world, rank, local = init_dist()
        if world > 1:
            raise SystemExit(f"the {args.workload} workload runs on one GPU")
        return (run_moe if args.workload == "qwen3-30b-a3b" else run_deepseek)(args, world, rank, local)
    if args.op or args.sweep:
        from spilltune_b200 import build
        build.build()
        if args.sweep:
            probe_sweep(tuple(int(m) for m in args.sweep_m.split(",")), split=not args.no_split)
        else:
            probe_op(args)
        return 0
    world, rank, local = init_dist()
    if args.impl == "reference":
        rc = run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return rc
    from spilltune_b200 import build
    from spilltune_b200.streaming import PackedSlotSession
    build.build()
    dev = torch.device("cuda", local)
    M, L = args.tokens, args.layers
    layer_bufs, weights, loras = build_model(L, args.codec, dev, seed=1234)  # same weights on every rank
    bufs = make_buffers(M, dev, seed=100 + rank)                             # rank-local micro-batch
    params = [t for ll in loras for gname, *_ in GROUPS for t in ll[gname].params()]
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)

    @contextlib.contextmanager
    def resident(l, phase):
        yield weights[l]

    step = Step(resident, loras, bufs, world, opt)
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    step.record = True
    step.events.clear()
    step.launches = 0
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        barrier(world)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("timed_step")
        t0.record()
        for _ in range(args.steps):
            step()
        t1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, world)
    launches = step.launches
    kern_ms = statistics.mean(s.elapsed_time(e) for s, e in step.events)
    step.record = False

    # ------------------------------------------------------------ e2e
    e2e = None
    if not args.no_e2e:
        host_layers = [{k: w.to("cpu").pin_memory() for k, w in lw.items()} for lw in weights]
        for lw in weights:
            lw.clear()
        layer_bufs.clear()
        torch.cuda.empty_cache()
        # N > 1: each rank copies its 1/N of every layer from the host and the
        # slot is all-gathered over NVLink on a communicator of its own.
        wgroup = None
        if world > 1:
            import torch.distributed as dist
            wgroup = dist.new_group(backend="nccl")
        sess = PackedSlotSession(host_layers, dev, slots=2, group=wgroup)
        if wgroup is not None:
            host_layers = None  # the session keeps this rank's shards only
        # The host link the slot copies run over: a plain pinned-host -> device copy
        # of one layer image and of 1 GiB, alone on a stream (outside the timed region).
        link = {"layer_image": host_link_gbs(dev, sess.capacity), "1GiB": host_link_gbs(dev, 1 << 30)}
        x0_host = torch.randn(M, HIDDEN, dtype=torch.float32).to(torch.bfloat16).pin_memory()
        norm_host = torch.empty(1, dtype=torch.float32).pin_memory()
        estep = Step(sess.borrow, loras, bufs, world, opt)

        def e2e_step():
            bufs[0][0]["attn"].copy_(x0_host, non_blocking=True)
            estep()
            gn = torch.stack([t.grad.norm() for t in params[:14]]).norm()
            norm_host.copy_(gn.view(1), non_blocking=True)

        for _ in range(max(3, args.warmup)):
            e2e_step()
        torch.cuda.synchronize()
        sess.reset_stats()
        barrier(world)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(args.steps):
            e2e_step()
        t1.record()
        torch.cuda.synchronize()
        barrier(world)
        ems = max_over_ranks(t0.elapsed_time(t1) / args.steps, world)
        h2d = sess.h2d_bytes / args.steps + x0_host.numel() * 2
        copy_s = sess.h2d_seconds()
        e2e = {"value": world * M / (ems / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": int(h2d),
               "d2h_bytes_per_step": 4, "ms_per_step": ems,
               "slot_h2d_gbs": (sess.h2d_bytes / copy_s / 1e9) if copy_s > 0 else None,
               "host_link_gbs": link,
               "weights": "pinned host, 2 VRAM slots, one-layer prefetch (fwd + bwd reload)"}
        if wgroup is not None:
            e2e["weights"] = (f"pinned host, 1/{world} of each layer per rank, copied into 2 VRAM slots and "
                              "all-gathered over NVLink (NCCL, own communicator), one-layer prefetch")
            e2e["nvlink_gather_bytes_per_step"] = int(sess.h2d_bytes * (world - 1) / args.steps)
        sess.close()

    # ------------------------------------------------------------ report
    if rank == 0:
        peak, hbm, peak_kind = measured_peaks()
        # Algorithmic work of the dominant call (gate_proj, rank 16).
        fl = sum(algorithmic_fwd_flops(M, SHAPE[m][0], SHAPE[m][1], RANK)
                 for m in dict((g[0], g[1]) for g in GROUPS)[DOMINANT_GROUP])
        achieved = fl / (kern_ms / 1e3) / 1e12
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = reference_cpu_sample(args.tokens, args.codec, args.cpu_passes)
            cpu.pop("layer_seconds", None)
        total_flops = step_flops(M, L)
        line = {
            "metric": "train tokens/s (8B NF4 LoRA frozen-linear stack)",
            "value": world * M / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": bench_config(args, world),
            "step_tflops": total_flops / (ms / 1e3) / 1e12,
            "roofline": {"bound": "tensor",
                         "kernel": "fl_fwd (fused dequant-GEMM + LoRA) gate_proj 8192x14336x4096, rank 16",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                         "peak_kind": f"{peak_kind} bf16 sustained", "traffic": load_profile_traffic(),
                         "launch_ms": kern_ms},
            "clocks": clk.summary(),
            "gpu_launches": launches,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
