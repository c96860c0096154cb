"""MoE expert layers over stacked packed expert records (grouped kernels).

The reference runs routed experts as a Python loop of small GEMMs over
decoded BF16 expert weights:

* Qwen3-MoE ``moe_feed_forward`` (ram_vram_finetune/adapters/qwen3_moe.py:95-113):
  softmax router, top-k, optional renormalisation, then per hit expert
  ``gather -> F.linear(gate_up[e]) -> silu(gate) * up -> F.linear(down[e])
  -> * routing weight -> index_add_``;
* DeepSeek-V3 (adapters/deepseek.py:115-126 router, :159-177 expert loop):
  sigmoid scores with a selection bias and group-limited top-k.

Here the routed (token, slot) rows are sorted by expert once on the device
(``expert_segments``), and each projection over ALL experts is one grouped
call (``fl_grouped_fwd`` / ``fl_grouped_bwd``: a tile list over the expert
segments, the 4-bit decode fused into the tcgen05 GEMM as for dense
projections), with an optional per-expert LoRA branch whose FP32 gradients
are summed over each expert's rows.  No host synchronisation: segment offsets
stay on the device.  The combine sums each token's k expert outputs in FP32
(one rounding to BF16) instead of k sequential BF16 ``index_add_`` steps.
"""
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _lib
from .codec import PackedWeight
from .ops import _need_cuda, _ptr, _stream


# ------------------------------------------------------------------ routing
def qwen3_route(flat, gate_weight, top_k, norm_topk_prob):
    """Router of qwen3_moe.py:97-101: FP32 softmax of the router logits, top-k,
    optional renormalisation, weights cast back to the logits' dtype."""
    logits = F.linear(flat, gate_weight)
    probs = F.softmax(logits, dtype=torch.float32, dim=-1)
    weights, indices = torch.topk(probs, top_k, dim=-1)
    if norm_topk_prob:
        weights = weights / weights.sum(dim=-1, keepdim=True)
    return weights.to(logits.dtype), indices


def deepseek_route(flat, weight, bias, *, groups, group_k, top_k, normalize, scale):
    """Router of deepseek.py:115-126: FP32 sigmoid scores; the correction bias
    steers selection only; experts are chosen inside the `group_k` groups
    with the best top-2 sums; weights optionally renormalised, then scaled."""
    logits = F.linear(flat.float(), weight.float())
    scores = logits.sigmoid()
    choice = scores + bias.float()
    E = choice.shape[-1]
    per_group = choice.view(-1, groups, E // groups)
    group_score = per_group.topk(2, dim=-1)[0].sum(-1)
    keep_groups = group_score.topk(group_k, dim=-1, sorted=False)[1]
    keep = torch.zeros_like(group_score).scatter_(1, keep_groups, 1).bool()
    keep = keep[:, :, None].expand(-1, groups, E // groups).reshape_as(choice)
    indices = choice.masked_fill(~keep, float("-inf")).topk(top_k, dim=-1, sorted=False)[1]
    weights = scores.gather(1, indices)
    if normalize:
        weights = weights / (weights.sum(-1, keepdim=True) + 1e-20)
    return weights * scale, indices


# ----------------------------------------------------------------- segments
@dataclass
class ExpertSegments:
    """Routed rows sorted by expert.

    Row p of the sorted order is routed pair ``order[p]`` = token * top_k +
    slot; ``token[p]`` its token; ``seg`` (int32 [E+1]) the prefix offsets of
    the experts' segments; ``inverse[q]`` the sorted row of pair q.
    """
    order: torch.Tensor
    token: torch.Tensor
    inverse: torch.Tensor
    seg: torch.Tensor
    experts: int
    top_k: int

    @property
    def rows(self):
        return self.order.numel()


def expert_segments(indices, experts):
    """Sort the routed (token, slot) pairs of `indices` [T, top_k] by expert
    (stable, so tokens stay in order inside an expert, as the reference's
    ``torch.where(mask[expert])`` visits them)."""
    T, k = indices.shape
    flat_e = indices.reshape(-1)
    order = torch.argsort(flat_e, stable=True)
    # scatter_add, not bincount: bincount reads the maximum back to the host.
    counts = torch.zeros(experts, dtype=torch.int64, device=indices.device)
    counts.scatter_add_(0, flat_e, torch.ones_like(flat_e))
    seg = torch.zeros(experts + 1, dtype=torch.int32, device=indices.device)
    seg[1:] = torch.cumsum(counts, 0).to(torch.int32)
    inverse = torch.empty_like(order)
    inverse[order] = torch.arange(order.numel(), device=order.device)
    return ExpertSegments(order, order // k, inverse, seg, experts, k)


class _GatherRows(torch.autograd.Function):
    """xs = flat[token]; the backward sums each token's top_k row gradients in
    FP32 through the inverse permutation (deterministic, no atomics)."""

    @staticmethod
    def forward(ctx, flat, segs: ExpertSegments):
        ctx.segs = segs
        ctx.dtype = flat.dtype
        return flat.index_select(0, segs.token)

    @staticmethod
    def backward(ctx, g):
        s = ctx.segs
        T = s.rows // s.top_k
        per_pair = g.index_select(0, s.inverse).view(T, s.top_k, -1)
        return per_pair.float().sum(1).to(ctx.dtype), None


def gather_rows(flat, segs):
    return _GatherRows.apply(flat, segs)


def combine_rows(values, weights, segs, out_dtype):
    """out[t] = sum_slot values[row of (t, slot)] * weights[t, slot]: the
    reference's ``value * routing`` + ``index_add_`` (qwen3_moe.py:110-111),
    summed in FP32 and rounded once."""
    T = segs.rows // segs.top_k
    w_sorted = weights.reshape(-1).index_select(0, segs.order)
    weighted = (values * w_sorted[:, None]).to(out_dtype)
    per_pair = weighted.index_select(0, segs.inverse).view(T, segs.top_k, -1)
    return per_pair.float().sum(1).to(out_dtype)


# ------------------------------------------------------------ grouped calls
def _stacked_shape(weight: PackedWeight):
    if len(weight.shape) != 3:
        raise ValueError("grouped ops need a stacked expert record [E, N, K]")
    return weight.shape


def _check_lora(A, B, E, N, K):
    rank = 0 if A is None else A.shape[-2]
    if rank:
        if A.dtype != torch.float32 or B is None or B.dtype != torch.float32 \
                or tuple(A.shape) != (E, rank, K) or tuple(B.shape) != (E, N, rank):
            raise ValueError("per-expert LoRA factors must be fp32 A[E, rank, K] and B[E, N, rank]")
    return rank


def _check_segs(x2, segs: ExpertSegments, E):
    if segs.experts != E:
        raise ValueError(f"segments cover {segs.experts} experts, record holds {E}")
    if x2.shape[0] != segs.rows:
        raise ValueError(f"expected {segs.rows} expert-sorted rows, got {x2.shape[0]}")
    if segs.seg.dtype != torch.int32 or not segs.seg.is_contiguous():
        raise ValueError("segment offsets must be a contiguous int32 tensor")


def _workspace(rows, E, N, K, rank, device):
    n = _lib.load().fl_grouped_workspace_bytes(rows, E, N, K, rank)
    return torch.empty(n, dtype=torch.uint8, device=device), n


def grouped_fwd(xs, segs: ExpertSegments, weight: PackedWeight, A=None, B=None, scale=0.0):
    """Y[rows, N] for expert-sorted rows xs [rows, K]: row p of segment e gets
    xs[p] . W_e^T + scale * (xs[p] . A_e^T) . B_e^T."""
    E, N, K = _stacked_shape(weight)
    if xs.dtype != torch.bfloat16 or xs.dim() != 2 or xs.shape[1] != K:
        raise ValueError(f"expert rows must be bf16 [rows, {K}]")
    xs = xs.contiguous()
    rank = _check_lora(A, B, E, N, K)
    _need_cuda(xs, segs.seg, weight.payload, A, B)
    _check_segs(xs, segs, E)
    if rank:
        A = A.detach().contiguous()
        B = B.detach().contiguous()
    rows = xs.shape[0]
    y = torch.empty((rows, N), dtype=torch.bfloat16, device=xs.device)
    if rows:
        ws, n = _workspace(rows, E, N, K, rank, xs.device)
        _lib.call("fl_grouped_fwd", _ptr(xs), _ptr(segs.seg), rows, K, E, _ptr(weight.payload),
                  _ptr(weight.scales), _ptr(weight.lut), N, _ptr(A), _ptr(B), rank, float(scale), _ptr(y),
                  _ptr(ws), n, _stream())
    return y


def grouped_bwd(dy, xs, segs: ExpertSegments, weight: PackedWeight, A=None, B=None, scale=0.0, dA=None, dB=None,
                accumulate=False):
    """(dX [rows, K] bf16, dA [E, rank, K] fp32, dB [E, N, rank] fp32) of grouped_fwd."""
    E, N, K = _stacked_shape(weight)
    if dy.dtype != torch.bfloat16 or dy.dim() != 2 or dy.shape[1] != N:
        raise ValueError(f"output gradient must be bf16 [rows, {N}]")
    dy = dy.contiguous()
    rank = _check_lora(A, B, E, N, K)
    _need_cuda(dy, segs.seg, weight.payload, A, B)
    _check_segs(dy, segs, E)
    rows = dy.shape[0]
    dx = torch.empty((rows, K), dtype=torch.bfloat16, device=dy.device)
    if rank:
        if xs is None or xs.dtype != torch.bfloat16 or tuple(xs.shape) != (rows, K):
            raise ValueError(f"expert rows must be bf16 [{rows}, {K}]")
        xs = xs.contiguous()
        A = A.detach().contiguous()
        B = B.detach().contiguous()
        if dA is None:
            dA = torch.empty((E, rank, K), dtype=torch.float32, device=dy.device)
            accumulate = False
        if dB is None:
            dB = torch.empty((E, N, rank), dtype=torch.float32, device=dy.device)
            accumulate = False
    if rows:
        ws, n = _workspace(rows, E, N, K, rank, dy.device)
        _lib.call("fl_grouped_bwd", _ptr(dy), _ptr(xs) if rank else None, _ptr(segs.seg), rows, N, K, E,
                  _ptr(weight.payload), _ptr(weight.scales), _ptr(weight.lut), _ptr(A), _ptr(B), rank,
                  float(scale), _ptr(dx), _ptr(dA), _ptr(dB), int(bool(accumulate)), _ptr(ws), n, _stream())
    elif rank and not accumulate:
        dA.zero_()
        dB.zero_()
    return dx, dA, dB


def grouped_frozen_lora_linear(xs, segs, weight: PackedWeight, A=None, B=None, scale=0.0):
    """Autograd-capable grouped projection of expert-sorted rows (experts frozen,
    A/B trainable), through the ``spilltune_b200::grouped_frozen_lora_linear``
    custom op (``spilltune_b200.library``)."""
    from . import library  # noqa: F401  (registers the ops)
    E, N, K = _stacked_shape(weight)
    if xs.dtype != torch.bfloat16 or xs.dim() != 2 or xs.shape[1] != K:
        raise ValueError(f"expert rows must be bf16 [rows, {K}]")
    _check_lora(A, B, E, N, K)
    _need_cuda(xs, segs.seg, weight.payload, A, B)
    _check_segs(xs, segs, E)
    return torch.ops.spilltune_b200.grouped_frozen_lora_linear(xs, segs.seg, weight.payload, weight.scales,
                                                               weight.lut, E, N, A, B, float(scale))


# ------------------------------------------------------------ expert layers
def _lora(lora, name):
    if not lora or name not in lora:
        return None, None, 0.0
    A, B, s = lora[name]
    return A, B, s


def routed_experts(flat, weights, indices, gate_up: PackedWeight, down: PackedWeight, lora=None):
    """The routed-expert part shared by Qwen3-MoE and DeepSeek-V3: gather,
    gate_up projection, silu(gate) * up, down projection, weighted combine.

    `gate_up` is the stacked [E, 2I, H] record, `down` [E, H, I]; `lora`
    optionally maps "gate_up" / "down" to (A [E, r, K], B [E, N, r], scale).
    """
    E = gate_up.experts
    if down.experts != E or gate_up.in_features != flat.shape[-1] or down.out_features != flat.shape[-1] \
            or gate_up.out_features != 2 * down.in_features:
        raise ValueError("expert record shapes do not match gate_up [E, 2I, H] / down [E, H, I]")
    segs = expert_segments(indices, E)
    xs = gather_rows(flat, segs)
    A1, B1, s1 = _lora(lora, "gate_up")
    h = grouped_frozen_lora_linear(xs, segs, gate_up, A1, B1, s1)
    gate, up = h.chunk(2, dim=-1)
    act = (F.silu(gate) * up).contiguous()
    A2, B2, s2 = _lora(lora, "down")
    v = grouped_frozen_lora_linear(act, segs, down, A2, B2, s2)
    return combine_rows(v, weights, segs, flat.dtype)


def moe_feed_forward(hidden, weights, *, num_experts, top_k, norm_topk_prob, lora=None):
    """Drop-in for qwen3_moe.moe_feed_forward (qwen3_moe.py:95-113) with the
    expert weights as stacked packed records: ``weights['mlp.gate.weight']``
    (BF16 router), ``weights['mlp.experts.gate_up_proj']`` and
    ``weights['mlp.experts.down_proj']`` (PackedWeight [E, 2I, H] / [E, H, I])."""
    shape = hidden.shape
    flat = hidden.reshape(-1, shape[-1])
    gate_up = weights["mlp.experts.gate_up_proj"]
    if gate_up.experts != num_experts:
        raise ValueError(f"expected {num_experts} experts, record holds {gate_up.experts}")
    routing, indices = qwen3_route(flat, weights["mlp.gate.weight"], top_k, norm_topk_prob)
    out = routed_experts(flat, routing, indices, gate_up, weights["mlp.experts.down_proj"], lora)
    return out.reshape(shape)


def deepseek_routed_experts(flat, weights, *, groups, group_k, top_k, normalize, scale, lora=None):
    """DeepSeek-V3 routed experts (deepseek.py:159-177 with packed experts):
    returns the routed sum for each row of `flat`; the shared expert is a
    dense frozen MLP added by the caller."""
    routing, indices = deepseek_route(flat, weights["mlp.gate.weight"], weights["mlp.gate.e_score_correction_bias"],
                                      groups=groups, group_k=group_k, top_k=top_k, normalize=normalize, scale=scale)
    return routed_experts(flat, routing, indices, weights["mlp.experts.gate_up_proj"],
                          weights["mlp.experts.down_proj"], lora)
