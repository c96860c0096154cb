"""Per-expert loop oracle for the MoE expert layers — TEST INFRASTRUCTURE ONLY.

A restatement of the reference's expert loop over decoded BF16 expert
matrices, used to check the grouped kernels.  Only ``tests/`` import it.

* ``qwen3_moe_loop`` follows ``moe_feed_forward``
  (ram_vram_finetune/adapters/qwen3_moe.py:95-113) op for op: router linear,
  FP32 softmax, top-k, optional renormalisation, cast to the logits' dtype,
  then for every expert hit (ascending expert id) gather, gate_up linear,
  chunk, silu(gate) * up, down linear, multiply by the routing weight and a
  BF16 ``index_add_`` into the output.  Pinned against the reference's own
  output in ``tests/golden/moe_small.npz``.
* ``grouped_linear_fp32`` is the FP32 reference of one grouped projection:
  for each expert segment, x . W_e^T + s (x . A_e^T) . B_e^T, with its
  gradients, used for the per-expert LoRA cases (the reference's experts
  carry no LoRA).
"""
import torch
import torch.nn.functional as F


def qwen3_moe_loop(hidden, gate_weight, gate_up, down, *, num_experts, top_k, norm_topk_prob):
    """`gate_up` [E, 2I, H] and `down` [E, H, I] are decoded BF16 tensors."""
    shape = hidden.shape
    flat = hidden.view(-1, shape[-1])
    logits = F.linear(flat, gate_weight)
    probs = F.softmax(logits, dtype=torch.float32, dim=-1)
    routing, chosen = torch.topk(probs, top_k, dim=-1)
    if norm_topk_prob:
        routing /= routing.sum(dim=-1, keepdim=True)
    routing = routing.to(logits.dtype)
    out = torch.zeros_like(flat)
    with torch.no_grad():
        hits = F.one_hot(chosen, num_classes=num_experts).permute(2, 1, 0)
        active = (hits.sum(dim=(-1, -2)) > 0).nonzero()
    for row in active:
        e = row[0]
        slot, tok = torch.where(hits[e])
        rows = flat[tok]
        g, u = F.linear(rows, gate_up[e]).chunk(2, dim=-1)
        val = F.linear(F.silu(g) * u, down[e])
        val = val * routing[tok, slot, None]
        out.index_add_(0, tok, val.to(out.dtype))
    return out.reshape(shape)


def grouped_linear_fp32(xs, seg, W, A=None, B=None, scale=0.0):
    """FP32 y for expert-sorted rows xs [rows, K]; W [E, N, K] decoded weights
    (any float dtype), A [E, r, K], B [E, N, r]; seg a host list of E+1 offsets."""
    E = W.shape[0]
    out = torch.empty(xs.shape[0], W.shape[1], dtype=torch.float32, device=xs.device)
    for e in range(E):
        a, b = seg[e], seg[e + 1]
        x = xs[a:b].float()
        y = x @ W[e].float().t()
        if A is not None:
            y = y + scale * ((x @ A[e].float().t()) @ B[e].float().t())
        out[a:b] = y
    return out


def grouped_linear_grads_fp32(dy, xs, seg, W, A=None, B=None, scale=0.0):
    """FP32 (dX, dA, dB) of grouped_linear_fp32 (dA/dB None without LoRA)."""
    E = W.shape[0]
    dx = torch.empty(xs.shape[0], W.shape[2], dtype=torch.float32, device=xs.device)
    dA = torch.zeros_like(A, dtype=torch.float32) if A is not None else None
    dB = torch.zeros_like(B, dtype=torch.float32) if B is not None else None
    for e in range(E):
        a, b = seg[e], seg[e + 1]
        g = dy[a:b].float()
        x = xs[a:b].float()
        d = g @ W[e].float()
        if A is not None:
            u = scale * (g @ B[e].float())          # [m, r]
            d = d + u @ A[e].float()
            dA[e] = u.t() @ x
            dB[e] = scale * (g.t() @ (x @ A[e].float().t()))
        dx[a:b] = d
    return dx, dA, dB
