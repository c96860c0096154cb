"""``torch.library`` custom ops of the fused frozen projections.

The C ABI (include/spilltune_b200.h) is the boundary; these ops are its thin
PyTorch face, with a schema, a fake (meta) implementation for tracing and an
autograd formula, so the fused path composes with ``torch.autograd`` the way
the reference's ``F.linear`` calls do (finetune/lora.py:205-220 forward,
training/recompute.py:102-127 backward):

* ``spilltune_b200::frozen_lora_linear(x, payload, scales, lut, out_features,
  layout, A?, B?, scale) -> (Y, Ts)``: x bf16 [M, K]; Y bf16 [M, N]; Ts the
  [M, 64] bf16 low-rank activations bf16(scale * x . A^T) the backward reuses
  (zeros where the decode-step kernels form them inside the backward; [0, 64]
  without LoRA).  layout 0 = group-128 record (payload, scales, codebook),
  layout 1 = bitsandbytes NF4-DQ64 (packed, FP32 block scales, quant map).
* ``spilltune_b200::frozen_lora_linear_backward(dy, x, payload, scales, lut,
  layout, A?, B?, scale, Ts) -> (dX, dA, dB)`` (dA/dB empty without LoRA).
* ``spilltune_b200::grouped_frozen_lora_linear(xs, seg, payload, scales, lut,
  experts, out_features, A?, B?, scale) -> Y`` over expert-sorted rows with
  prefix offsets ``seg`` (int32 [E + 1]), and its ``..._backward``.

The weight parts and the segment offsets get no gradient (frozen base, as
``recompute.py:168-169`` requires).  Every op runs on the current CUDA stream;
CPU tensors raise (no CPU fallback).
"""
from typing import Optional, Tuple

import torch
from torch import Tensor

from . import _lib
from .ops import _need_cuda, _ptr, _stream, keeps_ts, launch_bwd, launch_fwd, ts_view

_NS = "spilltune_b200"


# ------------------------------------------------------------------ dense
@torch.library.custom_op(f"{_NS}::frozen_lora_linear", mutates_args=(), device_types="cuda")
def _frozen_fwd(x: Tensor, payload: Tensor, scales: Tensor, lut: Tensor, out_features: int, layout: int,
                A: Optional[Tensor], B: Optional[Tensor], scale: float) -> Tuple[Tensor, Tensor]:
    x = x.contiguous()
    M, K = x.shape
    rank = 0 if A is None else A.shape[0]
    y, ws = launch_fwd(layout, x, payload, scales, lut, out_features, A, B, scale)
    if keeps_ts(layout, M, K, rank):
        ts = ts_view(ws, M)
    elif rank:
        ts = torch.zeros((M, 64), dtype=torch.bfloat16, device=x.device)
    else:
        ts = torch.empty((0, 64), dtype=torch.bfloat16, device=x.device)
    return y, ts


@_frozen_fwd.register_fake
def _(x, payload, scales, lut, out_features, layout, A, B, scale):
    M = x.shape[0]
    y = x.new_empty((M, out_features))
    ts = x.new_empty((M, 64)) if A is not None else x.new_empty((0, 64))
    return y, ts


@torch.library.custom_op(f"{_NS}::frozen_lora_linear_backward", mutates_args=(), device_types="cuda")
def _frozen_bwd(dy: Tensor, x: Tensor, payload: Tensor, scales: Tensor, lut: Tensor, layout: int,
                A: Optional[Tensor], B: Optional[Tensor], scale: float, ts: Tensor) -> Tuple[Tensor, Tensor, Tensor]:
    dy = dy.contiguous()
    x = x.contiguous()
    K = x.shape[1]
    rank = 0 if A is None else A.shape[0]
    M = dy.shape[0]
    dx, dA, dB = launch_bwd(layout, dy, x if rank else None, payload, scales, lut, K, A, B, scale,
                            ts=ts.contiguous() if keeps_ts(layout, M, K, rank) else None)
    if not rank:
        dA = torch.empty((0,), dtype=torch.float32, device=dy.device)
        dB = torch.empty((0,), dtype=torch.float32, device=dy.device)
    return dx, dA, dB


@_frozen_bwd.register_fake
def _(dy, x, payload, scales, lut, layout, A, B, scale, ts):
    dx = x.new_empty(x.shape)
    if A is None:
        return dx, dy.new_empty((0,), dtype=torch.float32), dy.new_empty((0,), dtype=torch.float32)
    return dx, A.new_empty(A.shape), B.new_empty(B.shape)


def _frozen_setup(ctx, inputs, output):
    x, payload, scales, lut, out_features, layout, A, B, scale = inputs
    _, ts = output
    ctx.layout, ctx.scale, ctx.has_lora = layout, scale, A is not None
    # Ts goes through save_for_backward like every other saved tensor, so an
    # in-place change of A (or of Ts) before the backward is caught by
    # autograd's version check instead of silently using stale activations.
    ctx.save_for_backward(x, payload, scales, lut, A, B, ts)


def _frozen_backward(ctx, dy, _dts):
    x, payload, scales, lut, A, B, ts = ctx.saved_tensors
    dx, dA, dB = torch.ops.spilltune_b200.frozen_lora_linear_backward(dy, x, payload, scales, lut, ctx.layout, A, B,
                                                                      ctx.scale, ts)
    if not ctx.has_lora:
        dA = dB = None
    return dx, None, None, None, None, None, dA, dB, None


_frozen_fwd.register_autograd(_frozen_backward, setup_context=_frozen_setup)


def frozen_linear(x, payload, scales, lut, out_features, in_features, layout=0, A=None, B=None, scale=0.0):
    """x [..., K] bf16 -> Y [..., N] through the custom op (autograd in x, A, B)."""
    if x.shape[-1] != in_features:
        raise ValueError(f"input width mismatch: expected {in_features}, got {x.shape[-1]}")
    if x.dtype != torch.bfloat16:
        raise ValueError("activations must be bf16")
    _need_cuda(x, payload, A, B)
    rank = 0 if A is None else A.shape[0]
    if rank and (B is None or tuple(A.shape) != (rank, in_features) or tuple(B.shape) != (out_features, rank)
                 or A.dtype != torch.float32 or B.dtype != torch.float32):
        raise ValueError("LoRA factors must be fp32 A[rank, K] and B[N, rank]")
    y, _ = torch.ops.spilltune_b200.frozen_lora_linear(x.reshape(-1, in_features), payload, scales, lut,
                                                        int(out_features), int(layout), A, B, float(scale))
    return y.view(*x.shape[:-1], out_features)


# ------------------------------------------------------------------ grouped (MoE experts)
def _grouped_ws(rows, E, N, K, rank, device):
    n = _lib.load().fl_grouped_workspace_bytes(rows, E, N, K, rank)
    return torch.empty(n, dtype=torch.uint8, device=device), n


@torch.library.custom_op(f"{_NS}::grouped_frozen_lora_linear", mutates_args=(), device_types="cuda")
def _grouped_fwd(xs: Tensor, seg: Tensor, payload: Tensor, scales: Tensor, lut: Tensor, experts: int,
                 out_features: int, A: Optional[Tensor], B: Optional[Tensor], scale: float) -> Tensor:
    xs = xs.contiguous()
    rows, K = xs.shape
    N, E = out_features, experts
    rank = 0 if A is None else A.shape[-2]
    y = torch.empty((rows, N), dtype=torch.bfloat16, device=xs.device)
    if rows:
        A = A.detach().contiguous() if rank else None
        B = B.detach().contiguous() if rank else None
        ws, n = _grouped_ws(rows, E, N, K, rank, xs.device)
        _lib.call("fl_grouped_fwd", _ptr(xs), _ptr(seg), rows, K, E, _ptr(payload), _ptr(scales), _ptr(lut), N,
                  _ptr(A), _ptr(B), rank, float(scale), _ptr(y), _ptr(ws), n, _stream())
    return y


@_grouped_fwd.register_fake
def _(xs, seg, payload, scales, lut, experts, out_features, A, B, scale):
    return xs.new_empty((xs.shape[0], out_features))


@torch.library.custom_op(f"{_NS}::grouped_frozen_lora_linear_backward", mutates_args=(), device_types="cuda")
def _grouped_bwd(dy: Tensor, xs: Tensor, seg: Tensor, payload: Tensor, scales: Tensor, lut: Tensor, experts: int,
                 A: Optional[Tensor], B: Optional[Tensor], scale: float) -> Tuple[Tensor, Tensor, Tensor]:
    dy = dy.contiguous()
    xs = xs.contiguous()
    rows, N = dy.shape
    K = xs.shape[1]
    E = experts
    rank = 0 if A is None else A.shape[-2]
    dx = torch.empty((rows, K), dtype=torch.bfloat16, device=dy.device)
    if rank:
        dA = torch.empty((E, rank, K), dtype=torch.float32, device=dy.device)
        dB = torch.empty((E, N, rank), dtype=torch.float32, device=dy.device)
        A, B = A.detach().contiguous(), B.detach().contiguous()
    else:
        dA = torch.empty((0,), dtype=torch.float32, device=dy.device)
        dB = torch.empty((0,), dtype=torch.float32, device=dy.device)
    if rows:
        ws, n = _grouped_ws(rows, E, N, K, rank, dy.device)
        _lib.call("fl_grouped_bwd", _ptr(dy), _ptr(xs) if rank else None, _ptr(seg), rows, N, K, E, _ptr(payload),
                  _ptr(scales), _ptr(lut), _ptr(A) if rank else None, _ptr(B) if rank else None, rank, float(scale),
                  _ptr(dx), _ptr(dA) if rank else None, _ptr(dB) if rank else None, 0, _ptr(ws), n, _stream())
    elif rank:
        dA.zero_()
        dB.zero_()
    return dx, dA, dB


@_grouped_bwd.register_fake
def _(dy, xs, seg, payload, scales, lut, experts, A, B, scale):
    dx = xs.new_empty(xs.shape)
    if A is None:
        return dx, dy.new_empty((0,), dtype=torch.float32), dy.new_empty((0,), dtype=torch.float32)
    return dx, A.new_empty(A.shape), B.new_empty(B.shape)


def _grouped_setup(ctx, inputs, output):
    xs, seg, payload, scales, lut, experts, out_features, A, B, scale = inputs
    ctx.experts, ctx.scale, ctx.has_lora = experts, scale, A is not None
    ctx.save_for_backward(xs, seg, payload, scales, lut, A, B)


def _grouped_backward(ctx, dy):
    xs, seg, payload, scales, lut, A, B = ctx.saved_tensors
    dx, dA, dB = torch.ops.spilltune_b200.grouped_frozen_lora_linear_backward(dy, xs, seg, payload, scales, lut,
                                                                              ctx.experts, A, B, ctx.scale)
    if not ctx.has_lora:
        dA = dB = None
    return dx, None, None, None, None, None, None, dA, dB, None


_grouped_fwd.register_autograd(_grouped_backward, setup_context=_grouped_setup)
