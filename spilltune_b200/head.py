"""Chunked LM head + shifted cross-entropy on the B200 kernels.

Drop-in for the reference's terminal ``chunked_causal_loss``
(ram_vram_finetune/quantization/native_terminal.py:11-47; the same loop runs
inline in ``microbatch``, training/engine.py:58-78): for each supervised token
chunk, logits = normalized[:, start:end] . head^T (bf16), summed FP32
cross-entropy against labels[:, start+1:end+1] (ignore index -100), and the
hidden-state VJP of loss / normalization, all retained as one full VJP.  One
chunk of logits exists at a time, in a caller-visible workspace.

Per chunk ``fl_ce_chunk`` runs the logits GEMM with the CE partials fused in
its epilogue, the row log-sum-exp, dlogits in place and the dh GEMM (see
csrc/fl_head.cu).  CUDA only; no CPU fallback.
"""
import math

import torch

from . import _lib
from .ops import _need_cuda, _ptr, _stream

IGNORE = -100


def ce_chunk(h, head, targets, normalization, loss_acc):
    """One chunk: h [T, H] bf16, head [V, H] bf16 (frozen), targets int64 [T]
    (IGNORE = no loss).  Adds the chunk's summed CE into ``loss_acc`` (fp32
    scalar on the device) and returns dh = d(CE / normalization) / dh (bf16).
    Targets are not checked on the host here (that would synchronise): a value
    outside [0, V) other than IGNORE adds no loss, gets a zero ``dh`` row and
    sets status bit 5, which ``_lib.status()`` reports."""
    _need_cuda(h, head, targets, loss_acc)
    h = h.contiguous()
    head = head.contiguous()
    targets = targets.to(torch.int64).contiguous()
    T, H = h.shape
    V = head.shape[0]
    if head.shape[1] != H or targets.numel() != T:
        raise ValueError("head [V, H] and targets [T] must match the hidden states [T, H]")
    dh = torch.empty_like(h)
    n = _lib.load().fl_ce_workspace_bytes(T, V)
    ws = torch.empty(n + 256, dtype=torch.uint8, device=h.device)
    base = (ws.data_ptr() + 255) // 256 * 256
    _lib.call("fl_ce_chunk", _ptr(h), T, H, _ptr(head), V, _ptr(targets), 1.0 / float(normalization),
              _ptr(loss_acc), _ptr(dh), base, n, _stream())
    return dh


class _ChunkedCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, normalized, head, labels, normalization, token_chunk, supervised_chunks):
        if type(token_chunk) is not int or token_chunk < 1 or not math.isfinite(normalization) or normalization <= 0:
            raise ValueError("invalid terminal token chunk/normalization")
        if labels.shape != normalized.shape[:2] or head.requires_grad:
            raise ValueError("invalid terminal labels/trainable frozen head")
        # F.cross_entropy raises for a target outside [0, V) that is not the
        # ignore index; so does this (one host check per call, not per chunk).
        bad = (labels != IGNORE) & ((labels < 0) | (labels >= head.shape[0]))
        if bool(bad.any()):
            raise ValueError(f"Target {int(labels[bad].reshape(-1)[0])} is out of bounds.")
        vjp = torch.zeros_like(normalized)
        total = torch.zeros((), dtype=torch.float32, device=normalized.device)
        Bsz, _, H = normalized.shape
        for start, end in supervised_chunks:
            h = normalized[:, start:end].reshape(-1, H)
            target = labels[:, start + 1:end + 1].reshape(-1)
            dh = ce_chunk(h, head, target, normalization, total)
            vjp[:, start:end].copy_(dh.view(Bsz, end - start, H))
        ctx.save_for_backward(vjp)
        return total / normalization

    @staticmethod
    def backward(ctx, output_gradient):
        (vjp,) = ctx.saved_tensors
        return vjp * output_gradient, None, None, None, None, None


def chunked_causal_loss(normalized, head, labels, *, normalization, token_chunk, supervised_chunks=None):
    """Same arguments, result and errors as the reference's function; the
    supervised chunk intervals must be prepared up front for CUDA labels."""
    if supervised_chunks is None:
        if labels.device.type != "cpu":
            raise RuntimeError("CUDA terminal requires startup-prepared supervised chunks")
        if type(token_chunk) is not int or token_chunk < 1:
            raise ValueError("invalid terminal token chunk")
        S = normalized.shape[1]
        supervised_chunks = tuple((s, min(s + token_chunk, S - 1)) for s in range(0, S - 1, token_chunk)
                                  if bool((labels[:, s + 1:min(s + token_chunk, S - 1) + 1] != IGNORE).any()))
    _need_cuda(normalized, head)
    return _ChunkedCE.apply(normalized, head, labels.to(normalized.device), normalization, token_chunk,
                            tuple(supervised_chunks))
