"""Chunked LM-head cross-entropy oracle — TEST INFRASTRUCTURE ONLY.

A restatement of the reference's ``_ChunkedCE.forward``
(ram_vram_finetune/quantization/native_terminal.py:11-34): per supervised
chunk, bf16 logits = F.linear(h, head), FP32 summed cross-entropy with
ignore_index -100 against the shifted labels, and the hidden-state gradient of
loss / normalization by autograd.  Returns (loss, vjp).
"""
import torch
import torch.nn.functional as F


def chunked_ce(normalized, head, labels, normalization, supervised_chunks):
    vjp = torch.zeros_like(normalized)
    total = torch.zeros((), dtype=torch.float32)
    for start, end in supervised_chunks:
        target = labels[:, start + 1:end + 1]
        h = normalized[:, start:end].detach().requires_grad_(True)
        logits = F.linear(h, head)
        value = F.cross_entropy(logits.float().reshape(-1, head.shape[0]), target.reshape(-1),
                                ignore_index=-100, reduction="sum")
        (grad,) = torch.autograd.grad(value / normalization, h)
        vjp[:, start:end].copy_(grad.detach())
        total += value.detach()
    return total / normalization, vjp
