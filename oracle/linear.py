"""CPU oracle of the frozen linear + LoRA projection — test infrastructure only.

Two restatements, both in torch on the CPU:

* ``*_reference`` keeps the reference's op order and roundings:
  ``LoRAProjection.forward`` (ram_vram_finetune/finetune/lora.py:205-220)
      base = F.linear(x, W)                     # BF16 GEMM, BF16 output
      lora = F.linear(F.linear(x.float(), A), B)
      out  = (base.float() + lora * s).to(bf16)
  and its autograd backward as driven by ``StreamingBlockFunction.backward``
  (ram_vram_finetune/training/recompute.py:85-127):
      dX = bf16(dY @ W) + bf16(s * (dY.f32 @ B) @ A)   (BF16 add)
      dA = s * (dY.f32 @ B).T @ x.f32,  dB = s * dY.f32.T @ (x.f32 @ A.T)

* ``*_fp32`` is the FP32 shadow (``W.float()``, ``x.float()``, no BF16
  rounding) that the parity bar rel-L2 <= 1e-2 is measured against.
"""
import torch
import torch.nn.functional as F


def lora_forward_reference(x, W, A, B, scale):
    base = F.linear(x, W)
    lora = F.linear(F.linear(x.float(), A), B)
    return (base.float() + lora * scale).to(base.dtype)


def lora_backward_reference(x, W, A, B, scale, dY):
    """Autograd through lora_forward_reference, exactly like recompute.py:102-105."""
    x = x.detach().requires_grad_(True)
    A = A.detach().clone().requires_grad_(True)
    B = B.detach().clone().requires_grad_(True)
    with torch.enable_grad():
        out = lora_forward_reference(x, W.detach(), A, B, scale)
        dx, da, db = torch.autograd.grad(out, (x, A, B), dY)
    return out.detach(), dx, da, db


def lora_forward_fp32(x, W, A, B, scale):
    xf = x.float()
    return xf @ W.float().t() + scale * (xf @ A.t()) @ B.t()


def lora_backward_fp32(x, W, A, B, scale, dY):
    xf, gf, Wf = x.float(), dY.float(), W.float()
    u = gf @ B                      # [M, r]
    t = xf @ A.t()                  # [M, r]
    dx = gf @ Wf + scale * u @ A
    da = scale * u.t() @ xf
    db = scale * gf.t() @ t
    return dx, da, db


def rel_l2(a, b):
    a = a.double()
    b = b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))
