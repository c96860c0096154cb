"""The torch.library custom ops: schema, fake (meta) kernels, autograd
registration and AOT dispatch checked by ``torch.library.opcheck``, and the
autograd results against the FP32 shadow."""
import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol

pytestmark = pytest.mark.gpu

# dA/dB are accumulated with atomic adds, so two runs can differ in the last bits.
TOL = dict(atol=1e-3, rtol=1e-3)


def _decode_cpu(pw):
    bits = oc.decode(pw.payload.cpu().numpy(), pw.scales.cpu().numpy(), pw.numel, lut=pw.lut.cpu().numpy())
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).view(*pw.shape)


def _dense(M, N, K, rank, seed=3):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(seed)
    pw = codec.encode(torch.randn(N, K, generator=g) * 0.02, "nf4-g128")
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    A = torch.randn(rank, K, generator=g) * 0.05 if rank else None
    B = torch.randn(N, rank, generator=g) * 0.05 if rank else None
    return pw, x, A, B


@pytest.mark.parametrize("M,N,K,rank", [(200, 256, 512, 16), (8, 256, 512, 16), (64, 128, 256, 0)])
def test_opcheck_frozen_lora_linear(cuda_lib, M, N, K, rank):
    import spilltune_b200.library  # noqa: F401
    pw, x, A, B = _dense(M, N, K, rank)
    pwc = pw.to("cuda")
    xc = x.cuda().requires_grad_(True)
    Ac = A.cuda().requires_grad_(True) if rank else None
    Bc = B.cuda().requires_grad_(True) if rank else None
    args = (xc, pwc.payload, pwc.scales, pwc.lut, N, 0, Ac, Bc, 2.0)
    torch.library.opcheck(torch.ops.spilltune_b200.frozen_lora_linear.default, args, **TOL)
    y, ts = torch.ops.spilltune_b200.frozen_lora_linear(*args)
    dy = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    # The backward op has no autograd formula of its own (no double backward):
    # its inputs are plain tensors.
    bargs = (dy, xc.detach(), pwc.payload, pwc.scales, pwc.lut, 0,
             None if Ac is None else Ac.detach(), None if Bc is None else Bc.detach(), 2.0, ts.detach())
    torch.library.opcheck(torch.ops.spilltune_b200.frozen_lora_linear_backward.default, bargs, **TOL)


def test_opcheck_grouped(cuda_lib):
    import spilltune_b200.library  # noqa: F401
    from spilltune_b200 import codec, moe
    g = torch.Generator().manual_seed(4)
    E, N, K, r, T, k = 4, 256, 256, 8, 96, 2
    pw = codec.encode(torch.randn(E, N, K, generator=g) * 0.02, "nf4-g128").to("cuda")
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).cuda()
    segs = moe.expert_segments(idx, E)
    xs = torch.randn(T * k, K, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    A = (torch.randn(E, r, K, generator=g) * 0.05).cuda().requires_grad_(True)
    B = (torch.randn(E, N, r, generator=g) * 0.05).cuda().requires_grad_(True)
    args = (xs, segs.seg, pw.payload, pw.scales, pw.lut, E, N, A, B, 2.0)
    torch.library.opcheck(torch.ops.spilltune_b200.grouped_frozen_lora_linear.default, args, **TOL)


def test_autograd_through_op_matches_fp32_shadow(cuda_lib):
    from spilltune_b200 import ops
    M, N, K, r, s = 300, 384, 512, 16, 2.0
    pw, x, A, B = _dense(M, N, K, r, seed=8)
    dy = torch.randn(M, N, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16)
    xc = x.cuda().requires_grad_(True)
    Ac, Bc = A.cuda().requires_grad_(True), B.cuda().requires_grad_(True)
    y = ops.frozen_lora_linear(xc.view(3, 100, K), pw.to("cuda"), Ac, Bc, s)
    assert y.shape == (3, 100, N)
    gx, gA, gB = torch.autograd.grad(y, (xc, Ac, Bc), dy.cuda().view(3, 100, N))
    W = _decode_cpu(pw)
    rdx, rdA, rdB = ol.lora_backward_fp32(x, W, A, B, s, dy)
    assert ol.rel_l2(y.detach().view(M, N).cpu(), ol.lora_forward_fp32(x, W, A, B, s)) <= 5e-3
    assert max(ol.rel_l2(gx.cpu(), rdx), ol.rel_l2(gA.cpu(), rdA), ol.rel_l2(gB.cpu(), rdB)) <= 5e-3


def test_in_place_change_of_A_before_backward_is_caught(cuda_lib):
    """Ts (bf16(s * x . A^T)) is saved for the backward with autograd's version
    check: changing A in place between forward and backward raises, as the
    reference's autograd does, instead of using stale low-rank activations."""
    from spilltune_b200 import ops
    pw, x, A, B = _dense(256, 256, 256, 8, seed=12)
    xc = x.cuda().requires_grad_(True)
    Ac, Bc = A.cuda().requires_grad_(True), B.cuda().requires_grad_(True)
    y = ops.frozen_lora_linear(xc, pw.to("cuda"), Ac, Bc, 2.0)
    with torch.no_grad():
        Ac.add_(1.0)
    with pytest.raises(RuntimeError, match="modified by an inplace operation"):
        y.sum().backward()
