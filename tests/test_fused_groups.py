"""Projections that share their input (q, k, v; gate, up) as one fused call.

CPU: a layer packed like a slot image (``streaming.pack_layer`` /
``PackedSlotSession``) holds adjacent matrices back to back, so
``ops.concat_records`` sees them as one stacked record, and refuses records
that are not adjacent; ``ops.concat_lora`` builds [A_1; A_2] and
blockdiag(B_1, B_2) with zero blocks for projections without LoRA.
GPU: the fused call equals the separate calls (outputs within the usual 5e-3
of each other and of the FP32 shadow), and through autograd every A_i, B_i and
the input get the separate calls' gradients.
"""
import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol


def _layer(seed=3, shapes=(("q", 512, 256), ("k", 128, 256), ("v", 128, 256), ("o", 256, 512))):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(seed)
    return {n: codec.encode(torch.randn(N, K, generator=g) * 0.02, "nf4-g128") for n, N, K in shapes}


def test_concat_records_over_a_packed_layer():
    from spilltune_b200 import ops, streaming
    layer = _layer()
    _, v = streaming.pack_layer(layer, "cpu")
    cat = ops.concat_records([v["q"], v["k"], v["v"]])
    assert cat is not None and cat.shape == (768, 256)
    assert torch.equal(cat.payload, torch.cat([layer[n].payload for n in ("q", "k", "v")]))
    assert torch.equal(cat.scales, torch.cat([layer[n].scales for n in ("q", "k", "v")]))
    assert ops.concat_records([v["q"], v["v"]]) is None         # not adjacent
    assert ops.concat_records([v["v"], v["o"]]) is None         # different input width
    assert ops.concat_records([layer["q"], layer["k"]]) is None  # separate allocations
    assert ops.concat_records([v["q"]]) is None


def test_concat_lora_block_layout():
    from spilltune_b200 import ops
    g = torch.Generator().manual_seed(1)
    Aq, Bq = torch.randn(8, 256, generator=g), torch.randn(512, 8, generator=g)
    Av, Bv = torch.randn(8, 256, generator=g), torch.randn(128, 8, generator=g)
    A, B = ops.concat_lora([(Aq, Bq), None, (Av, Bv)], [512, 128, 128])
    assert A.shape == (16, 256) and B.shape == (768, 16)
    assert torch.equal(A[:8], Aq) and torch.equal(A[8:], Av)
    assert torch.equal(B[:512, :8], Bq) and torch.equal(B[640:, 8:], Bv)
    assert int(B[:512, 8:].count_nonzero()) == 0 and int(B[512:640].count_nonzero()) == 0
    assert int(B[640:, :8].count_nonzero()) == 0
    assert ops.concat_lora([None, None], [4, 4]) == (None, None)


def _decode(pw):
    bits = oc.decode(pw.payload.cpu().numpy(), pw.scales.cpu().numpy(), pw.numel, lut=pw.lut.cpu().numpy())
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).view(*pw.shape)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [300, 12])
def test_fused_matches_separate_calls(cuda_lib, M):
    from spilltune_b200 import ops, streaming
    layer = _layer(shapes=(("q", 512, 512), ("k", 128, 512), ("v", 128, 512)))
    _, v = streaming.pack_layer(layer, "cuda")
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M, 512, generator=g).to(torch.bfloat16).cuda()
    f = {n: ((torch.randn(8, 512, generator=g) * 0.05).cuda().requires_grad_(True),
             (torch.randn(v[n].shape[0], 8, generator=g) * 0.05).cuda().requires_grad_(True)) for n in ("q", "v")}
    names = ("q", "k", "v")
    factors = [f.get(n) for n in names]
    xf = x.clone().requires_grad_(True)
    fused = ops.fused_lora_linears(xf, [v[n] for n in names], factors, 2.0)
    xs = x.clone().requires_grad_(True)
    sep = [ops.frozen_lora_linear(xs, v[n], *(f[n] if n in f else (None, None)), 2.0) for n in names]
    for a, b, n in zip(fused, sep, names):
        assert a.shape == b.shape
        assert ol.rel_l2(a.float().cpu(), b.float().cpu()) <= 5e-3, n
        W = _decode(layer[n])
        ref = ol.lora_forward_fp32(x.cpu(), W, *(t.detach().cpu() for t in f[n]), 2.0) if n in f \
            else x.cpu().float() @ W.float().t()
        assert ol.rel_l2(a.float().cpu(), ref) <= 5e-3, n
    gy = [torch.randn(a.shape, generator=g).to(torch.bfloat16).cuda() for a in fused]
    leaves = [xf] + [t for n in ("q", "v") for t in f[n]]
    gf = torch.autograd.grad(fused, leaves, gy)
    gs = torch.autograd.grad(sep, [xs] + [t for n in ("q", "v") for t in f[n]], gy)
    for a, b in zip(gf, gs):
        assert ol.rel_l2(a.float().cpu(), b.float().cpu()) <= 5e-3
