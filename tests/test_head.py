"""Chunked LM head + cross-entropy (the reference's terminal, native_terminal.py:11-47).

GPU: loss and hidden-state VJP of ``spilltune_b200.head.chunked_causal_loss``
against the oracle restatement of ``_ChunkedCE`` (CPU, same bf16 logits, FP32
CE): loss within 1e-3 relative, VJP within rel-L2 1e-2.  CPU: argument checks.
"""
import pytest
import torch

import oracle.head as oh
import oracle.linear as ol


def _case(Bsz, S, H, V, seed, ignore_frac=0.2):
    g = torch.Generator().manual_seed(seed)
    normalized = torch.randn(Bsz, S, H, generator=g).to(torch.bfloat16)
    head = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16)
    labels = torch.randint(0, V, (Bsz, S), generator=g)
    labels[torch.rand(Bsz, S, generator=g) < ignore_frac] = -100
    return normalized, head, labels


def test_argument_checks():
    from spilltune_b200 import head as hd
    n, h, l = _case(1, 8, 16, 32, 0)
    with pytest.raises(ValueError, match="token chunk/normalization"):
        hd._ChunkedCE.forward(None, n, h, l, 0.0, 4, ((0, 4),))
    with pytest.raises(ValueError, match="labels/trainable"):
        hd._ChunkedCE.forward(None, n, h, l[:, :4], 1.0, 4, ((0, 4),))
    with pytest.raises(ValueError, match="CUDA tensors"):
        hd.chunked_causal_loss(n, h, l, normalization=1.0, token_chunk=4)
    # A target outside [0, V) that is not the ignore index: F.cross_entropy raises, so does this.
    bad = l.clone()
    bad[0, 3] = 32
    with pytest.raises(ValueError, match="out of bounds"):
        hd._ChunkedCE.forward(None, n, h, bad, 1.0, 4, ((0, 4),))
    bad[0, 3] = -3
    with pytest.raises(ValueError, match="out of bounds"):
        hd._ChunkedCE.forward(None, n, h, bad, 1.0, 4, ((0, 4),))


@pytest.mark.gpu
@pytest.mark.parametrize("Bsz,S,H,V,chunk", [(2, 64, 256, 1000, 32), (1, 300, 512, 4096, 128),
                                             (2, 129, 128, 2048, 64)])
def test_matches_reference_chunked_ce(cuda_lib, Bsz, S, H, V, chunk):
    from spilltune_b200 import head as hd
    normalized, head, labels = _case(Bsz, S, H, V, S + V)
    norm = float((labels[:, 1:] != -100).sum())
    chunks = tuple((s, min(s + chunk, S - 1)) for s in range(0, S - 1, chunk)
                   if bool((labels[:, s + 1:min(s + chunk, S - 1) + 1] != -100).any()))
    ref_loss, ref_vjp = oh.chunked_ce(normalized, head, labels, norm, chunks)
    x = normalized.cuda().requires_grad_(True)
    loss = hd.chunked_causal_loss(x, head.cuda(), labels.cuda(), normalization=norm, token_chunk=chunk,
                                  supervised_chunks=chunks)
    (vjp,) = torch.autograd.grad(loss, (x,))
    assert abs(float(loss) - float(ref_loss)) <= 1e-3 * abs(float(ref_loss))
    assert ol.rel_l2(vjp.cpu(), ref_vjp) <= 1e-2


@pytest.mark.gpu
def test_llama3_head_shape_chunk(cuda_lib):
    """One 256-token chunk at the Llama-3-8B head shape (V=128256, H=4096):
    loss and sampled gradient rows against an FP32 evaluation of the same
    bf16 logits (computed with torch on the GPU as the checker)."""
    from spilltune_b200 import head as hd
    T, H, V = 256, 4096, 128256
    g = torch.Generator().manual_seed(7)
    h = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    head = (torch.randn(V, H, generator=g) * 0.02).to(torch.bfloat16).cuda()
    tg = torch.randint(0, V, (T,), generator=g)
    tg[::7] = -100
    tg = tg.cuda()
    loss = torch.zeros((), dtype=torch.float32, device="cuda")
    dh = hd.ce_chunk(h, head, tg, 1.0, loss)
    logits = (h.float() @ head.float().t()).to(torch.bfloat16).float()
    keep = tg != -100
    ref_loss = float((torch.logsumexp(logits[keep], -1) - logits[keep, tg[keep]]).sum())
    assert abs(float(loss) - ref_loss) <= 1e-3 * abs(ref_loss)
    rows = torch.tensor([0, 1, 100, 255], device="cuda")
    p = torch.softmax(logits[rows], dim=-1)
    p[torch.arange(4, device="cuda"), tg[rows].clamp_min(0)] -= 1.0
    p[~keep[rows]] = 0
    ref_dh = p.to(torch.bfloat16).float() @ head.float()
    assert ol.rel_l2(dh[rows].cpu(), ref_dh.cpu()) <= 1e-2


def _golden():
    import os
    import numpy as np
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "head_small.npz"))
    bf = lambda a, shp: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).view(*shp)
    B, S, H, V = (int(g[k]) for k in ("B", "S", "H", "V"))
    return (bf(g["normalized_bf16"], (B, S, H)), bf(g["head_bf16"], (V, H)), torch.from_numpy(g["labels"]),
            float(g["normalization"]), int(g["token_chunk"]), float(g["loss"]), bf(g["dnormalized_bf16"], (B, S, H)))


def _chunks(labels, S, chunk):
    return tuple((s, min(s + chunk, S - 1)) for s in range(0, S - 1, chunk)
                 if bool((labels[:, s + 1:min(s + chunk, S - 1) + 1] != -100).any()))


def test_oracle_matches_reference_golden():
    """oracle/head.py against the reference's own chunked_causal_loss output
    (tests/golden/head_small.npz, made by tests/golden/make_golden.py)."""
    normalized, head, labels, norm, chunk, ref_loss, ref_grad = _golden()
    loss, vjp = oh.chunked_ce(normalized, head, labels, norm, _chunks(labels, normalized.shape[1], chunk))
    assert abs(float(loss) - ref_loss) <= 1e-6 * abs(ref_loss)
    assert ol.rel_l2(vjp, ref_grad) <= 1e-6


@pytest.mark.gpu
def test_fused_head_matches_reference_golden(cuda_lib):
    from spilltune_b200 import head as hd
    normalized, head, labels, norm, chunk, ref_loss, ref_grad = _golden()
    x = normalized.cuda().requires_grad_(True)
    loss = hd.chunked_causal_loss(x, head.cuda(), labels.cuda(), normalization=norm, token_chunk=chunk,
                                  supervised_chunks=_chunks(labels, normalized.shape[1], chunk))
    (vjp,) = torch.autograd.grad(loss, (x,))
    assert abs(float(loss) - ref_loss) <= 1e-3 * abs(ref_loss)
    assert ol.rel_l2(vjp.cpu(), ref_grad) <= 1e-2
