"""GPU parity of the grouped (MoE expert) path through the C ABI.

* grouped forward rows are bit-identical to the dense kernel run with the
  row's expert weight (both use the same per-row tcgen05 accumulation order);
  grouped dX likewise; per-expert dA/dB equal the dense kernel's on the
  expert's rows up to FP32 summation order;
* all outputs within rel-L2 <= 1e-2 (and the tighter 5e-3 line) of the FP32
  per-expert reference (oracle/moe.py) on the oracle-decoded weights;
* the whole Qwen3-MoE expert layer reproduces the reference's own
  moe_feed_forward output and hidden-state gradient (tests/golden/moe_small.npz)
  and, at the Qwen3-30B-A3B expert shape, the per-expert loop oracle;
* invalid segment offsets are reported through the status word, not a fault.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol
import oracle.moe as om

pytestmark = pytest.mark.gpu

BAR = 1e-2
TIGHT = 5e-3
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _decode_cpu(pw):
    bits = oc.decode(pw.payload.cpu().numpy(), pw.scales.cpu().numpy(), pw.numel, lut=pw.lut.cpu().numpy())
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).view(*pw.shape)


def _segments(lengths, device="cuda"):
    from spilltune_b200 import moe
    rows = int(sum(lengths))
    seg = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32, device=device)
    ar = torch.arange(rows, device=device)
    return moe.ExpertSegments(ar, ar, ar, seg, len(lengths), 1)


def _expert_view(pw, e):
    from spilltune_b200 import codec
    E, N, K = pw.shape
    per = N * K
    return codec.PackedWeight(pw.payload[e * per // 2:(e + 1) * per // 2], pw.scales[e * per // 128:(e + 1) * per // 128],
                              pw.lut, (N, K), pw.codec)


def _grouped_problem(lengths, N, K, rank, codec_name, seed):
    from spilltune_b200 import codec
    E = len(lengths)
    rows = int(sum(lengths))
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(E, N, K, generator=g) * 0.02
    pw = codec.encode(w, codec_name)
    x = torch.randn(rows, K, generator=g).to(torch.bfloat16)
    A = torch.randn(E, rank, K, generator=g) * 0.05 if rank else None
    B = torch.randn(E, N, rank, generator=g) * 0.05 if rank else None
    dy = torch.randn(rows, N, generator=g).to(torch.bfloat16)
    return pw, x, A, B, dy


def _cuda(t):
    return None if t is None else t.cuda()


CASES = [
    # lengths per expert (empty, 1-row and tile-crossing segments), N, K, rank
    ([17, 0, 283, 1], 256, 256, 0),
    ([17, 0, 283, 1], 256, 256, 8),
    ([5, 130, 257, 0, 64, 300, 2, 40], 384, 512, 16),
    ([200, 90, 512, 33, 129, 0], 1536, 2048, 8),     # Qwen3-30B-A3B expert gate_up
    ([200, 90, 512, 33, 129, 0], 2048, 768, 8),      # ... and down
    ([600, 1, 1, 700], 512, 1024, 64),
    ([512, 700, 300, 600], 4096, 1024, 16),         # >= 384 rows per expert, N >= 4096: 512-token backward tiles
    ([128, 0, 200, 64], 4096, 7168, 16),            # DeepSeek-V3 expert gate_up (2 x 2048), ~128 rows each
    ([128, 0, 200, 64], 7168, 2048, 16),            # ... and down
]


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("lengths,N,K,rank", CASES)
def test_grouped_fwd(cuda_lib, codec_name, lengths, N, K, rank):
    from spilltune_b200 import moe, ops
    pw, x, A, B, _ = _grouped_problem(lengths, N, K, rank, codec_name, seed=N + K + rank)
    s = 2.0
    segs = _segments(lengths)
    pwc, xc, Ac, Bc = pw.to("cuda"), x.cuda(), _cuda(A), _cuda(B)
    y = moe.grouped_fwd(xc, segs, pwc, Ac, Bc, s)
    seg = segs.seg.tolist()
    for e in range(len(lengths)):
        a, b = seg[e], seg[e + 1]
        if a == b:
            continue
        # Without a split of the reduction: the grouped kernel sums each output tile in one pass too.
        dense = ops.fwd(xc, _expert_view(pwc, e), None if A is None else Ac[e], None if B is None else Bc[e], s,
                        split_reduction=False)
        assert torch.equal(y[a:b], dense[a:b]), e
    ref = om.grouped_linear_fp32(x, seg, _decode_cpu(pw), A, B, s)
    err = ol.rel_l2(y.cpu(), ref)
    assert err <= BAR and err <= TIGHT, err


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("lengths,N,K,rank", CASES)
def test_grouped_bwd(cuda_lib, codec_name, lengths, N, K, rank):
    from spilltune_b200 import moe, ops
    pw, x, A, B, dy = _grouped_problem(lengths, N, K, rank, codec_name, seed=3 * N + K + rank)
    s = 2.0
    segs = _segments(lengths)
    pwc, xc, Ac, Bc, dyc = pw.to("cuda"), x.cuda(), _cuda(A), _cuda(B), dy.cuda()
    dx, dA, dB = moe.grouped_bwd(dyc, xc, segs, pwc, Ac, Bc, s)
    seg = segs.seg.tolist()
    for e in range(len(lengths)):
        a, b = seg[e], seg[e + 1]
        pe = _expert_view(pwc, e)
        if rank:
            if a == b:
                assert torch.count_nonzero(dA[e]) == 0 and torch.count_nonzero(dB[e]) == 0
                continue
            ddx, _, _ = ops.bwd(dyc, xc, pe, Ac[e], Bc[e], s, split_reduction=False)
            _, edA, edB = ops.bwd(dyc[a:b].contiguous(), xc[a:b].contiguous(), pe, Ac[e], Bc[e], s)
            # A segment of <= 16 rows takes the decode-step backward when run alone, whose
            # Us / Ts are exact FP32 sums (the grouped path's low-rank kernel carries ~16
            # mantissa bits), so a bf16 rounding of Us / Ts may differ there.
            tol = 1e-5 if b - a > 16 else TIGHT
            assert ol.rel_l2(dA[e].cpu(), edA.cpu()) < tol
            assert ol.rel_l2(dB[e].cpu(), edB.cpu()) < tol
        elif a == b:
            continue
        else:
            ddx, _, _ = ops.bwd(dyc, None, pe, split_reduction=False)
        assert torch.equal(dx[a:b], ddx[a:b]), e
    rdx, rdA, rdB = om.grouped_linear_grads_fp32(dy, x, seg, _decode_cpu(pw), A, B, s)
    errs = [ol.rel_l2(dx.cpu(), rdx)]
    if rank:
        errs += [ol.rel_l2(dA.cpu(), rdA), ol.rel_l2(dB.cpu(), rdB)]
    assert max(errs) <= BAR and max(errs) <= TIGHT, errs


def test_grouped_bwd_accumulate(cuda_lib):
    from spilltune_b200 import moe
    lengths = [64, 0, 300, 7]
    pw, x, A, B, dy = _grouped_problem(lengths, 256, 256, 8, "nf4-g128", seed=77)
    segs = _segments(lengths)
    pw, x, A, B, dy = pw.to("cuda"), x.cuda(), A.cuda(), B.cuda(), dy.cuda()
    _, dA1, dB1 = moe.grouped_bwd(dy, x, segs, pw, A, B, 2.0)
    dA, dB = dA1.clone(), dB1.clone()
    moe.grouped_bwd(dy, x, segs, pw, A, B, 2.0, dA=dA, dB=dB, accumulate=True)
    assert ol.rel_l2(dA.cpu(), 2 * dA1.cpu()) < 1e-6 and ol.rel_l2(dB.cpu(), 2 * dB1.cpu()) < 1e-6
    moe.grouped_bwd(dy, x, segs, pw, A, B, 2.0, dA=dA, dB=dB, accumulate=False)
    assert ol.rel_l2(dA.cpu(), dA1.cpu()) < 1e-6


def _fixture_records():
    from spilltune_b200 import codec
    z = np.load(os.path.join(GOLD, "moe_small.npz"))
    E, H, I, T = int(z["E"]), int(z["H"]), int(z["I"]), int(z["T"])
    bf = lambda a, shp: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).view(*shp)
    gu = codec.PackedWeight(torch.from_numpy(z["gate_up_payload"]), torch.from_numpy(z["gate_up_scales"]),
                            codec.INT4_SYM_LUT, (E, 2 * I, H))
    dn = codec.PackedWeight(torch.from_numpy(z["down_payload"]), torch.from_numpy(z["down_scales"]),
                            codec.INT4_SYM_LUT, (E, H, I))
    shp = (2, T // 2, H)
    return z, E, int(z["top_k"]), gu, dn, bf(z["gate_bf16"], (E, H)), bf(z["hidden_bf16"], shp), \
        bf(z["out_bf16"], shp), bf(z["dout_bf16"], shp), bf(z["dhidden_bf16"], shp)


def test_moe_feed_forward_matches_reference_golden(cuda_lib):
    """Output and hidden-state gradient of the reference's own moe_feed_forward."""
    from spilltune_b200 import moe
    z, E, k, gu, dn, gate, hidden, out_ref, dout, dh_ref = _fixture_records()
    weights = {"mlp.gate.weight": gate.cuda(), "mlp.experts.gate_up_proj": gu.to("cuda"),
               "mlp.experts.down_proj": dn.to("cuda")}
    h = hidden.cuda().requires_grad_(True)
    out = moe.moe_feed_forward(h, weights, num_experts=E, top_k=k, norm_topk_prob=True)
    (dh,) = torch.autograd.grad(out, (h,), dout.cuda())
    assert ol.rel_l2(out.detach().cpu(), out_ref) <= BAR
    assert ol.rel_l2(dh.cpu(), dh_ref) <= BAR


@pytest.mark.parametrize("T,E,k,H,I", [(512, 128, 8, 2048, 768), (256, 16, 4, 1024, 512)])
def test_moe_layer_matches_loop_oracle(cuda_lib, T, E, k, H, I):
    """Qwen3-30B-A3B expert shapes (E=128, top-8, H=2048, I=768) with random
    routing: the grouped layer against the per-expert loop on decoded weights."""
    from spilltune_b200 import codec, moe, ops
    g = torch.Generator().manual_seed(T + E)
    hidden = torch.randn(1, T, H, generator=g).to(torch.bfloat16)
    gate = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    gu = codec.encode(torch.randn(E, 2 * I, H, generator=g) * 0.02, "nf4-g128").to("cuda")
    dn = codec.encode(torch.randn(E, H, I, generator=g) * 0.02, "nf4-g128").to("cuda")
    weights = {"mlp.gate.weight": gate.cuda(), "mlp.experts.gate_up_proj": gu, "mlp.experts.down_proj": dn}
    h = hidden.cuda().requires_grad_(True)
    out = moe.moe_feed_forward(h, weights, num_experts=E, top_k=k, norm_topk_prob=True)
    dout = torch.randn(out.shape, generator=g).to(torch.bfloat16).cuda()
    (dh,) = torch.autograd.grad(out, (h,), dout)
    hr = hidden.cuda().requires_grad_(True)
    ref = om.qwen3_moe_loop(hr, gate.cuda(), ops.dequant(gu), ops.dequant(dn), num_experts=E, top_k=k,
                            norm_topk_prob=True)
    (dh_ref,) = torch.autograd.grad(ref, (hr,), dout)
    assert ol.rel_l2(out.detach().cpu(), ref.detach().cpu()) <= BAR
    assert ol.rel_l2(dh.cpu(), dh_ref.cpu()) <= BAR


def test_moe_layer_with_expert_lora_gradients(cuda_lib):
    """Per-expert LoRA on gate_up and down: the A/B gradients through the whole
    layer against autograd of an FP32 per-expert shadow of the same layer."""
    from spilltune_b200 import codec, moe, ops
    T, E, k, H, I, r, s = 128, 8, 2, 256, 128, 8, 2.0
    g = torch.Generator().manual_seed(5)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    gate = (torch.randn(E, H, generator=g) * 0.05).to(torch.bfloat16).cuda()
    gu = codec.encode(torch.randn(E, 2 * I, H, generator=g) * 0.05, "nf4-g128").to("cuda")
    dn = codec.encode(torch.randn(E, H, I, generator=g) * 0.05, "nf4-g128").to("cuda")
    fac = lambda *shp: (torch.randn(*shp, generator=g) * 0.05).cuda().requires_grad_(True)
    A1, B1, A2, B2 = fac(E, r, H), fac(E, 2 * I, r), fac(E, r, I), fac(E, H, r)
    lora = {"gate_up": (A1, B1, s), "down": (A2, B2, s)}
    weights = {"mlp.gate.weight": gate, "mlp.experts.gate_up_proj": gu, "mlp.experts.down_proj": dn}
    out = moe.moe_feed_forward(hidden, weights, num_experts=E, top_k=k, norm_topk_prob=True, lora=lora)
    dout = torch.randn(out.shape, generator=g).to(torch.bfloat16).cuda()
    grads = torch.autograd.grad(out, (A1, B1, A2, B2), dout)
    # FP32 shadow: same routing, per-expert FP32 GEMMs with the LoRA terms.
    W1, W2 = ops.dequant(gu).float(), ops.dequant(dn).float()
    F1, G1, F2, G2 = [t.detach().clone().requires_grad_(True) for t in (A1, B1, A2, B2)]
    routing, idx = moe.qwen3_route(hidden, gate, k, True)
    ref = torch.zeros(T, H, dtype=torch.float32, device="cuda")
    for e in range(E):
        slot_tok = (idx == e).nonzero()
        if slot_tok.numel() == 0:
            continue
        tok, slot = slot_tok[:, 0], slot_tok[:, 1]
        x = hidden[tok].float()
        hcur = x @ W1[e].t() + s * (x @ F1[e].t()) @ G1[e].t()
        ga, up = hcur.chunk(2, dim=-1)
        act = torch.nn.functional.silu(ga) * up
        v = act @ W2[e].t() + s * (act @ F2[e].t()) @ G2[e].t()
        ref = ref.index_add(0, tok, v * routing[tok, slot, None].float())
    rgrads = torch.autograd.grad(ref, (F1, G1, F2, G2), dout.float())
    assert ol.rel_l2(out.float().cpu(), ref.detach().cpu()) <= BAR
    for got, want in zip(grads, rgrads):
        assert ol.rel_l2(got.cpu(), want.cpu()) <= BAR


def test_invalid_segments_reported_not_faulted(cuda_lib):
    from spilltune_b200 import moe
    lengths = [100, 50]
    pw, x, _, _, _ = _grouped_problem(lengths, 256, 256, 0, "nf4-g128", seed=1)
    segs = _segments(lengths)
    segs.seg[-1] = 151  # last offset past the rows: the plan kernel rejects it
    v = ctypes.c_uint32(0)
    assert cuda_lib.fl_status(1, ctypes.byref(v)) == 0
    moe.grouped_fwd(x.cuda(), segs, pw.to("cuda"))
    assert cuda_lib.fl_status(1, ctypes.byref(v)) == 0
    assert v.value & (1 << 4)
    assert cuda_lib.fl_status(0, ctypes.byref(v)) == 0 and v.value == 0
