"""MoE host logic and oracle checks that need no GPU.

* the per-expert loop oracle (oracle/moe.py) reproduces the reference's
  Qwen3-MoE ``moe_feed_forward`` output and input gradient stored in
  tests/golden/moe_small.npz;
* the host routers match the reference's (golden vectors);
* expert sorting, gather and combine of spilltune_b200.moe, with the grouped
  kernel call replaced by a torch stand-in on decoded weights, reproduce the
  oracle loop (forward and the hidden-state gradient);
* the grouped C-ABI entry points reject bad arguments before any launch.
"""
import os

import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.moe as om

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bf16(a, shape=None):
    t = torch.from_numpy(np.asarray(a).astype(np.uint16).view(np.int16)).view(torch.bfloat16)
    return t if shape is None else t.reshape(shape)


def _decode(payload, scales, shape):
    n = int(np.prod(shape))
    return _bf16(oc.decode(payload, scales, n), shape)


def _moe_fixture():
    z = np.load(os.path.join(GOLD, "moe_small.npz"))
    E, H, I, T = int(z["E"]), int(z["H"]), int(z["I"]), int(z["T"])
    return dict(
        z=z, E=E, H=H, I=I, T=T, top_k=int(z["top_k"]),
        hidden=_bf16(z["hidden_bf16"], (2, T // 2, H)),
        gate=_bf16(z["gate_bf16"], (E, H)),
        gate_up=_decode(z["gate_up_payload"], z["gate_up_scales"], (E, 2 * I, H)),
        down=_decode(z["down_payload"], z["down_scales"], (E, H, I)),
        out=_bf16(z["out_bf16"], (2, T // 2, H)),
        dout=_bf16(z["dout_bf16"], (2, T // 2, H)),
        dhidden=_bf16(z["dhidden_bf16"], (2, T // 2, H)),
    )


def _rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_loop_oracle_matches_reference_fixture():
    f = _moe_fixture()
    h = f["hidden"].clone().requires_grad_(True)
    out = om.qwen3_moe_loop(h, f["gate"], f["gate_up"], f["down"], num_experts=f["E"], top_k=f["top_k"],
                            norm_topk_prob=True)
    (dh,) = torch.autograd.grad(out, (h,), f["dout"])
    # Same torch ops in the same order on the CPU: equal up to BF16 matmul
    # blocking; the fixture was produced single-threaded.
    assert _rel(out, f["out"]) < 1e-3
    assert _rel(dh, f["dhidden"]) < 1e-3


def test_qwen3_router_matches_reference_fixture():
    from spilltune_b200 import moe
    f = _moe_fixture()
    flat = f["hidden"].reshape(-1, f["H"])
    w, idx = moe.qwen3_route(flat, f["gate"], f["top_k"], True)
    assert w.dtype == torch.bfloat16 and idx.shape == (f["T"], f["top_k"])
    # Expert 5 is never routed in the fixture.
    assert not (idx == 5).any()
    assert torch.allclose(w.float().sum(-1), torch.ones(f["T"]), atol=1e-2)


def test_deepseek_router_matches_reference_fixture():
    from spilltune_b200 import moe
    z = np.load(os.path.join(GOLD, "deepseek_route.npz"))
    flat = _bf16(z["flat_bf16"]).reshape(32, 64)
    w, idx = moe.deepseek_route(flat, torch.from_numpy(z["weight"]), torch.from_numpy(z["bias"]),
                                groups=int(z["groups"]), group_k=int(z["group_k"]), top_k=int(z["top_k"]),
                                normalize=True, scale=float(z["scale"]))
    order = torch.argsort(idx, dim=-1)
    assert np.array_equal(torch.gather(idx, 1, order).numpy(), z["indices"])
    assert np.array_equal(torch.gather(w, 1, order).numpy(), z["weights"])


@pytest.mark.parametrize("T,E,k", [(1, 4, 1), (24, 6, 2), (257, 16, 4), (64, 128, 8)])
def test_expert_segments(T, E, k):
    from spilltune_b200 import moe
    g = torch.Generator().manual_seed(T * 31 + E)
    scores = torch.rand(T, E, generator=g)
    idx = scores.topk(k, dim=-1)[1]
    s = moe.expert_segments(idx, E)
    seg = s.seg.tolist()
    assert seg[0] == 0 and seg[-1] == T * k and all(a <= b for a, b in zip(seg, seg[1:]))
    flat_e = idx.reshape(-1)
    sorted_e = flat_e[s.order]
    for e in range(E):
        assert (sorted_e[seg[e]:seg[e + 1]] == e).all()
        toks = s.token[seg[e]:seg[e + 1]]
        assert (toks[1:] > toks[:-1]).all()          # stable: tokens ascending inside an expert
    assert torch.equal(s.order[s.inverse], torch.arange(T * k))
    assert torch.equal(s.token, s.order // k)


class _TorchGrouped(torch.autograd.Function):
    """Stand-in for the grouped kernel call on decoded weights (CPU)."""

    @staticmethod
    def forward(ctx, xs, A, B, segs, weight, scale):
        W = weight
        seg = segs.seg.tolist()
        ctx.save_for_backward(xs)
        ctx.seg, ctx.W = seg, W
        out = torch.empty(xs.shape[0], W.shape[1], dtype=torch.bfloat16)
        for e in range(W.shape[0]):
            a, b = seg[e], seg[e + 1]
            out[a:b] = (xs[a:b].float() @ W[e].float().t()).to(torch.bfloat16)
        return out

    @staticmethod
    def backward(ctx, dy):
        seg, W = ctx.seg, ctx.W
        dx = torch.empty(dy.shape[0], W.shape[2], dtype=torch.bfloat16)
        for e in range(W.shape[0]):
            a, b = seg[e], seg[e + 1]
            dx[a:b] = (dy[a:b].float() @ W[e].float()).to(torch.bfloat16)
        return dx, None, None, None, None, None


class _DecodedRecord:
    """Just enough of PackedWeight for routed_experts' shape checks."""

    def __init__(self, W):
        self.W = W
        self.experts, self.out_features, self.in_features = W.shape


def test_routed_experts_host_logic_matches_loop(monkeypatch):
    from spilltune_b200 import moe
    f = _moe_fixture()
    monkeypatch.setattr(moe, "grouped_frozen_lora_linear",
                        lambda xs, segs, w, A=None, B=None, scale=0.0: _TorchGrouped.apply(xs, A, B, segs, w.W,
                                                                                           scale))
    h = f["hidden"].clone().requires_grad_(True)
    weights = {"mlp.gate.weight": f["gate"], "mlp.experts.gate_up_proj": _DecodedRecord(f["gate_up"]),
               "mlp.experts.down_proj": _DecodedRecord(f["down"])}
    out = moe.moe_feed_forward(h, weights, num_experts=f["E"], top_k=f["top_k"], norm_topk_prob=True)
    (dh,) = torch.autograd.grad(out, (h,), f["dout"])
    assert out.shape == f["out"].shape and out.dtype == torch.bfloat16
    # FP32-accumulated expert GEMMs and a single-rounding combine vs the
    # reference's BF16 GEMMs and sequential BF16 index_add_.
    assert _rel(out, f["out"]) < 1e-2
    assert _rel(dh, f["dhidden"]) < 1e-2


def test_grouped_abi_rejects_bad_arguments():
    from spilltune_b200 import _lib
    lib = _lib.load()
    # Pointer arguments are dummy addresses: every call is rejected before any
    # pointer is used.
    assert lib.fl_grouped_workspace_bytes(0, 4, 256, 256, 8) == 0
    assert lib.fl_grouped_workspace_bytes(1000, 4, 256, 256, 8) >= 2 * 1000 * 128
    # K not a multiple of 128
    rc = lib.fl_grouped_fwd(16, 16, 100, 200, 4, 16, 16, 16, 256, None, None, 0, 0.0, 16, 16, 1 << 20, None)
    assert rc == _lib.FL_ERR_ARG and b"multiple of 128" in lib.fl_last_error()
    # N not a multiple of 64
    rc = lib.fl_grouped_bwd(16, 16, 16, 100, 96, 256, 4, 16, 16, 16, None, None, 0, 0.0, 16, None, None, 0, 16,
                            1 << 20, None)
    assert rc == _lib.FL_ERR_ARG and b"multiple of 64" in lib.fl_last_error()
    # null segment offsets
    rc = lib.fl_grouped_fwd(16, None, 100, 256, 4, 16, 16, 16, 256, None, None, 0, 0.0, 16, 16, 1 << 20, None)
    assert rc == _lib.FL_ERR_ARG and b"segment" in lib.fl_last_error()
    # rank above the maximum
    rc = lib.fl_grouped_fwd(16, 16, 100, 256, 4, 16, 16, 16, 256, 16, 16, 65, 1.0, 16, 16, 1 << 20, None)
    assert rc == _lib.FL_ERR_UNSUPPORTED
    # short workspace
    rc = lib.fl_grouped_fwd(16, 16, 100, 256, 4, 16, 16, 16, 256, None, None, 0, 0.0, 16, 16, 8, None)
    assert rc == _lib.FL_ERR_ARG and b"workspace" in lib.fl_last_error()


def test_stacked_record_shapes():
    from spilltune_b200 import codec, ops
    w = torch.randn(3, 64, 128) * 0.02
    pw = codec.encode(w, "int4-sym-g128")
    assert pw.shape == (3, 64, 128) and pw.experts == 3
    assert pw.out_features == 64 and pw.in_features == 128 and pw.numel == 3 * 64 * 128
    # Expert e's groups are a contiguous slice of the record.
    one = codec.encode(w[1], "int4-sym-g128")
    assert torch.equal(pw.payload[64 * 64:2 * 64 * 64], one.payload)
    with pytest.raises(ValueError, match="grouped"):
        ops.fwd(torch.zeros(4, 128, dtype=torch.bfloat16), pw)
