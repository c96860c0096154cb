"""bitsandbytes NF4-DQ64 records (the reference's Qwen3.5 NF4 path).

bitsandbytes is absent here, so the decode rule is pinned only to its own
restatement (oracle/codec_oracle.c) — parity with the package is unpinned.
CPU: the oracle's encode/prologue/decode agree with an independent numpy
evaluation of the stated rule; the host record/metadata checks mirror
nf4_backend.py:188-244.  GPU: the device prologue and dequant are bit-exact
with the oracle; forward/backward within rel-L2 1e-2 (and 5e-3) of the FP32
shadow on the decoded weight.
"""
import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol

BAR, TIGHT = 1e-2, 5e-3


def _record(N, K, seed):
    g = np.random.default_rng(seed)
    w = (g.standard_normal((N, K)) * 0.02).astype(np.float32)
    packed, absmax_q, nested, offset = oc.nf4dq_encode(w)
    return w, packed, absmax_q, nested, offset


def _numpy_decode(packed, absmax_q, nested, offset, numel):
    nmap = oc.dynamic_map()
    scales = (nmap[absmax_q].astype(np.float32) * nested[np.arange(absmax_q.size) // 256]).astype(np.float32)
    scales = (scales + np.float32(offset)).astype(np.float32)
    codes = np.empty(numel, np.int64)
    bytes_ = packed.astype(np.int64)
    codes[0::2] = bytes_[: (numel + 1) // 2] >> 4
    codes[1::2] = bytes_[: numel // 2] & 15
    vals = (oc.NF4_LUT[codes] * scales[np.arange(numel) // 64]).astype(np.float32)
    return scales, vals


@pytest.mark.parametrize("N,K", [(3, 40), (64, 128), (7, 321)])
def test_oracle_rule_matches_numpy(N, K):
    w, packed, absmax_q, nested, offset = _record(N, K, N * K)
    numel = N * K
    scales = oc.nf4dq_absmax(absmax_q, nested, oc.dynamic_map(), offset)
    ref_scales, vals = _numpy_decode(packed, absmax_q, nested, offset, numel)
    assert np.array_equal(scales, ref_scales)
    bits = oc.nf4dq_decode(packed, scales, numel)
    f32 = oc.bf16_bits_to_f32(bits)
    # numpy has no bf16: compare against the rounding of the fp32 products
    rounded = oc.bf16_bits_to_f32(np.array([oc.lib().oracle_f32_to_bf16(float(v)) for v in vals], np.uint16))
    assert np.array_equal(f32, rounded)
    assert np.linalg.norm(f32 - w.reshape(-1)) / np.linalg.norm(w) < 0.15


def test_dynamic_map_shape():
    m = oc.dynamic_map()
    assert m.shape == (256,) and m[0] == -m[-2] and m[-1] == 1.0 and np.all(np.diff(m) > 0)


def test_host_record_checks():
    from spilltune_b200 import nf4dq
    w, packed, absmax_q, nested, offset = _record(8, 128, 1)
    meta = {"quant_type": "nf4", "blocksize": 64, "dtype": "bfloat16", "shape": [8, 128], "nested_blocksize": 256,
            "nested_dtype": "float32", "nested_offset": offset}
    parts = {"absmax": torch.from_numpy(absmax_q), "nested_absmax": torch.from_numpy(nested),
             "nested_quant_map": torch.from_numpy(oc.dynamic_map()), "quant_map": torch.from_numpy(oc.NF4_LUT.copy()),
             nf4dq.QUANT_STATE_KEY: nf4dq.pack_metadata(meta)}
    rec = nf4dq.from_quant_state_parts(torch.from_numpy(packed).reshape(-1, 1), parts)
    assert rec.shape == (8, 128) and rec.numel == 1024 and abs(rec.offset - offset) < 1e-12
    with pytest.raises(ValueError, match="uint8 \\[bytes, 1\\]"):
        nf4dq.from_quant_state_parts(torch.from_numpy(packed), parts)
    bad = dict(meta, blocksize=128)
    with pytest.raises(ValueError, match="blocksize 64"):
        nf4dq.from_quant_state_parts(torch.from_numpy(packed).reshape(-1, 1),
                                     dict(parts, **{nf4dq.QUANT_STATE_KEY: nf4dq.pack_metadata(bad)}))
    with pytest.raises(ValueError, match="byte count"):
        nf4dq.NF4DQRecord(torch.from_numpy(packed[:-1]), parts["absmax"], parts["nested_absmax"],
                          parts["nested_quant_map"], parts["quant_map"], offset, (8, 128))
    with pytest.raises(ValueError, match="CUDA only"):
        nf4dq.stage(rec, "cpu")


def _staged(N, K, seed):
    from spilltune_b200 import nf4dq
    w, packed, absmax_q, nested, offset = _record(N, K, seed)
    rec = nf4dq.NF4DQRecord(torch.from_numpy(packed), torch.from_numpy(absmax_q), torch.from_numpy(nested),
                            torch.from_numpy(oc.dynamic_map()), torch.from_numpy(oc.NF4_LUT.copy()), offset, (N, K))
    scales = oc.nf4dq_absmax(absmax_q, nested, oc.dynamic_map(), offset)
    W = torch.from_numpy(oc.nf4dq_decode(packed, scales, N * K).view(np.int16)).view(torch.bfloat16).view(N, K)
    return rec, scales, W


@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(256, 256), (1000, 384), (7, 4097)])
def test_prologue_and_dequant_bit_exact(cuda_lib, N, K):
    from spilltune_b200 import nf4dq
    rec, scales, W = _staged(N, K, N + K)
    st = nf4dq.stage(rec)
    assert np.array_equal(st.block_scales.cpu().numpy(), scales)
    out = nf4dq.dequant(st).cpu()
    assert torch.equal(out.view(torch.int16), W.view(torch.int16))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,rank", [(256, 256, 256, 0), (300, 384, 512, 16), (16, 1024, 1024, 8),
                                        (3, 640, 384, 4), (2048, 4096, 4096, 16),
                                        (256, 1024, 4096, 16)])  # reduction split: 8 slices fwd, 2 bwd
def test_fwd_bwd_parity(cuda_lib, M, N, K, rank):
    from spilltune_b200 import nf4dq
    rec, _, W = _staged(N, K, M + N)
    st = nf4dq.stage(rec)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    dy = torch.randn(M, N, generator=g).to(torch.bfloat16)
    A = torch.randn(rank, K, generator=g) * 0.05 if rank else None
    B = torch.randn(N, rank, generator=g) * 0.05 if rank else None
    s = 2.0
    cu = lambda t: None if t is None else t.cuda()
    y = nf4dq.fwd(x.cuda(), st, cu(A), cu(B), s).cpu()
    ref = ol.lora_forward_fp32(x, W, A, B, s) if rank else x.float() @ W.float().t()
    assert ol.rel_l2(y, ref) <= TIGHT
    dx, dA, dB = nf4dq.bwd(dy.cuda(), x.cuda(), st, cu(A), cu(B), s)
    if rank:
        rdx, rdA, rdB = ol.lora_backward_fp32(x, W, A, B, s, dy)
        errs = [ol.rel_l2(dx.cpu(), rdx), ol.rel_l2(dA.cpu(), rdA), ol.rel_l2(dB.cpu(), rdB)]
    else:
        errs = [ol.rel_l2(dx.cpu(), dy.float() @ W.float())]
    assert max(errs) <= TIGHT, errs
    if rank:
        # fl_bwd_nf4dq_ts with the forward's Ts: dX bit for bit, dA/dB up to the
        # order of the gradient kernels' atomic adds.
        y2, ts = nf4dq.fwd(x.cuda(), st, cu(A), cu(B), s, return_ts=True)
        assert torch.equal(y2.cpu(), y)
        dx2, dA2, dB2 = nf4dq.bwd(dy.cuda(), x.cuda(), st, cu(A), cu(B), s, ts=ts)
        assert torch.equal(dx2, dx)
        assert ol.rel_l2(dA2.cpu(), dA.cpu()) < 1e-6 and ol.rel_l2(dB2.cpu(), dB.cpu()) < 1e-6


@pytest.mark.gpu
def test_linear_autograd_matches_reference_op_order(cuda_lib):
    """nf4dq_linear + autograd against the reference projection's op order on
    the decoded weight (base bf16 linear, FP32 LoRA, one cast)."""
    from spilltune_b200 import nf4dq
    N, K, M, r, s = 384, 256, 64, 8, 2.0
    rec, _, W = _staged(N, K, 5)
    st = nf4dq.stage(rec)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, M // 2, K, generator=g).to(torch.bfloat16)
    A = torch.randn(r, K, generator=g) * 0.05
    B = torch.randn(N, r, generator=g) * 0.05
    dy = torch.randn(2, M // 2, N, generator=g).to(torch.bfloat16)
    xc, Ac, Bc = x.cuda().requires_grad_(True), A.cuda().requires_grad_(True), B.cuda().requires_grad_(True)
    y = nf4dq.nf4dq_linear(xc, st, Ac, Bc, s)
    gx, gA, gB = torch.autograd.grad(y, (xc, Ac, Bc), dy.cuda())
    xr, Ar, Br = x.clone().requires_grad_(True), A.clone().requires_grad_(True), B.clone().requires_grad_(True)
    yr = ol.lora_forward_reference(xr, W, Ar, Br, s)
    rx, rA, rB = torch.autograd.grad(yr, (xr, Ar, Br), dy)
    assert y.shape == (2, M // 2, N) and y.dtype == torch.bfloat16
    assert ol.rel_l2(y.detach().cpu(), yr.detach()) <= BAR
    for got, want in ((gx, rx), (gA, rA), (gB, rB)):
        assert ol.rel_l2(got.cpu(), want) <= BAR
