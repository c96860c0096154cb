"""GPU parity of the CUDA path (through the C ABI) against the CPU oracle.

Bars (the project's correctness requirements):
  * dequantized weights bit-exact with decode_into;
  * Y, dX, dA, dB within rel-L2 <= 1e-2 of the FP32 reference
    (oracle.linear.*_fp32 on the oracle-decoded weight).  The tests also hold a
    tighter 5e-3 line: the kernels accumulate in fp32, so only the bf16 output
    rounding and the bf16 low-rank operands separate them from the FP32 shadow.
At the kernel sweep's full sizes the CPU cannot run the whole product, so the
check samples token rows (the oracle computes those rows exactly) and checks
row independence of the GPU result.
"""
import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol

pytestmark = pytest.mark.gpu

BAR = 1e-2
TIGHT = 5e-3


def _decode_cpu(pw):
    bits = oc.decode(pw.payload.cpu().numpy(), pw.scales.cpu().numpy(), pw.numel, lut=pw.lut.cpu().numpy())
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).view(*pw.shape)


def _problem(M, N, K, rank, codec_name, seed=0, wstd=0.02, fstd=0.05):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(N, K, generator=g) * wstd
    pw = codec.encode(w, codec_name)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    A = torch.randn(rank, K, generator=g) * fstd if rank else None
    B = torch.randn(N, rank, generator=g) * fstd if rank else None
    dy = torch.randn(M, N, generator=g).to(torch.bfloat16)
    return pw, x, A, B, dy


def _cuda(t):
    return None if t is None else t.cuda()


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("numel", [1, 128, 129, 257, 4096 * 130 + 77, 4096 * 4096])
def test_dequant_bit_exact(cuda_lib, codec_name, numel):
    from spilltune_b200 import codec, ops
    g = torch.Generator().manual_seed(numel % 9973)
    w = torch.randn(1, numel, generator=g) * 0.02
    pw = codec.encode(w, codec_name)
    out = ops.dequant(pw.to("cuda")).cpu()
    ref = oc.decode(pw.payload.numpy(), pw.scales.numpy(), numel, lut=pw.lut.numpy())
    assert np.array_equal(out.view(torch.int16).numpy().reshape(-1).view(np.uint16), ref)


def test_dequant_matches_reference_golden(cuda_lib):
    from spilltune_b200 import codec, ops
    d = np.load("tests/golden/codec_int4.npz")
    for name in ("kat", "len129", "len257", "mat32x256"):
        n = d[name + "/input"].size
        pw = codec.PackedWeight(torch.from_numpy(d[name + "/payload"]), torch.from_numpy(d[name + "/scales"]),
                                codec.INT4_SYM_LUT, (1, n))
        out = ops.dequant(pw.to("cuda")).cpu().view(torch.int16).numpy().reshape(-1).view(np.uint16)
        assert np.array_equal(out, d[name + "/decoded_bf16"]), name


FWD_CASES = [
    # M, N, K, rank
    (256, 128, 128, 0),
    (256, 128, 256, 16),
    (300, 384, 256, 8),     # ragged token tile
    (17, 200, 384, 16),     # ragged weight-row tile, tiny M
    (1, 256, 512, 16),
    (512, 1024, 4096, 16),
    (640, 256, 1024, 64),
    (256, 512, 768, 32),
]


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("M,N,K,rank", FWD_CASES)
def test_fwd_parity(cuda_lib, codec_name, M, N, K, rank):
    from spilltune_b200 import ops
    pw, x, A, B, _ = _problem(M, N, K, rank, codec_name, seed=M * 7 + N)
    s = 2.0
    y = ops.fwd(x.cuda(), pw.to("cuda"), _cuda(A), _cuda(B), s).cpu()
    W = _decode_cpu(pw)
    if rank:
        ref = ol.lora_forward_fp32(x, W, A, B, s)
    else:
        ref = x.float() @ W.float().t()
    err = ol.rel_l2(y, ref)
    assert err <= BAR and err <= TIGHT, err


BWD_CASES = [
    (256, 128, 128, 0),
    (256, 128, 256, 16),
    (300, 384, 256, 8),
    (18, 384, 256, 8),
    (512, 1024, 4096, 16),
    (256, 512, 768, 64),
]


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("M,N,K,rank", BWD_CASES)
def test_bwd_parity(cuda_lib, codec_name, M, N, K, rank):
    from spilltune_b200 import ops
    pw, x, A, B, dy = _problem(M, N, K, rank, codec_name, seed=M * 3 + K)
    s = 2.0
    dx, dA, dB = ops.bwd(dy.cuda(), x.cuda(), pw.to("cuda"), _cuda(A), _cuda(B), s)
    W = _decode_cpu(pw)
    if rank:
        rdx, rdA, rdB = ol.lora_backward_fp32(x, W, A, B, s, dy)
        e = (ol.rel_l2(dx.cpu(), rdx), ol.rel_l2(dA.cpu(), rdA), ol.rel_l2(dB.cpu(), rdB))
    else:
        e = (ol.rel_l2(dx.cpu(), dy.float() @ W.float()),)
    assert max(e) <= BAR and max(e) <= TIGHT, e


SMALLM_BWD_CASES = [
    # M, N, K, rank
    (1, 4096, 4096, 16),
    (16, 14336, 4096, 16),   # reduction over 224 chunks of 64 rows, 2-CTA clusters
    (16, 4096, 14336, 64),   # 112 column blocks, rank 64
    (7, 1024, 4096, 0),      # plain frozen VJP, 8-CTA clusters
    (9, 64, 512, 0),         # one chunk, four column blocks
    (9, 128, 512, 8),        # two chunks, LoRA (its reduction over N needs N % 128 == 0)
    (13, 256, 1024, 32),     # four chunks over a cluster
]


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("M,N,K,rank", SMALLM_BWD_CASES)
def test_small_m_bwd_parity(cuda_lib, codec_name, M, N, K, rank):
    """M <= 16 with K % 512 == 0 runs the decode-step backward (scale folded into bf16(dY * scale),
    transposed byte-table decode); dA and dB stay on the low-rank kernels."""
    from spilltune_b200 import ops
    pw, x, A, B, dy = _problem(M, N, K, rank, codec_name, seed=M * 5 + N + K)
    s = 2.0
    dx, dA, dB = ops.bwd(dy.cuda(), x.cuda(), pw.to("cuda"), _cuda(A), _cuda(B), s)
    W = _decode_cpu(pw)
    if rank:
        rdx, rdA, rdB = ol.lora_backward_fp32(x, W, A, B, s, dy)
        e = (ol.rel_l2(dx.cpu(), rdx), ol.rel_l2(dA.cpu(), rdA), ol.rel_l2(dB.cpu(), rdB))
    else:
        e = (ol.rel_l2(dx.cpu(), dy.float() @ W.float()),)
    assert max(e) <= BAR and max(e) <= TIGHT, e


def test_bwd_accumulate(cuda_lib):
    from spilltune_b200 import ops
    pw, x, A, B, dy = _problem(256, 256, 256, 16, "int4-sym-g128", seed=5)
    pw, x, A, B, dy = pw.to("cuda"), x.cuda(), A.cuda(), B.cuda(), dy.cuda()
    _, dA1, dB1 = ops.bwd(dy, x, pw, A, B, 2.0)
    dA, dB = dA1.clone(), dB1.clone()
    ops.bwd(dy, x, pw, A, B, 2.0, dA=dA, dB=dB, accumulate=True)
    assert ol.rel_l2(dA.cpu(), 2 * dA1.cpu()) < 1e-6 and ol.rel_l2(dB.cpu(), 2 * dB1.cpu()) < 1e-6
    ops.bwd(dy, x, pw, A, B, 2.0, dA=dA, dB=dB, accumulate=False)
    assert ol.rel_l2(dA.cpu(), dA1.cpu()) < 1e-6


@pytest.mark.parametrize("M,N,K,rank", [(512, 1024, 4096, 16), (300, 384, 256, 8), (3, 640, 384, 4),
                                         (16, 512, 1024, 16)])
def test_bwd_with_forward_ts_matches_bwd(cuda_lib, M, N, K, rank):
    """fl_bwd_ts given the forward's Ts gives fl_bwd's results: dX bit for bit, dA
    and dB up to the order of the gradient kernels' atomic adds.  The last shape
    takes the decode-step kernels, where the forward keeps no Ts."""
    from spilltune_b200 import ops
    s = 2.0
    pw, x, A, B, dy = _problem(M, N, K, rank, "nf4-g128", seed=21)
    pw, x, A, B, dy = pw.to("cuda"), x.cuda(), A.cuda(), B.cuda(), dy.cuda()
    y, ts = ops.fwd(x, pw, A, B, s, return_ts=True)
    assert torch.equal(y, ops.fwd(x, pw, A, B, s))
    if M <= 16 and K % 512 == 0:
        assert ts is None
    else:
        # Ts = bf16(s * x . A^T) against FP32 (one bf16 rounding), zero past the rank.
        ref = s * x.float().cpu() @ A.cpu().t()
        assert ol.rel_l2(ts[:, :rank].float().cpu(), ref) <= TIGHT
        assert int(ts[:, rank:].count_nonzero()) == 0
    dx0, dA0, dB0 = ops.bwd(dy, x, pw, A, B, s)
    dx1, dA1, dB1 = ops.bwd(dy, x, pw, A, B, s, ts=ts)
    torch.cuda.synchronize()
    assert torch.equal(dx0, dx1)
    assert ol.rel_l2(dA1.cpu(), dA0.cpu()) < 1e-6 and ol.rel_l2(dB1.cpu(), dB0.cpu()) < 1e-6


def test_reference_golden_through_cuda_path(cuda_lib):
    """LoRAProjection.forward + autograd produced by the reference itself."""
    from spilltune_b200 import codec, ops
    g = np.load("tests/golden/lora_small.npz")
    M, K, N, r, alpha = [g[k].item() for k in ("M", "K", "N", "rank", "alpha")]
    bf = lambda a, shp: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).view(*shp)
    pw = codec.PackedWeight(torch.from_numpy(g["payload"]), torch.from_numpy(g["scales"]), codec.INT4_SYM_LUT,
                            (N, K)).to("cuda")
    x = bf(g["x_bf16"], (M, K)).cuda().requires_grad_(True)
    A = torch.from_numpy(g["A"]).cuda().requires_grad_(True)
    B = torch.from_numpy(g["B"]).cuda().requires_grad_(True)
    dY = bf(g["dY_bf16"], (M, N)).cuda()
    y = ops.frozen_lora_linear(x, pw, A, B, alpha / r)
    dx, dA, dB = torch.autograd.grad(y, (x, A, B), dY)
    assert ol.rel_l2(y.detach().cpu(), bf(g["Y_bf16"], (M, N))) <= BAR
    assert ol.rel_l2(dx.cpu(), bf(g["dX_bf16"], (M, K))) <= BAR
    assert ol.rel_l2(dA.cpu(), torch.from_numpy(g["dA"])) <= BAR
    assert ol.rel_l2(dB.cpu(), torch.from_numpy(g["dB"])) <= BAR


@pytest.mark.parametrize("N,K", [(4096, 4096), (1024, 4096), (14336, 4096), (4096, 14336)])
def test_full_size_sampled_rows(cuda_lib, N, K):
    """Kernel-sweep shapes at M=2048: oracle-exact rows + row independence."""
    from spilltune_b200 import ops
    M, rank, s = 2048, 16, 2.0
    pw, x, A, B, dy = _problem(M, N, K, rank, "nf4-g128", seed=N + K, fstd=0.01)
    pwc, xc, Ac, Bc, dyc = pw.to("cuda"), x.cuda(), A.cuda(), B.cuda(), dy.cuda()
    y = ops.fwd(xc, pwc, Ac, Bc, s)
    dx, dA, dB = ops.bwd(dyc, xc, pwc, Ac, Bc, s)
    W = _decode_cpu(pw)
    rows = torch.tensor([0, 1, 255, 256, 1023, 1500, 2046, 2047])
    ref_y = ol.lora_forward_fp32(x[rows], W, A, B, s)
    assert ol.rel_l2(y[rows.cuda()].cpu(), ref_y) <= TIGHT
    ref_dx, _, _ = ol.lora_backward_fp32(x[rows], W, A, B, s, dy[rows])
    assert ol.rel_l2(dx[rows.cuda()].cpu(), ref_dx) <= TIGHT
    # dA, dB reduce over all tokens: fp32 shadow on the CPU is cheap (rank 16).
    xf, gf = x.float(), dy.float()
    rdA = s * (gf @ B).t() @ xf
    rdB = s * gf.t() @ (xf @ A.t())
    assert ol.rel_l2(dA.cpu(), rdA) <= TIGHT and ol.rel_l2(dB.cpu(), rdB) <= TIGHT
    # Row independence: a 256-token slice through the kernel equals the same rows of the full
    # call (both without a split of the reduction, whose slice count depends on the token count).
    y1 = ops.fwd(xc, pwc, Ac, Bc, s, split_reduction=False)
    y_slice = ops.fwd(xc[256:512].contiguous(), pwc, Ac, Bc, s, split_reduction=False)
    assert torch.equal(y_slice, y1[256:512])
    # A split changes only the order of the FP32 sums.
    assert ol.rel_l2(y.cpu(), y1.cpu()) <= 1e-3


# Calls whose output has too few 256 x 256 tiles for the GPU's CTA pairs: the
# forward splits its reduction over K, the backward dX's over N (slices at rank
# 16 on a B200: fwd 4 / bwd 4; fwd 8; fwd 4; bwd 4; fwd 4 with ragged token and
# output tiles; fwd 4 beside a wider low-rank grid; fwd 2 and bwd 2 with slices
# long enough to use every pair; bwd 2 for DeepSeek-V3's kv_b_proj at 4096 tokens).
SPLIT_CASES = [(256, 4096, 4096), (256, 1024, 4096), (256, 4096, 14336), (256, 14336, 4096), (300, 384, 2048),
               (512, 1024, 4096), (512, 4096, 14336), (512, 14336, 4096), (4096, 32768, 512)]


@pytest.mark.parametrize("M,N,K", SPLIT_CASES)
def test_split_reduction_parity(cuda_lib, M, N, K):
    """Split calls against the FP32 shadow on sampled rows (forward, and the backward from
    the forward's Ts), and against the same call without a split: only the order of the
    FP32 sums differs, so the bf16 outputs agree to within a rounding step."""
    from spilltune_b200 import ops
    lib = cuda_lib
    rank, s = 16, 2.0
    assert (lib.fl_fwd_workspace_bytes_split(M, N, K, rank) > lib.fl_fwd_workspace_bytes(M, K, rank)
            or lib.fl_bwd_workspace_bytes_split(M, N, K, rank) > lib.fl_bwd_workspace_bytes(M, N, K, rank))
    pw, x, A, B, dy = _problem(M, N, K, rank, "nf4-g128", seed=M + N + 3 * K, fstd=0.01)
    pwc, xc, Ac, Bc, dyc = pw.to("cuda"), x.cuda(), A.cuda(), B.cuda(), dy.cuda()
    y, ts = ops.fwd(xc, pwc, Ac, Bc, s, return_ts=True)
    dx, dA, dB = ops.bwd(dyc, xc, pwc, Ac, Bc, s, ts=ts)
    y1 = ops.fwd(xc, pwc, Ac, Bc, s, split_reduction=False)
    dx1, dA1, dB1 = ops.bwd(dyc, xc, pwc, Ac, Bc, s, split_reduction=False)
    torch.cuda.synchronize()
    W = _decode_cpu(pw)
    rows = torch.tensor(sorted({0, 1, 127, 128, 255, M // 2, M - 1}))
    assert ol.rel_l2(y[rows.cuda()].cpu(), ol.lora_forward_fp32(x[rows], W, A, B, s)) <= TIGHT
    ref_dx, _, _ = ol.lora_backward_fp32(x[rows], W, A, B, s, dy[rows])
    assert ol.rel_l2(dx[rows.cuda()].cpu(), ref_dx) <= TIGHT
    xf, gf = x.float(), dy.float()
    assert ol.rel_l2(dA.cpu(), s * (gf @ B).t() @ xf) <= TIGHT
    assert ol.rel_l2(dB.cpu(), s * gf.t() @ (xf @ A.t())) <= TIGHT
    assert ol.rel_l2(y.cpu(), y1.cpu()) <= 1e-3 and ol.rel_l2(dx.cpu(), dx1.cpu()) <= 1e-3
    assert ol.rel_l2(dA.cpu(), dA1.cpu()) < 1e-5 and ol.rel_l2(dB.cpu(), dB1.cpu()) < 1e-5
    # Same inputs, same split: the same bits (fixed order of the partial sums).
    assert torch.equal(ops.fwd(xc, pwc, Ac, Bc, s), y)


def test_no_kernel_reported_timeouts(cuda_lib):
    import ctypes
    v = ctypes.c_uint32(0)
    assert cuda_lib.fl_status(0, ctypes.byref(v)) == 0
    assert v.value == 0


def test_backward_from_a_fresh_thread(cuda_lib):
    """torch runs CUDA backward on its autograd worker thread; the ops must not
    depend on a CUDA context already being current there."""
    import threading
    from spilltune_b200 import ops
    pw, x, A, B, dy = _problem(256, 256, 256, 16, "nf4-g128", seed=9)
    pw, x, A, B, dy = pw.to("cuda"), x.cuda(), A.cuda(), B.cuda(), dy.cuda()
    ref = ops.bwd(dy, x, pw, A, B, 2.0)
    torch.cuda.synchronize()
    out = {}

    def work():
        out["r"] = ops.bwd(dy, x, pw, A, B, 2.0)
        torch.cuda.synchronize()

    t = threading.Thread(target=work)
    t.start()
    t.join()
    for a, b in zip(out["r"], ref):
        assert ol.rel_l2(a.cpu(), b.cpu()) < 1e-6


SMALLM_CASES = [
    # M, N, K, rank
    (1, 4096, 4096, 16),
    (5, 1024, 4096, 0),
    (8, 384, 256, 8),
    (16, 14336, 4096, 16),
    (16, 4096, 14336, 16),
    (13, 200, 512, 64),      # ragged rows and tokens
    (16, 1024, 1024, 8),     # reduction split over a 2-CTA cluster
    (3, 1000, 2048, 32),     # row count not a multiple of 32
    (16, 8192, 512, 16),     # one 512-wide chunk per CTA
    (9, 4096, 14336, 64),    # 28 chunks through the slot ring, rank 64
    (7, 640, 384, 16),       # K % 512 != 0: the tile GEMM
    (16, 8, 128, 4),         # one group, 8 valid rows (tile GEMM)
    (2, 29568, 4096, 0),     # 924 row blocks: no split
    # <= 8 tokens with >= 4 chunks per CTA: 128-row CTAs with the byte-permute table
    (4, 14300, 4096, 8),     # last row block ragged
    (1, 4096, 14336, 16),    # reduction split over a 4-CTA cluster (7 chunks each)
    (6, 6144, 4096, 64),     # 2-CTA cluster, rank 64
]


@pytest.mark.parametrize("codec_name", ["int4-sym-g128", "nf4-g128"])
@pytest.mark.parametrize("M,N,K,rank", SMALLM_CASES)
def test_small_m_fwd_parity(cuda_lib, codec_name, M, N, K, rank):
    """M <= 16 with K % 512 == 0 runs the decode-step kernel (operand bf16(lut), scale on each
    group's partial sum, LoRA term added in FP32 from the bf16 Ts of the small-M low-rank kernel);
    other K take the tile GEMM."""
    from spilltune_b200 import ops
    pw, x, A, B, _ = _problem(M, N, K, rank, codec_name, seed=M * 11 + N + K)
    s = 2.0
    y = ops.fwd(x.cuda(), pw.to("cuda"), _cuda(A), _cuda(B), s).cpu()
    W = _decode_cpu(pw)
    ref = ol.lora_forward_fp32(x, W, A, B, s) if rank else x.float() @ W.float().t()
    err = ol.rel_l2(y, ref)
    assert err <= BAR and err <= TIGHT, err
