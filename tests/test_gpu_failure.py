"""Failure paths on the GPU that fault nothing.

* A bounded device wait runs out: ``fl_wait_selftest`` runs the pipelines' own
  wait code (mbar_wait_warp) with a 1 ms limit on an mbarrier phase nothing
  completes.  The call must return FL_ERR_DEVICE with the timeout status bit
  set, after about the limit (not the 2 s production limit, not a hang), and
  the context must stay usable: a normal fused forward afterwards matches the
  oracle.
* A cross-entropy target outside [0, V) that is not -100 (the reference's
  F.cross_entropy raises for it): the C ABI adds no loss for the row, writes a
  zero gradient row and sets status bit 5; the Python terminal raises before
  launching.
"""
import time

import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol

pytestmark = pytest.mark.gpu


def _decode_cpu(pw):
    bits = oc.decode(pw.payload.cpu().numpy(), pw.scales.cpu().numpy(), pw.numel, lut=pw.lut.cpu().numpy())
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).view(*pw.shape)


def test_bounded_wait_expires_and_context_survives(cuda_lib):
    from spilltune_b200 import _lib, codec, ops
    torch.cuda.synchronize()
    assert _lib.status(reset=True) == 0
    t0 = time.perf_counter()
    rc = cuda_lib.fl_wait_selftest(1_000_000, None)
    dt = time.perf_counter() - t0
    assert rc == _lib.FL_ERR_DEVICE, cuda_lib.fl_last_error()
    assert b"bounded wait expired" in cuda_lib.fl_last_error()
    assert dt < 1.0  # the 1 ms limit, not the 2 s production limit
    st = _lib.status(reset=True)
    assert st & 1  # FL_STATUS_TIMEOUT_FULL
    assert _lib.status() == 0
    # Out-of-range limits are argument errors, checked before any launch.
    assert cuda_lib.fl_wait_selftest(0, None) == _lib.FL_ERR_ARG
    assert cuda_lib.fl_wait_selftest(3_000_000_000, None) == _lib.FL_ERR_ARG

    # The context still runs the fused path correctly.
    g = torch.Generator().manual_seed(5)
    M, N, K, r = 300, 256, 512, 16
    pw = codec.encode(torch.randn(N, K, generator=g) * 0.02, "nf4-g128")
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    A = torch.randn(r, K, generator=g) * 0.05
    B = torch.randn(N, r, generator=g) * 0.05
    y = ops.fwd(x.cuda(), pw.to("cuda"), A.cuda(), B.cuda(), 2.0).cpu()
    ref = ol.lora_forward_fp32(x, _decode_cpu(pw), A, B, 2.0)
    assert ol.rel_l2(y, ref) <= 5e-3
    assert _lib.status() == 0


def test_ce_target_out_of_range_sets_status(cuda_lib):
    from spilltune_b200 import _lib
    from spilltune_b200 import head as hd
    T, H, V = 96, 256, 1000
    g = torch.Generator().manual_seed(11)
    h = torch.randn(T, H, generator=g).to(torch.bfloat16).cuda()
    head = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16).cuda()
    tg = torch.randint(0, V, (T,), generator=g)
    tg[3] = V + 5      # past the vocabulary
    tg[40] = -7        # negative, not the ignore index
    tg[41] = -100      # ignored
    torch.cuda.synchronize()
    assert _lib.status(reset=True) == 0
    loss = torch.zeros((), dtype=torch.float32, device="cuda")
    dh = hd.ce_chunk(h, head, tg.cuda(), 1.0, loss)
    st = _lib.status(reset=True)
    assert st & (1 << 5)
    logits = (h.float() @ head.float().t()).to(torch.bfloat16).float().cpu()
    keep = (tg >= 0) & (tg < V)
    ref = float((torch.logsumexp(logits[keep], -1) - logits[keep, tg[keep]]).sum())
    assert abs(float(loss) - ref) <= 1e-3 * abs(ref)
    dhc = dh.cpu()
    for row in (3, 40, 41):
        assert torch.count_nonzero(dhc[row]) == 0
    assert torch.count_nonzero(dhc[0]) > 0
    # The autograd terminal checks labels on the host and raises like F.cross_entropy.
    labels = torch.randint(0, V, (1, 33), generator=g)
    labels[0, 5] = V
    x = torch.randn(1, 33, H, generator=g).to(torch.bfloat16).cuda().requires_grad_(True)
    with pytest.raises(ValueError, match="out of bounds"):
        hd.chunked_causal_loss(x, head, labels.cuda(), normalization=32.0, token_chunk=16,
                               supervised_chunks=((0, 16), (16, 32)))
