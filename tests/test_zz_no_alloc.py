"""fl_fwd_noalloc: the forward entry point for callers that cannot allocate
device memory per call (it keeps its scratch in the library's own fixed device
array).  Checked through the C ABI against fl_fwd, which takes caller scratch,
on two calls in a row with different inputs, so a stale scratch would show.

This file is named to be collected last: run alone (fresh process) or after the
other tests, it must pass either way.
"""
import ctypes

import pytest
import torch

import oracle.linear as ol

pytestmark = pytest.mark.gpu

TIGHT = 5e-3  # the same line the parity tests hold


def _case(M, N, K, rank, seed):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(seed)
    pw = codec.encode_nf4(torch.randn(N, K, generator=g) * 0.02).to("cuda")
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    A = (torch.randn(rank, K, generator=g) * 0.05).cuda()
    B = (torch.randn(N, rank, generator=g) * 0.05).cuda()
    return pw, x, A, B


def _fwd_with_workspace(lib, pw, x, A, B, s):
    M, K = x.shape
    N = pw.shape[0]
    rank = A.shape[0]
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ws_bytes = lib.fl_fwd_workspace_bytes(M, K, rank)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    rc = lib.fl_fwd(x.data_ptr(), M, K, pw.payload.data_ptr(), pw.scales.data_ptr(), pw.lut.data_ptr(), N,
                    A.data_ptr(), B.data_ptr(), rank, s, y.data_ptr(), ws.data_ptr(), ws_bytes,
                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.fl_last_error()
    return y


def _fwd_noalloc(lib, pw, x, A, B, s):
    M, K = x.shape
    N = pw.shape[0]
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    rc = lib.fl_fwd_noalloc(x.data_ptr(), M, K, pw.payload.data_ptr(), pw.scales.data_ptr(), pw.lut.data_ptr(),
                            N, A.data_ptr(), B.data_ptr(), A.shape[0], s, y.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.fl_last_error()
    return y


def test_noalloc_matches_workspace_entry_on_two_calls(cuda_lib):
    s = 2.0
    # The last two are decode-step shapes: the small-M kernel with its LoRA partial sums in the scratch.
    for seed, (M, N, K, rank) in ((1, (512, 1024, 4096, 16)), (2, (300, 384, 256, 8)), (3, (16, 4096, 4096, 16)),
                                  (4, (3, 1024, 2048, 8))):
        pw, x, A, B = _case(M, N, K, rank, seed)
        ref = _fwd_with_workspace(cuda_lib, pw, x, A, B, s)
        out = _fwd_noalloc(cuda_lib, pw, x, A, B, s)
        torch.cuda.synchronize()
        assert ol.rel_l2(out.cpu(), ref.cpu()) <= TIGHT
        assert torch.equal(out, ref)  # same kernels, same arithmetic


def test_noalloc_rejects_tokens_beyond_scratch(cuda_lib):
    from spilltune_b200._lib import FL_ERR_ARG
    P = 1024
    rc = cuda_lib.fl_fwd_noalloc(P, 32769, 256, P, P, P, 256, P, P, 16, 2.0, P, None)
    assert rc == FL_ERR_ARG
    assert b"exceeds" in cuda_lib.fl_last_error()


def test_noalloc_left_no_timeouts(cuda_lib):
    v = ctypes.c_uint32(0)
    assert cuda_lib.fl_status(0, ctypes.byref(v)) == 0 and v.value == 0
