"""Consecutive library calls on one stream, with no synchronisation between them.

The kernels inside one fl_fwd / fl_bwd_ts call overlap each other (programmatic
dependent launch); each call's first launch is an ordinary one.  So a call must
see everything the calls before it wrote: an output fed straight into the next
call as its input, and a workspace and gradient buffers reused by the next call.
Checked by running the same sequence twice, once with a device synchronise after
every call, and comparing every result.
"""
import pytest
import torch

import oracle.linear as ol

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _fwd(lib, x, pw, A, B, s, y, ws):
    M, K = x.shape
    rc = lib.fl_fwd(x.data_ptr(), M, K, pw.payload.data_ptr(), pw.scales.data_ptr(), pw.lut.data_ptr(), pw.shape[0],
                    A.data_ptr(), B.data_ptr(), A.shape[0], s, y.data_ptr(), ws.data_ptr(), ws.numel(), _stream())
    assert rc == 0, lib.fl_last_error()


def _bwd_ts(lib, dy, x, pw, A, B, s, ts_ptr, dx, dA, dB, accumulate, ws):
    M, K = x.shape
    N = pw.shape[0]
    rc = lib.fl_bwd_ts(dy.data_ptr(), x.data_ptr(), M, N, K, pw.payload.data_ptr(), pw.scales.data_ptr(),
                       pw.lut.data_ptr(), A.data_ptr(), B.data_ptr(), A.shape[0], s, ts_ptr, dx.data_ptr(),
                       dA.data_ptr(), dB.data_ptr(), int(accumulate), ws.data_ptr(), ws.numel(), _stream())
    assert rc == 0, lib.fl_last_error()


def _sequence(lib, sync, pw1, pw2, x, dy1, dy2, A1, B1, A2, B2, s):
    """y = f1(x), z = f2(y), the backward of f2 (its dX is f1's upstream gradient), f1
    recomputed into the shared forward workspace, then two backward calls of f1 into
    one set of gradient buffers (the second accumulating)."""
    M, K = x.shape
    N1, N2 = pw1.shape[0], pw2.shape[0]
    rank = A1.shape[0]
    dev = x.device
    ws_f = torch.empty(lib.fl_fwd_workspace_bytes(M, max(K, N1), rank), dtype=torch.uint8, device=dev)
    ws_b = torch.empty(lib.fl_bwd_workspace_bytes(M, max(N1, N2), max(K, N1), rank), dtype=torch.uint8,
                       device=dev)
    y = torch.empty(M, N1, dtype=torch.bfloat16, device=dev)
    z = torch.empty(M, N2, dtype=torch.bfloat16, device=dev)
    dA = torch.empty(rank, K, dtype=torch.float32, device=dev)
    dB = torch.empty(N1, rank, dtype=torch.float32, device=dev)
    step = torch.cuda.synchronize if sync else (lambda: None)
    ts = ws_f.data_ptr()  # fl_fwd leaves Ts at the start of its workspace
    _fwd(lib, x, pw1, A1, B1, s, y, ws_f)                 # y = f1(x)
    step()
    _fwd(lib, y, pw2, A2, B2, s, z, ws_f)                 # z = f2(y): reads the previous call's output
    step()
    # Backward of f2 writes dY1 = dz . W2 + ..., which the backward of f1 reads.
    dy_1 = torch.empty(M, N1, dtype=torch.bfloat16, device=dev)
    dA2 = torch.empty_like(A2)
    dB2 = torch.empty_like(B2)
    _bwd_ts(lib, dy2, y, pw2, A2, B2, s, ts, dy_1, dA2, dB2, 0, ws_b)
    step()
    # Recompute f1 (its Ts overwrites the shared forward workspace), then its backward
    # twice into the same gradient buffers: the second call accumulates.
    _fwd(lib, x, pw1, A1, B1, s, y, ws_f)
    step()
    dx1 = torch.empty(M, K, dtype=torch.bfloat16, device=dev)
    _bwd_ts(lib, dy_1, x, pw1, A1, B1, s, ts, dx1, dA, dB, 0, ws_b)
    step()
    _bwd_ts(lib, dy1, x, pw1, A1, B1, s, ts, dx1, dA, dB, 1, ws_b)
    step()
    torch.cuda.synchronize()
    return [t.clone() for t in (y, z, dy_1, dA2, dB2, dx1, dA, dB)]


def test_consecutive_calls_see_each_others_results(cuda_lib):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(77)
    M, K, N1, N2, r, s = 1024, 2048, 1024, 512, 16, 2.0
    pw1 = codec.encode_nf4(torch.randn(N1, K, generator=g) * 0.02).to("cuda")
    pw2 = codec.encode_nf4(torch.randn(N2, N1, generator=g) * 0.02).to("cuda")
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    dy1 = torch.randn(M, N1, generator=g).to(torch.bfloat16).cuda()
    dy2 = torch.randn(M, N2, generator=g).to(torch.bfloat16).cuda()
    A1 = (torch.randn(r, K, generator=g) * 0.05).cuda()
    B1 = (torch.randn(N1, r, generator=g) * 0.05).cuda()
    A2 = (torch.randn(r, N1, generator=g) * 0.05).cuda()
    B2 = (torch.randn(N2, r, generator=g) * 0.05).cuda()
    args = (pw1, pw2, x, dy1, dy2, A1, B1, A2, B2, s)
    ref = _sequence(cuda_lib, True, *args)
    out = _sequence(cuda_lib, False, *args)
    names = ("y", "z", "dY1", "dA2", "dB2", "dX", "dA", "dB")
    for name, a, b in zip(names, out, ref):
        if a.dtype == torch.bfloat16:
            assert torch.equal(a, b), name  # deterministic kernels
        else:
            # fp32 gradients: equal up to the order of the gradient kernels' atomic adds
            assert ol.rel_l2(a.cpu(), b.cpu()) < 1e-6, name
