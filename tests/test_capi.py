"""The C-ABI library builds for sm_100a, loads, exports every declared entry point
and validates arguments before touching the GPU (runs without a GPU)."""
import ctypes
import os
import re
import shutil

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = []
    for f in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if f.endswith(".h"):
            text = open(os.path.join(ROOT, "include", f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(fl_\w+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from spilltune_b200 import build, _lib
    if not os.path.exists(build.LIB) and not (shutil.which("nvcc") or os.path.exists("/usr/local/cuda/bin/nvcc")):
        pytest.skip("nvcc unavailable and library not prebuilt")
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert "fl_fwd" in names and "fl_bwd" in names and "fl_dequant" in names
    for n in names:
        assert hasattr(lib, n), n


def test_python_binding_covers_header():
    from spilltune_b200 import _lib
    assert set(_declared()) <= set(_lib.SIGNATURES)


def test_version_and_workspace_sizes(lib):
    assert lib.fl_version() >= 200  # 0.2.0 adds fl_bwd_ts and fl_bwd_nf4dq_ts
    # Ts (M x 64 bf16) + the factor converted to a bf16 hi/lo pair (4 * rank' * K) and its
    # per-64-unit masks (4 * K / 64 bytes, padded to 16).
    mask = lambda R: (R // 64 * 4 + 15) // 16 * 16
    assert lib.fl_fwd_workspace_bytes(8192, 4096, 16) == 8192 * 128 + 4 * 16 * 4096 + mask(4096)
    assert lib.fl_fwd_workspace_bytes(8192, 4096, 20) == 8192 * 128 + 4 * 32 * 4096 + mask(4096)
    assert lib.fl_fwd_workspace_bytes(8192, 4096, 0) == 0
    assert lib.fl_bwd_workspace_bytes(100, 384, 256, 8) == 100 * 256 + 4 * 16 * (384 + 256) + mask(384) + mask(256)


def test_split_workspace_sizes(lib):
    """Room for the FP32 partial sums only when the output has too few 256 x 256 tiles for
    the 74 CTA pairs of a B200 (the count the query assumes without a device, too)."""
    a256 = lambda b: (b + 255) // 256 * 256
    fwd, fwd_s = lib.fl_fwd_workspace_bytes, lib.fl_fwd_workspace_bytes_split
    bwd, bwd_s = lib.fl_bwd_workspace_bytes, lib.fl_bwd_workspace_bytes_split
    # Enough tiles, or the decode-step kernels: no split.
    assert fwd_s(8192, 14336, 4096, 16) == fwd(8192, 4096, 16)
    assert fwd_s(16, 4096, 4096, 16) == fwd(16, 4096, 16)
    assert bwd_s(8192, 14336, 4096, 16) == bwd(8192, 14336, 4096, 16)
    # 256 tokens of a 4096-wide projection: 16 tiles x 4 slices of 16 stages.
    assert fwd_s(256, 4096, 4096, 16) == a256(fwd(256, 4096, 16)) + 4 * 256 * 4096 * 4
    assert fwd_s(256, 4096, 14336, 0) == 4 * 256 * 4096 * 4
    # 4 tiles: 8 slices (each keeps 8 stages of 64).
    assert fwd_s(256, 1024, 4096, 0) == 8 * 256 * 1024 * 4
    # Backward: dX [M, K] tiles, reduction over N.
    assert bwd_s(256, 14336, 4096, 16) == a256(bwd(256, 14336, 4096, 16)) + 4 * 256 * 4096 * 4
    assert bwd_s(2048, 1024, 4096, 0) == bwd(2048, 1024, 4096, 0)  # 16 x 8 = 128 dX tiles: no split
    assert fwd_s(2048, 1024, 4096, 0) == 2 * 2048 * 1024 * 4  # 4 x 8 = 32 Y tiles: 2 slices


def _fwd(lib, M=16, K=256, N=128, rank=0, ptr=1024, ws=0):
    P = ptr
    return lib.fl_fwd(P, M, K, P, P, P, N, P if rank else None, P if rank else None, rank, 2.0, P,
                      P if ws else None, ws, None)


def test_argument_validation_without_gpu(lib):
    from spilltune_b200._lib import FL_ERR_ARG, FL_ERR_UNSUPPORTED
    assert _fwd(lib, K=100) == FL_ERR_ARG
    assert b"multiple of 128" in lib.fl_last_error()
    assert _fwd(lib, rank=65) == FL_ERR_UNSUPPORTED
    assert _fwd(lib, rank=16, ws=0) == FL_ERR_ARG
    assert _fwd(lib, ptr=1032) == FL_ERR_ARG  # misaligned payload
    assert lib.fl_dequant(None, None, None, 10, None, None) == FL_ERR_ARG
    assert lib.fl_dequant(None, None, None, 0, None, None) == 0
    P = 1024
    rc = lib.fl_bwd(P, P, 16, 100, 256, P, P, P, None, None, 0, 1.0, P, None, None, 0, None, 0, None)
    assert rc == FL_ERR_ARG and b"multiple of 64" in lib.fl_last_error()
    # fl_bwd_ts: the forward's Ts must be 16-byte aligned (checked before any device work).
    ws = lib.fl_bwd_workspace_bytes(300, 256, 256, 8)
    rc = lib.fl_bwd_ts(P, P, 300, 256, 256, P, P, P, P, P, 8, 1.0, P + 8, P, P, P, 0, P, ws, None)
    assert rc == FL_ERR_ARG and b"Ts must be 16-byte aligned" in lib.fl_last_error()


def test_ops_reject_cpu_tensors():
    from spilltune_b200 import codec, ops
    w = codec.encode_int4_sym(torch.randn(128, 256) * 0.02)
    x = torch.randn(4, 256).to(torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU fallback"):
        ops.fwd(x, w)
