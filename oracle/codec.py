"""ctypes front end of the C codec oracle (``codec_oracle.c``) — test infrastructure.

Restates ``ram_vram_finetune/quantization/codecs.py`` (encode :66-116,
unpack_codes :55-64, decode_into :158-170, validate_spec :119-155) for the
int4-sym-g128 format, plus the NF4 group-128 codebook variant, plus the
bitsandbytes NF4 double-quantized block-64 record the reference's NF4 path
uses (layout validated at quantization/nf4_backend.py:184-278; bitsandbytes
itself is absent, so that decode is a restatement with parity unpinned).
"""
import ctypes
import os
import subprocess

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
GROUP = 128

# NF4 codebook as published in the QLoRA paper (Dettmers et al., 2023,
# Appendix E): asymmetric N(0,1) quantiles normalised to [-1, 1].
NF4_LUT = np.array([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=np.float32)

INT4_SYM_LUT = (np.arange(16, dtype=np.float32) - 8.0)


def nf4_construction():
    """Recompute the NF4 codebook from its published construction (float64)."""
    from scipy.stats import norm
    offset = 0.9677083
    pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1]).tolist()
    neg = (-norm.ppf(np.linspace(offset, 0.5, 8)[:-1])).tolist()
    v = np.array(sorted(pos + [0.0] + neg))
    return v / v.max()


def build():
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                os.path.join(HERE, "codec_oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        L.oracle_decode_g128.argtypes = [p, p, p, i64, p]
        L.oracle_decode_mt.argtypes = [p, p, p, i64, p, ctypes.c_int]
        L.oracle_encode_int4_sym.argtypes = [p, i64, p, p]
        L.oracle_encode_int4_sym.restype = ctypes.c_int
        L.oracle_encode_nf4.argtypes = [p, i64, p, p, p]
        L.oracle_encode_nf4.restype = ctypes.c_int
        L.oracle_validate_int4_sym.argtypes = [p, p, i64]
        L.oracle_validate_int4_sym.restype = ctypes.c_int
        L.oracle_nf4dq_absmax.argtypes = [p, p, p, ctypes.c_float, i64, p]
        L.oracle_nf4dq_decode.argtypes = [p, p, p, i64, p]
        L.oracle_nf4dq_encode.argtypes = [p, i64, p, p, p, p, p, p]
        L.oracle_nf4dq_encode.restype = ctypes.c_float
        L.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def encode_int4_sym(x):
    """int4-sym-g128 encode of a float32 array (any shape, flattened)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    groups = (x.size + GROUP - 1) // GROUP
    payload = np.zeros(groups * 64, np.uint8)
    scales = np.zeros(groups, np.float32)
    rc = lib().oracle_encode_int4_sym(_ptr(x), x.size, _ptr(payload), _ptr(scales))
    if rc == -1:
        raise ValueError("nonfinite quantization input")
    if rc == -2:
        raise ValueError("quantized value overflows BF16 compute range")
    return payload, scales


def encode_nf4(x, lut=NF4_LUT):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    lut = np.ascontiguousarray(lut, dtype=np.float32)
    groups = (x.size + GROUP - 1) // GROUP
    payload = np.zeros(groups * 64, np.uint8)
    scales = np.zeros(groups, np.float32)
    rc = lib().oracle_encode_nf4(_ptr(x), x.size, _ptr(lut), _ptr(payload), _ptr(scales))
    if rc:
        raise ValueError("nonfinite quantization input")
    return payload, scales


def decode(payload, scales, numel, lut=INT4_SYM_LUT, threads=1):
    """decode_into restatement: returns uint16 BF16 bit patterns [numel]."""
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    lut = np.ascontiguousarray(lut, dtype=np.float32)
    out = np.empty(numel, np.uint16)
    if threads > 1:
        lib().oracle_decode_mt(_ptr(payload), _ptr(scales), _ptr(lut), numel, _ptr(out), threads)
    else:
        lib().oracle_decode_g128(_ptr(payload), _ptr(scales), _ptr(lut), numel, _ptr(out))
    return out


def validate_int4_sym(payload, scales, numel):
    payload = np.ascontiguousarray(payload, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    return lib().oracle_validate_int4_sym(_ptr(payload), _ptr(scales), numel)


def bf16_bits_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---------------------------------------------------------------- NF4-DQ64
DQ_BLOCK = 64
DQ_NESTED = 256


def dynamic_map():
    """The 256-entry signed dynamic ("dynamic tree") map that bitsandbytes uses
    as the nested_quant_map of double quantization, rebuilt from its published
    construction (Dettmers et al., 8-bit optimizers via block-wise
    quantization): for each exponent level i = 0..6, the 2**i midpoints of
    2**i + 1 evenly spaced points on [0.1, 1], scaled by 10**(i - 6), with
    both signs; plus 0 and 1; sorted.  Parity with the package is unpinned."""
    vals = [0.0, 1.0]
    for i in range(7):
        pts = np.linspace(0.1, 1.0, 2 ** i + 1, dtype=np.float64)
        mids = (pts[:-1] + pts[1:]) / 2.0 * 10.0 ** (i - 6)
        vals += list(mids) + list(-mids)
    assert len(vals) == 256
    return np.sort(np.array(vals, dtype=np.float32))


def nf4dq_encode(x, quant_map=NF4_LUT, nested_map=None):
    """Test-fixture NF4-DQ64 record of a float array (flattened): returns
    (packed uint8[(n+1)/2], absmax uint8[blocks], nested_absmax fp32, offset)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    quant_map = np.ascontiguousarray(quant_map, dtype=np.float32)
    nested_map = dynamic_map() if nested_map is None else np.ascontiguousarray(nested_map, dtype=np.float32)
    blocks = (x.size + DQ_BLOCK - 1) // DQ_BLOCK
    packed = np.zeros((x.size + 1) // 2, np.uint8)
    absmax_q = np.zeros(blocks, np.uint8)
    nested = np.zeros((blocks + DQ_NESTED - 1) // DQ_NESTED, np.float32)
    tmp = np.zeros(blocks, np.float32)
    offset = lib().oracle_nf4dq_encode(_ptr(x), x.size, _ptr(quant_map), _ptr(nested_map), _ptr(packed),
                                       _ptr(absmax_q), _ptr(nested), _ptr(tmp))
    return packed, absmax_q, nested, float(offset)


def nf4dq_absmax(absmax_q, nested_absmax, nested_map, offset):
    """FP32 block scales of a DQ64 record (the double-quantization prologue)."""
    absmax_q = np.ascontiguousarray(absmax_q, dtype=np.uint8)
    nested_absmax = np.ascontiguousarray(nested_absmax, dtype=np.float32)
    nested_map = np.ascontiguousarray(nested_map, dtype=np.float32)
    out = np.empty(absmax_q.size, np.float32)
    lib().oracle_nf4dq_absmax(_ptr(absmax_q), _ptr(nested_absmax), _ptr(nested_map), float(offset), absmax_q.size,
                              _ptr(out))
    return out


def nf4dq_decode(packed, absmax_f32, numel, quant_map=NF4_LUT):
    """BF16 bit patterns of a DQ64 record given its FP32 block scales."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    absmax_f32 = np.ascontiguousarray(absmax_f32, dtype=np.float32)
    quant_map = np.ascontiguousarray(quant_map, dtype=np.float32)
    out = np.empty(numel, np.uint16)
    lib().oracle_nf4dq_decode(_ptr(packed), _ptr(absmax_f32), _ptr(quant_map), numel, _ptr(out))
    return out


DECODE_CHUNK_GROUPS = 8192  # codecs.py CHUNK_GROUPS: <= 1,048,576 elements per FP32 chunk


def decode_torch(payload, scales, numel, lut, out):
    """The reference's ``decode_into`` (quantization/codecs.py:158-170) as torch
    ops, on whatever device the tensors live on: per chunk of 8192 groups,
    unpack the two codes of every byte (low nibble first, ``unpack_codes``
    :55-64), map them through the 16-entry codebook (``c - 8`` for int4-sym,
    exactly the reference's ``.float() - 8``; the NF4 table for nf4-g128),
    multiply by the group scale in FP32 and round into the BF16 destination.
    ``out`` is a BF16 tensor of ``numel`` elements (any shape, contiguous).
    This is the reference's CPU path when run on the CPU, and its GPU path
    (``SlotSession.load`` decodes on the device, memory.py:224-229) on CUDA."""
    flat = out.view(-1)
    groups = (numel + GROUP - 1) // GROUP
    for g in range(0, groups, DECODE_CHUNK_GROUPS):
        end = min(g + DECODE_CHUNK_GROUPS, groups)
        raw = payload[g * 64:end * 64]
        codes = torch.stack((raw & 15, raw >> 4), 1).flatten().long()
        values = lut[codes].view(-1, GROUP) * scales[g:end, None]
        valid = min(end * GROUP, numel) - g * GROUP
        flat[g * GROUP:g * GROUP + valid].copy_(values.flatten()[:valid])
    return out
