"""ctypes front end of the C codec oracle (``codec_oracle.c``) — test infrastructure.

Restates ``ram_vram_finetune/quantization/codecs.py`` (encode :66-116,
unpack_codes :55-64, decode_into :158-170, validate_spec :119-155) for the
int4-sym-g128 format, plus the NF4 group-128 codebook variant.
"""
import ctypes
import os
import subprocess

import numpy as np

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
