"""Host-side view of frozen weight records (the storage format is unchanged).

A frozen projection weight arrives as the reference's group-128 record
(``ram_vram_finetune/quantization/codecs.py``): ``Record(spec, parts)`` with
``spec = {'version':1, 'shape':[N,K], 'dtype':'bfloat16', 'codec':
'int4-sym-g128', 'group_size':128, 'numel':N*K}`` and ``parts = {'payload':
uint8[groups*64], 'scales': float32[groups]}`` (codecs.py:34-43, :105-106).
``PackedWeight`` carries those two parts plus the 16-entry codebook the kernels
decode with.  The NF4 group-128 variant (codec name ``nf4-g128``) shares the
byte layout and uses the NF4 codebook with ``scale = absmax``.

The encoders here are offline host tools (like the reference's ``encode``,
codecs.py:66-116); they are not on the GPU hot path.
"""
from dataclasses import dataclass
import math

import torch

GROUP = 128
INT4_SYM = "int4-sym-g128"
NF4 = "nf4-g128"
CODECS = (INT4_SYM, NF4)

# int4-sym-g128: code c -> c - 8 (codecs.py:62).
INT4_SYM_LUT = torch.arange(16, dtype=torch.float32) - 8.0
# NF4 codebook as published with QLoRA (Dettmers et al., 2023, Appendix E).
NF4_LUT = torch.tensor([
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0], dtype=torch.float32)


def lut_for(codec):
    if codec == INT4_SYM:
        return INT4_SYM_LUT
    if codec == NF4:
        return NF4_LUT
    raise ValueError(f"unsupported_quantization: {codec!r}; supported={CODECS}")


@dataclass
class PackedWeight:
    """One frozen [N, K] matrix, or a stack of E expert matrices [E, N, K]
    (the layout of ``mlp.experts.gate_up_proj`` / ``down_proj``), in group-128
    4-bit form.  Groups run over the flattened row-major tensor, so with
    K % 128 == 0 expert e's groups are a contiguous slice of the record."""
    payload: torch.Tensor  # uint8 [ceil(numel/128)*64]
    scales: torch.Tensor   # float32 [ceil(numel/128)]
    lut: torch.Tensor      # float32 [16]
    shape: tuple           # (N, K) or (E, N, K)
    codec: str = INT4_SYM

    def __post_init__(self):
        self.shape = tuple(int(s) for s in self.shape)
        if len(self.shape) not in (2, 3) or min(self.shape) < 1:
            raise ValueError("invalid stored weight shape")
        numel = math.prod(self.shape)
        groups = (numel + GROUP - 1) // GROUP
        if self.payload.dtype != torch.uint8 or tuple(self.payload.shape) != (groups * 64,):
            raise ValueError("invalid quantized part inventory/shape/dtype: payload")
        if self.scales.dtype != torch.float32 or tuple(self.scales.shape) != (groups,):
            raise ValueError("invalid quantized part inventory/shape/dtype: scales")
        if self.lut.dtype != torch.float32 or tuple(self.lut.shape) != (16,):
            raise ValueError("codebook must be float32[16]")
        if len({self.payload.device, self.scales.device, self.lut.device}) != 1:
            raise ValueError("record parts must live on one device")

    @property
    def out_features(self):
        return self.shape[-2]

    @property
    def in_features(self):
        return self.shape[-1]

    @property
    def experts(self):
        """Number of stacked expert matrices (1 for a plain [N, K] record)."""
        return self.shape[0] if len(self.shape) == 3 else 1

    @property
    def numel(self):
        return math.prod(self.shape)

    @property
    def device(self):
        return self.payload.device

    @property
    def nbytes(self):
        return self.payload.numel() + 4 * self.scales.numel()

    def to(self, device, non_blocking=False):
        return PackedWeight(self.payload.to(device, non_blocking=non_blocking),
                            self.scales.to(device, non_blocking=non_blocking),
                            self.lut.to(device, non_blocking=non_blocking), self.shape, self.codec)

    def pin_memory(self):
        return PackedWeight(self.payload.pin_memory(), self.scales.pin_memory(), self.lut.pin_memory(),
                            self.shape, self.codec)


def from_record(spec, parts):
    """Wrap a reference ``Record`` (spec dict + parts dict) without copying."""
    codec = spec.get("codec")
    if codec not in CODECS:
        raise ValueError(f"unsupported_quantization: {codec!r}; supported={CODECS}")
    if spec.get("group_size") != GROUP or spec.get("dtype") != "bfloat16":
        raise ValueError("invalid quantized storage schema")
    shape = tuple(spec["shape"])
    if len(shape) not in (2, 3) or spec.get("numel") != math.prod(shape):
        raise ValueError("frozen projection records must be 2-D (or 3-D stacked experts) with a matching numel")
    lut = lut_for(codec).to(parts["payload"].device)
    return PackedWeight(parts["payload"], parts["scales"], lut, shape, codec)


def validate(w: PackedWeight, chunk_groups=1 << 20):
    """The value checks of the reference's ``validate_spec`` (quantization/codecs.py:
    119-156), which it runs on every stored record when a slot session is built
    (memory.py:128): scales finite and positive, no reserved int4 code (stored
    nibble 0, the value -8), padding past ``numel`` decoding to zero, and no
    decoded value fp32(lut[c] * scale) overflowing BF16.  Raises ValueError with
    the reference's messages.  Runs where the record lives, in bounded chunks."""
    scales = w.scales
    if not torch.isfinite(scales).all() or (scales <= 0).any():
        raise ValueError("invalid stored scales")
    mag = w.lut.abs()
    limit = mag.max()
    n = w.numel
    for g0 in range(0, scales.numel(), chunk_groups):
        g1 = min(g0 + chunk_groups, scales.numel())
        raw = w.payload[g0 * 64:g1 * 64]
        codes = torch.stack((raw & 15, raw >> 4), 1).view(-1)  # element order
        if w.codec == INT4_SYM and (codes == 0).any():
            raise ValueError("reserved int4 -8 code")
        valid = max(0, min(codes.numel(), n - g0 * GROUP))
        if valid < codes.numel() and (w.lut[codes[valid:].long()] != 0).any():
            raise ValueError("nonzero quantized tail padding")
        sc = scales[g0:g1]
        # Only a group whose largest codebook magnitude overflows can overflow:
        # those get the exact per-code check.
        risky = ~torch.isfinite((limit * sc).to(torch.bfloat16))
        if risky.any():
            top = mag[codes.view(-1, GROUP)[risky].long()].amax(1)
            if not torch.isfinite((top * sc[risky]).to(torch.bfloat16)).all():
                raise ValueError("quantized value overflows BF16 compute range")


def _groups(w):
    flat = w.detach().reshape(-1).to(torch.float32)
    n = flat.numel()
    g = (n + GROUP - 1) // GROUP
    chunk = torch.zeros(g * GROUP, dtype=torch.float32, device=flat.device)
    chunk[:n] = flat
    return chunk.view(g, GROUP), n


def _reject_bf16_overflow(codes, scale, lut):
    """The reference rejects a record any of whose decoded values, fp32(lut[c] * scale)
    rounded to BF16, is not finite (quantization/codecs.py:110-114).  |fp32(a * s)|
    grows with |a|, so each group's largest |lut[c]| over its codes decides it."""
    mag = lut.abs()
    for i in range(0, codes.shape[0], 8192):  # bounded scratch
        top = mag[codes[i:i + 8192].long()].amax(1)
        if not torch.isfinite((top * scale[i:i + 8192]).to(torch.bfloat16)).all():
            raise ValueError("quantized value overflows BF16 compute range")


def encode_int4_sym(w):
    """int4-sym-g128 encoder (same arithmetic as codecs.py:86-105).  Runs on the
    tensor's device (CPU, or a CUDA device for large synthetic models)."""
    chunk, _ = _groups(w)
    if not torch.isfinite(chunk).all():
        raise ValueError("nonfinite quantization input")
    scale = chunk.abs().amax(1) / 7
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = ((chunk / scale[:, None]).clamp(-7, 7).round().to(torch.uint8) + 8)
    lut = INT4_SYM_LUT.to(chunk.device)
    _reject_bf16_overflow(q, scale, lut)
    q = q.flatten().view(-1, 2)
    payload = (q[:, 0] | (q[:, 1] << 4)).contiguous()
    return PackedWeight(payload, scale.contiguous(), lut, tuple(w.shape), INT4_SYM)


def encode_nf4(w, lut=None):
    """NF4 group-128 encoder: scale = group absmax (1 for an all-zero group),
    code = nearest codebook entry to x/scale (first index on ties)."""
    chunk, _ = _groups(w)
    lut = (NF4_LUT if lut is None else lut).to(chunk.device)
    if not torch.isfinite(chunk).all():
        raise ValueError("nonfinite quantization input")
    scale = chunk.abs().amax(1)
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    normalized = chunk / scale[:, None]
    codes = torch.empty_like(normalized, dtype=torch.uint8)
    for i in range(0, normalized.shape[0], 8192):  # bounded scratch
        part = normalized[i:i + 8192]
        codes[i:i + 8192] = (part[..., None] - lut).abs().argmin(-1).to(torch.uint8)
    _reject_bf16_overflow(codes, scale, lut)
    q = codes.flatten().view(-1, 2)
    payload = (q[:, 0] | (q[:, 1] << 4)).contiguous()
    return PackedWeight(payload, scale.contiguous(), lut.clone(), tuple(w.shape), NF4)


def encode(w, codec):
    if codec == INT4_SYM:
        return encode_int4_sym(w)
    if codec == NF4:
        return encode_nf4(w)
    raise ValueError(f"unsupported_quantization: {codec!r}; supported={CODECS}")
