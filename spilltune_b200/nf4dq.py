"""bitsandbytes NF4 double-quantized (block 64) records on the fused kernels.

The reference's Qwen3.5 NF4 path stores every frozen projection as the
record bitsandbytes' ``quantize_4bit(..., blocksize=64, compress_statistics=True,
quant_type="nf4", quant_storage=uint8)`` produces, validates it
(ram_vram_finetune/quantization/nf4_backend.py:184-278), stages its six parts
to the GPU (``stage_cuda`` / ``CUDARecord``, nf4_backend_cuda.py:522-644,
747-837) and multiplies with ``bnb.matmul_4bit`` (``linear_cuda``,
nf4_backend_cuda.py:888-917), adding the FP32 LoRA term in
``_NF4CUDAProjection.forward`` (adapters/qwen35/nf4_cuda.py:170-187).

Here the record stays packed: ``stage`` copies the parts and runs the
double-quantization prologue once (FP32 scale per 64-block on the device), and
``nf4dq_linear`` runs the fused dequant-GEMM + LoRA forward and the recomputed
backward through ``fl_fwd_nf4dq`` / ``fl_bwd_nf4dq``.  bitsandbytes is not
available in this build environment, so the decode is a restatement of its
published format (the C header gives the rule); parity with the package is
unpinned.
"""
import json
import math
from dataclasses import dataclass

import torch

from . import _lib
from .ops import _flat, _need_cuda, _ptr, _stream, keeps_ts, launch_bwd, launch_fwd, ts_view

BLOCK = 64
NESTED_BLOCK = 256
QUANT_STATE_KEY = "quant_state.bitsandbytes__nf4"
PART_KEYS = {"absmax", "nested_absmax", "nested_quant_map", "quant_map", QUANT_STATE_KEY}
METADATA_KEYS = {"quant_type", "blocksize", "dtype", "shape", "nested_blocksize", "nested_dtype", "nested_offset"}


def pack_metadata(meta):
    """The quant-state metadata part: the dictionary as UTF-8 JSON bytes in a
    uint8 tensor (the form the reference's state parts carry)."""
    return torch.tensor(list(json.dumps(meta).encode("utf-8")), dtype=torch.uint8)


def unpack_metadata(t):
    if not isinstance(t, torch.Tensor) or t.dtype != torch.uint8 or t.dim() != 1 or t.numel() == 0:
        raise ValueError("packed quant-state metadata must be a nonempty one-dimensional uint8 tensor")
    try:
        meta = json.loads(bytes(t.cpu().tolist()).decode("utf-8"))
    except (UnicodeDecodeError, ValueError) as exc:
        raise ValueError("packed quant-state metadata is malformed") from exc
    if not isinstance(meta, dict):
        raise ValueError("packed quant-state metadata must decode to a dictionary")
    return meta


@dataclass
class NF4DQRecord:
    """One frozen [N, K] projection in NF4-DQ64 form (host or device tensors)."""
    packed: torch.Tensor         # uint8 [(N*K+1)//2]
    absmax: torch.Tensor         # uint8 [ceil(N*K/64)]
    nested_absmax: torch.Tensor  # float32 [ceil(blocks/256)]
    nested_map: torch.Tensor     # float32 [256]
    quant_map: torch.Tensor      # float32 [16]
    offset: float
    shape: tuple                 # (N, K)

    def __post_init__(self):
        self.shape = tuple(int(x) for x in self.shape)
        if len(self.shape) != 2 or min(self.shape) < 1:
            raise ValueError("NF4 state shape must contain two positive integer dimensions")
        numel = self.shape[0] * self.shape[1]
        blocks = (numel + BLOCK - 1) // BLOCK
        nested = (blocks + NESTED_BLOCK - 1) // NESTED_BLOCK
        packed = self.packed.reshape(-1)
        if packed.dtype != torch.uint8 or packed.numel() != (numel + 1) // 2:
            raise ValueError("packed byte count does not match the NF4 state shape")
        self.packed = packed
        if self.absmax.dtype != torch.uint8 or tuple(self.absmax.shape) != (blocks,):
            raise ValueError("primary NF4 absmax state has an invalid dtype or shape")
        if self.nested_absmax.dtype != torch.float32 or tuple(self.nested_absmax.shape) != (nested,):
            raise ValueError("secondary DQ absmax state has an invalid dtype or shape")
        if self.nested_map.dtype != torch.float32 or tuple(self.nested_map.shape) != (256,):
            raise ValueError("secondary DQ codebook must be a 256-entry float32 vector")
        if self.quant_map.dtype != torch.float32 or tuple(self.quant_map.shape) != (16,):
            raise ValueError("NF4 codebook must be a 16-entry float32 vector")
        if not math.isfinite(self.offset) or self.offset < 0:
            raise ValueError("secondary DQ offset must be finite and non-negative")

    @property
    def numel(self):
        return self.shape[0] * self.shape[1]

    @property
    def device(self):
        return self.packed.device

    def to(self, device, non_blocking=False):
        mv = lambda t: t.to(device, non_blocking=non_blocking)
        return NF4DQRecord(mv(self.packed), mv(self.absmax), mv(self.nested_absmax), mv(self.nested_map),
                           mv(self.quant_map), self.offset, self.shape)


def from_quant_state_parts(packed, parts):
    """Wrap a reference NF4 state (``packed`` uint8 [bytes, 1] plus the
    ``quant_state_parts`` mapping) without copying, with the layout checks of
    nf4_backend.py:188-244 (the codebook-identity checks need bitsandbytes and
    are left to the caller that has it)."""
    if not isinstance(packed, torch.Tensor) or packed.dtype != torch.uint8 or packed.dim() != 2 \
            or packed.shape[1] != 1:
        raise ValueError("packed must use the official uint8 [bytes, 1] layout")
    if set(parts.keys()) != PART_KEYS:
        raise ValueError("malformed quant_state_parts keys")
    meta = unpack_metadata(parts[QUANT_STATE_KEY])
    if set(meta) != METADATA_KEYS:
        raise ValueError("packed quant-state metadata has missing or unknown fields")
    if meta["quant_type"] != "nf4":
        raise ValueError("only official NF4 quantization state is supported")
    if meta["blocksize"] != BLOCK:
        raise ValueError("NF4 state must use blocksize 64")
    if meta["nested_blocksize"] != NESTED_BLOCK:
        raise ValueError("double-quantization state must use secondary blocksize 256")
    if meta["dtype"] != "bfloat16" or meta["nested_dtype"] != "float32":
        raise ValueError("NF4/DQ state has an unsupported compute or nested dtype")
    offset = meta["nested_offset"]
    if type(offset) not in (int, float):
        raise ValueError("secondary DQ offset must be finite and non-negative")
    return NF4DQRecord(packed, parts["absmax"], parts["nested_absmax"], parts["nested_quant_map"],
                       parts["quant_map"], float(offset), tuple(meta["shape"]))


@dataclass
class StagedNF4DQ:
    """A record on its GPU with the prologue's FP32 block scales."""
    record: NF4DQRecord
    block_scales: torch.Tensor  # float32 [blocks], on the record's device

    @property
    def shape(self):
        return self.record.shape


def stage(record: NF4DQRecord, device="cuda", non_blocking=True):
    """Copy the record's parts to `device` (on the current stream) and compute
    its block scales there; the counterpart of stage_cuda + CUDARecord."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("unsupported_capability: NF4-DQ64 records stage to CUDA only (no CPU fallback)")
    rec = record.to(dev, non_blocking=non_blocking)
    scales = torch.empty(rec.absmax.numel(), dtype=torch.float32, device=dev)
    _lib.call("fl_nf4dq_scales", _ptr(rec.absmax), _ptr(rec.nested_absmax), _ptr(rec.nested_map), float(rec.offset),
              rec.absmax.numel(), _ptr(scales), _stream())
    return StagedNF4DQ(rec, scales)


def dequant(staged: StagedNF4DQ, out=None):
    """BF16 [N, K] decode of a staged record."""
    rec = staged.record
    _need_cuda(rec.packed)
    if out is None:
        out = torch.empty(rec.shape, dtype=torch.bfloat16, device=rec.device)
    if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != rec.numel:
        raise ValueError("dequant destination must be a contiguous bf16 tensor of the record's numel")
    _lib.call("fl_dequant_nf4dq", _ptr(rec.packed), _ptr(staged.block_scales), _ptr(rec.quant_map), rec.numel,
              _ptr(out), _stream())
    return out


def _factors(A, B, N, K):
    rank = 0 if A is None else A.shape[0]
    if rank and (A.dtype != torch.float32 or B is None or B.dtype != torch.float32
                 or tuple(A.shape) != (rank, K) or tuple(B.shape) != (N, rank)):
        raise ValueError("LoRA factors must be fp32 A[rank, K] and B[N, rank]")
    return rank


def fwd(x, staged: StagedNF4DQ, A=None, B=None, scale=0.0, return_ts=False):
    """return_ts: also return Ts = bf16(scale * x . A^T) ([tokens, 64] bf16, a view
    of the workspace) for ``bwd(..., ts=)``; None when rank == 0."""
    N, K = staged.shape
    x2 = _flat(x, K)
    rank = _factors(A, B, N, K)
    rec = staged.record
    y, ws = launch_fwd(1, x2, rec.packed, staged.block_scales, rec.quant_map, N, A, B, scale)
    y = y.view(*x.shape[:-1], N)
    if not return_ts:
        return y
    # Every M takes the tile GEMM for these records: Ts leads the workspace.
    M = x2.shape[0]
    return y, (ts_view(ws, M) if keeps_ts(1, M, K, rank) else None)


def bwd(dy, x, staged: StagedNF4DQ, A=None, B=None, scale=0.0, dA=None, dB=None, accumulate=False, ts=None):
    """ts: the Ts ``fwd(..., return_ts=True)`` returned for the same x, A and
    scale (X . A^T is then not recomputed; results identical)."""
    N, K = staged.shape
    dy2 = _flat(dy, N)
    rank = _factors(A, B, N, K)
    rec = staged.record
    x2 = _flat(x, K) if rank else None
    dx, dA, dB = launch_bwd(1, dy2, x2, rec.packed, staged.block_scales, rec.quant_map, K, A, B, scale, dA, dB,
                            accumulate, ts)
    return dx.view(*dy.shape[:-1], K), dA, dB


def nf4dq_linear(inputs, staged: StagedNF4DQ, A=None, B=None, scale=0.0):
    """Drop-in for ``linear_cuda(inputs, state)`` (+ the projection's LoRA
    term): bf16 inputs [..., K] -> bf16 [..., N], autograd-capable in the
    inputs and the LoRA factors; input checks as nf4_backend_cuda.py:896-905."""
    if not isinstance(inputs, torch.Tensor):
        raise TypeError("inputs must be a torch.Tensor")
    if inputs.device.type != "cuda":
        raise ValueError("inputs must be on CUDA")
    if inputs.dtype is not torch.bfloat16:
        raise TypeError("inputs must have dtype torch.bfloat16")
    if inputs.ndim < 1:
        raise ValueError("inputs must have at least one dimension")
    if inputs.shape[-1] != staged.shape[1]:
        raise ValueError(f"input feature size {inputs.shape[-1]} does not match NF4 weight size {staged.shape[1]}")
    from . import library
    rec = staged.record
    N, K = staged.shape
    _factors(A, B, N, K)
    return library.frozen_linear(inputs, rec.packed, staged.block_scales, rec.quant_map, N, K, 1, A, B, scale)
