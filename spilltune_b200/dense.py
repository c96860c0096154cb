"""Dense decoder block over packed frozen weights: the call site of the fused op.

The reference's dense Llama/Qwen block (``dense_block``,
ram_vram_finetune/adapters/dense.py:120-153) receives every frozen matrix as a
BF16 tensor the slot session has just decoded (memory.py:224-229) and calls,
per projection, ``linear(x, path, lora)`` = ``LoRAProjection.forward`` or
``F.linear`` (dense.py:122-124).  ``packed_dense_block`` is the same functional
(same signature, same keyword arguments, same math and op order) for a block
whose matrices stay packed: each projection is one fused dequant-GEMM + LoRA
call (``ops.lora_projection_forward`` / ``ops.frozen_lora_linear``).

Weights arrive as the slot delivers them, keyed the way the reference flattens
stored records (``flatten_records``, quantization/codecs.py:180-188): the two
parts of a matrix ``name`` as ``@name/payload`` (uint8) and ``@name/scales``
(float32), unquantized tensors (norm weights) under their own name.  Every value
is a plain frozen tensor, so the reference's ``StreamingBlockFunction``
(training/recompute.py:16-133), whose ``_call_functional_block`` accepts only
tensors, drives this functional unchanged: forward under a ``forward`` borrow,
recompute + ``torch.autograd.grad`` under a ``backward`` borrow.

``PackedBlockReloader`` is the matching ``weight_reloader`` (its ``borrow(phase)``
is what recompute.py:137-144 calls) over a ``PackedSlotSession``.
"""
from contextlib import contextmanager

import torch
import torch.nn.functional as F

from . import codec, ops

_LUTS = {}


def part_keys(name):
    """Slot keys of a stored matrix's two parts (codecs.flatten_records naming)."""
    return f"@{name}/payload", f"@{name}/scales"


def _lut(codec_name, device):
    key = (codec_name, device)
    if key not in _LUTS:
        _LUTS[key] = codec.lut_for(codec_name).to(device)
    return _LUTS[key]


def packed_weight(weights, name, in_features, codec_name=codec.INT4_SYM):
    """PackedWeight view of matrix `name` from the slot's parts (no copy).  The
    out-features follow from the payload size: numel = 128 * groups = N * K."""
    pk, sk = part_keys(name)
    payload, scales = weights[pk], weights[sk]
    numel = scales.numel() * codec.GROUP
    if numel % in_features:
        raise ValueError(f"{name}: stored record does not hold rows of {in_features} inputs")
    return codec.PackedWeight(payload.reshape(-1), scales.reshape(-1), _lut(codec_name, payload.device),
                              (numel // in_features, in_features), codec_name)


def rms(hidden, weight, eps):
    """RMSNorm in the reference's op order (adapters/dense.py:115-117)."""
    value = hidden.float()
    return weight * (value * torch.rsqrt(value.square().mean(-1, keepdim=True) + eps)).to(hidden.dtype)


def block_forward(hidden_states, position_embeddings, attention_mask, linear, weights, *, heads, kv_heads,
                  head_dim, eps, qk_norm=False, feed_forward=None, fused=None):
    """The dense block's math (adapters/dense.py:120-153) with the projections
    supplied by ``linear(x, path)``: RMSNorm, GQA attention with full RoPE and
    an additive mask (softmax in FP32), residuals, SwiGLU MLP.  The op order
    follows the reference so BF16 roundings match.  ``fused(x, paths)``, when
    given, computes projections that share their input (q, k, v; gate, up)
    together and returns their outputs in order."""
    if fused is None:
        fused = lambda x, paths: [linear(x, p) for p in paths]  # noqa: E731
    residual = hidden_states
    x = rms(hidden_states, weights["input_layernorm.weight"], eps)
    shape = (*x.shape[:-1], -1, head_dim)
    q, k, v = fused(x, ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"))
    q = q.view(shape)
    k = k.view(shape)
    v = v.view(shape).transpose(1, 2)
    if qk_norm:
        q = rms(q, weights["self_attn.q_norm.weight"], eps)
        k = rms(k, weights["self_attn.k_norm.weight"], eps)
    q, k = q.transpose(1, 2), k.transpose(1, 2)
    cos, sin = (value.unsqueeze(1) for value in position_embeddings)

    def rotate(t):
        left, right = t.chunk(2, dim=-1)
        return t * cos + torch.cat((-right, left), dim=-1) * sin

    q, k = rotate(q), rotate(k)

    def repeat(t):
        b, h, s, d = t.shape
        return t[:, :, None].expand(b, h, heads // kv_heads, s, d).reshape(b, heads, s, d)

    k, v = repeat(k), repeat(v)
    scores = (q @ k.transpose(-2, -1)) * head_dim ** -0.5
    probabilities = torch.softmax(scores + attention_mask, dim=-1, dtype=torch.float32).to(q.dtype)
    attended = (probabilities @ v).transpose(1, 2).contiguous().reshape(*x.shape[:-1], heads * head_dim)
    x = residual + linear(attended, "self_attn.o_proj")
    residual = x
    x = rms(x, weights["post_attention_layernorm.weight"], eps)
    if feed_forward is not None:
        return residual + feed_forward(x, weights)
    gate, up = fused(x, ("mlp.gate_proj", "mlp.up_proj"))
    return residual + linear(F.silu(gate) * up, "mlp.down_proj")


def packed_dense_block(hidden_states, position_embeddings, attention_mask, *, heads, kv_heads, head_dim, eps,
                       lora_q, lora_v, lora_o, qk_norm=False, feed_forward=None, codec_name=codec.INT4_SYM,
                       lora_k=None, lora_gate=None, lora_up=None, lora_down=None, **weights):
    """Drop-in for the reference's ``dense_block`` functional over packed parts.

    ``lora_q``/``lora_v``/``lora_o`` are the block's ``LoRAProjection`` objects
    (or None) exactly as the reference binds them (its default targets,
    adapters/targets.py:3-9); ``lora_k``/``lora_gate``/``lora_up``/``lora_down``
    optionally adapt the other four projections, for plans that target all
    seven.  Each is a keyword argument of its own, so ``StreamingBlockFunction``'s
    binding check (recompute.py:180-203) sees every bound projection.  Each
    projection runs as one fused call; unadapted projections run the plain
    frozen F.linear (rank 0)."""
    adapters = {"self_attn.q_proj": lora_q, "self_attn.k_proj": lora_k, "self_attn.v_proj": lora_v,
                "self_attn.o_proj": lora_o, "mlp.gate_proj": lora_gate, "mlp.up_proj": lora_up,
                "mlp.down_proj": lora_down}

    def record(x, path):
        if weights.get(path + ".bias") is not None:
            raise ValueError("unsupported_capability: fused frozen linear has no bias term")
        return packed_weight(weights, path + ".weight", x.shape[-1], codec_name)

    def linear(x, path):
        pw = record(x, path)
        proj = adapters.get(path)
        if proj is not None:
            return ops.lora_projection_forward(proj, x, pw)
        return ops.frozen_lora_linear(x, pw)

    def fused(x, paths):
        """Projections of one input as one call when the slot holds them back
        to back and their LoRA branches share one scale (q, k, v; gate, up);
        each adapted projection is checked like LoRAProjection.forward."""
        pws = [record(x, p) for p in paths]
        projs = [adapters.get(p) for p in paths]
        for p, pw in zip(projs, pws):
            if p is not None:
                ops.check_projection(p, x, pw)
        scales = {p.scale for p in projs if p is not None}
        if len(scales) <= 1:
            factors = [(p.A, p.B) if p is not None else None for p in projs]
            return ops.fused_lora_linears(x, pws, factors, scales.pop() if scales else 0.0)
        return [linear(x, p) for p in paths]

    return block_forward(hidden_states, position_embeddings, attention_mask, linear, weights, heads=heads,
                         kv_heads=kv_heads, head_dim=head_dim, eps=eps, qk_norm=qk_norm, feed_forward=feed_forward,
                         fused=fused)


class PackedBlockReloader:
    """The ``weight_reloader`` of one block over a ``PackedSlotSession``.

    ``borrow(phase)`` (the hook ``StreamingBlockFunction`` uses, recompute.py:
    137-144) borrows layer `index` of the session for `phase` ('forward' or
    'backward', which sets the prefetch direction) and yields the functional's
    weights: each packed matrix as its two flat part tensors under the
    reference's part keys, plus the block's small unquantized tensors
    (``raw``, e.g. norm weights, kept resident on the device).  The views are
    valid only inside the borrow, like the reference's slot views."""

    def __init__(self, session, index, raw=None):
        self.session = session
        self.index = index
        self.raw = dict(raw or {})

    @contextmanager
    def borrow(self, phase):
        with self.session.borrow(self.index, phase) as views:
            out = dict(self.raw)
            for name, pw in views.items():
                pk, sk = part_keys(name)
                out[pk] = pw.payload
                out[sk] = pw.scales
            yield out

    def __call__(self):
        raise RuntimeError("packed slot views are only valid inside borrow(phase)")
