"""Torch-facing frozen-linear operators over the C ABI.

``frozen_lora_linear(x, weight, A, B, scale)`` is the drop-in for the
reference's ``LoRAProjection.forward(x, base_weight)`` (finetune/lora.py:205-220)
when the slot hands the projection its packed record instead of a decoded BF16
matrix.  Its autograd backward returns ``(dX, dA, dB)`` in one fused call, so
``torch.autograd.grad(output, [hidden, A0, B0, ...])`` inside the reference's
``StreamingBlockFunction.backward`` (training/recompute.py:102-127) works
unchanged and accumulates into ``grad_A``/``grad_B`` exactly as before.

All work runs on the current CUDA stream.  CPU tensors are rejected: the path
has no CPU fallback.
"""
import torch

from . import _lib
from .codec import PackedWeight

FL_MAX_RANK = 64


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _need_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("unsupported_capability: spilltune_b200 ops need CUDA tensors (no CPU fallback)")


def _ptr(t):
    return None if t is None else t.data_ptr()


def dequant(weight: PackedWeight, out=None):
    """Decode a packed record into a BF16 [N, K] tensor (bit-exact decode_into)."""
    _need_cuda(weight.payload, weight.scales, weight.lut)
    if out is None:
        out = torch.empty(weight.shape, dtype=torch.bfloat16, device=weight.device)
    if out.dtype != torch.bfloat16 or not out.is_contiguous() or out.numel() != weight.numel:
        raise ValueError("dequant destination must be a contiguous bf16 tensor of the record's numel")
    _lib.call("fl_dequant", _ptr(weight.payload), _ptr(weight.scales), _ptr(weight.lut), weight.numel,
              _ptr(out), _stream())
    return out


def _flat(x, K):
    if x.shape[-1] != K:
        raise ValueError(f"input width mismatch: expected {K}, got {x.shape[-1]}")
    x2 = x.reshape(-1, K)
    if x2.dtype != torch.bfloat16:
        raise ValueError("activations must be bf16")
    return x2.contiguous()


def _matrix_shape(weight: PackedWeight):
    if len(weight.shape) != 2:
        raise ValueError("stacked expert records [E, N, K] go through spilltune_b200.moe (grouped ops)")
    return weight.shape


# Entry points per record layout: 0 = group-128 (int4-sym / NF4 codebook),
# 1 = bitsandbytes NF4-DQ64 (packed high nibble first, FP32 block scales).
_FWD_ENTRY = {0: "fl_fwd", 1: "fl_fwd_nf4dq"}
_BWD_ENTRY = {0: ("fl_bwd", "fl_bwd_ts"), 1: ("fl_bwd_nf4dq", "fl_bwd_nf4dq_ts")}


def keeps_ts(layout, M, K, rank):
    """Whether the forward leaves Ts = bf16(s * X . A^T) in the first M * 128
    bytes of its workspace (the rule fl_bwd_ts documents): every LoRA call but
    the decode-step kernels' (group-128 layout, <= 16 tokens, K % 512 == 0)."""
    return rank > 0 and M > 0 and not (layout == 0 and M <= 16 and K % 512 == 0)


def launch_fwd(layout, x2, payload, scales, lut, N, A=None, B=None, scale=0.0, split_reduction=True):
    """One forward call on raw record parts: x2 bf16 [M, K] contiguous ->
    (Y bf16 [M, N], workspace uint8 or None).  A/B fp32 [rank, K] / [N, rank].

    split_reduction: give the call room to split its reduction when it has few
    output tiles (fl_fwd_workspace_bytes_split); False keeps one pass per
    output tile (the summation order of the grouped kernels).  When the split
    was possible the returned workspace is a copy of just its Ts rows, so a
    saved Ts does not hold the partial-sum scratch."""
    M, K = x2.shape
    rank = 0 if A is None else A.shape[0]
    _need_cuda(x2, payload, A, B)
    if rank:
        if A.dtype != torch.float32 or B is None or B.dtype != torch.float32 or tuple(A.shape) != (rank, K) \
                or tuple(B.shape) != (N, rank):
            raise ValueError("LoRA factors must be fp32 A[rank, K] and B[N, rank]")
        A = A.detach().contiguous()
        B = B.detach().contiguous()
    y = torch.empty((M, N), dtype=torch.bfloat16, device=x2.device)
    lib = _lib.load()
    base = lib.fl_fwd_workspace_bytes(M, K, rank)
    ws_bytes = lib.fl_fwd_workspace_bytes_split(M, N, K, rank) if split_reduction and M else base
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x2.device) if ws_bytes else None
    if M:
        _lib.call(_FWD_ENTRY[layout], _ptr(x2), M, K, _ptr(payload), _ptr(scales), _ptr(lut), N, _ptr(A), _ptr(B),
                  rank, float(scale), _ptr(y), _ptr(ws), ws_bytes, _stream())
    if ws_bytes > base and keeps_ts(layout, M, K, rank):
        ws = ws[:M * 128].clone()
    return y, ws


def ts_view(ws, M):
    """The Ts rows a forward left at the start of its workspace ([M, 64] bf16)."""
    return ws[:M * 128].view(torch.bfloat16).view(M, 64)


def launch_bwd(layout, dy2, x2, payload, scales, lut, K, A=None, B=None, scale=0.0, dA=None, dB=None,
               accumulate=False, ts=None, split_reduction=True):
    """One backward call on raw record parts -> (dX bf16 [M, K], dA, dB).
    split_reduction as for launch_fwd (dX's reduction over N)."""
    M, N = dy2.shape
    rank = 0 if A is None else A.shape[0]
    _need_cuda(dy2, x2, payload, A, B)
    dx = torch.empty((M, K), dtype=torch.bfloat16, device=dy2.device)
    if rank:
        if A.dtype != torch.float32 or B is None or B.dtype != torch.float32 or tuple(A.shape) != (rank, K) \
                or tuple(B.shape) != (N, rank):
            raise ValueError("LoRA factors must be fp32 A[rank, K] and B[N, rank]")
        if x2 is None or tuple(x2.shape) != (M, K):
            raise ValueError(f"the LoRA backward needs the forward's input [{M}, {K}]")
        A = A.detach().contiguous()
        B = B.detach().contiguous()
        if dA is None:
            dA = torch.empty((rank, K), dtype=torch.float32, device=dy2.device)
            accumulate = False
        if dB is None:
            dB = torch.empty((N, rank), dtype=torch.float32, device=dy2.device)
            accumulate = False
    lib = _lib.load()
    ws_bytes = (lib.fl_bwd_workspace_bytes_split if split_reduction and M else lib.fl_bwd_workspace_bytes)(
        M, N, K, rank)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dy2.device) if ws_bytes else None
    if ts is not None and rank:
        if ts.dtype != torch.bfloat16 or tuple(ts.shape) != (M, 64) or not ts.is_contiguous():
            raise ValueError("ts must be the [tokens, 64] bf16 Ts that fwd(..., return_ts=True) returned")
        _need_cuda(ts)
    plain, with_ts = _BWD_ENTRY[layout]
    if M and ts is not None and rank:
        _lib.call(with_ts, _ptr(dy2), _ptr(x2), M, N, K, _ptr(payload), _ptr(scales), _ptr(lut), _ptr(A), _ptr(B),
                  rank, float(scale), _ptr(ts), _ptr(dx), _ptr(dA), _ptr(dB), int(bool(accumulate)), _ptr(ws),
                  ws_bytes, _stream())
    elif M:
        _lib.call(plain, _ptr(dy2), _ptr(x2), M, N, K, _ptr(payload), _ptr(scales), _ptr(lut), _ptr(A), _ptr(B),
                  rank, float(scale), _ptr(dx), _ptr(dA), _ptr(dB), int(bool(accumulate)), _ptr(ws), ws_bytes,
                  _stream())
    elif rank and not accumulate:
        dA.zero_()
        dB.zero_()
    return dx, dA, dB


def fwd(x, weight: PackedWeight, A=None, B=None, scale=0.0, return_ts=False, split_reduction=True):
    """Y = x . W^T + scale * (x . A^T) . B^T  (bf16 out; plain frozen linear if A is None).

    return_ts: also return Ts = bf16(scale * x . A^T) ([tokens, 64] bf16, zero past
    the rank) as a view of the call's workspace, for ``bwd(..., ts=)`` -- the
    intermediate the reference's autograd keeps from the forward for grad_B
    (finetune/lora.py:219-220).  None when rank == 0 or when the decode-step
    kernels take the call (<= 16 tokens, K % 512 == 0: they form Ts themselves).
    split_reduction=False: no split of the reduction for few output tiles (see
    launch_fwd; the grouped kernels' summation order).
    """
    N, K = _matrix_shape(weight)
    x2 = _flat(x, K)
    rank = 0 if A is None else A.shape[0]
    y, ws = launch_fwd(0, x2, weight.payload, weight.scales, weight.lut, N, A, B, scale, split_reduction)
    y = y.view(*x.shape[:-1], N)
    if not return_ts:
        return y
    M = x2.shape[0]
    return y, (ts_view(ws, M) if keeps_ts(0, M, K, rank) else None)


def bwd(dy, x, weight: PackedWeight, A=None, B=None, scale=0.0, dA=None, dB=None, accumulate=False, ts=None,
        split_reduction=True):
    """Returns (dX, dA, dB) of fwd(); dA/dB are fp32 (accumulated into when given and accumulate).

    ts: the Ts that ``fwd(..., return_ts=True)`` returned for the same x, A and
    scale; X . A^T is then not recomputed (results identical).
    split_reduction: as for fwd (dX's reduction over N)."""
    N, K = _matrix_shape(weight)
    dy2 = _flat(dy, N)
    rank = 0 if A is None else A.shape[0]
    x2 = _flat(x, K) if rank else None
    dx, dA, dB = launch_bwd(0, dy2, x2, weight.payload, weight.scales, weight.lut, K, A, B, scale, dA, dB,
                            accumulate, ts, split_reduction)
    return dx.view(*dy.shape[:-1], K), dA, dB


def frozen_lora_linear(x, weight: PackedWeight, A=None, B=None, scale=0.0):
    """Autograd-capable Y = x . W^T + scale * (x . A^T) . B^T over a packed frozen weight.

    Runs the ``spilltune_b200::frozen_lora_linear`` custom op (registered in
    ``spilltune_b200.library``), whose backward returns (dX, dA, dB) from one
    fused call, so ``torch.autograd.grad(output, [hidden, A0, B0, ...])`` inside
    the reference's ``StreamingBlockFunction.backward`` (training/recompute.py:
    102-127) accumulates into ``grad_A``/``grad_B`` exactly as before."""
    from . import library
    N, K = _matrix_shape(weight)
    return library.frozen_linear(x, weight.payload, weight.scales, weight.lut, N, K, 0, A, B, scale)


def concat_records(weights):
    """One stacked record over matrices that share their input and sit back to
    back in memory (a slot image or ``streaming.pack_layer`` places a layer's
    payloads contiguously, then its scales): the view [sum N_i, K] whose rows
    are the matrices' rows in order, or None when the parts are not adjacent,
    the input widths or codebooks differ, or a record is not a plain [N, K]
    matrix.  No copy."""
    if len(weights) < 2:
        return None
    first = weights[0]
    K = first.shape[-1]
    # Host-side checks only (pointers, shapes, codec names): nothing here may
    # touch the device, which would synchronise the stream on every call.  The
    # codebook follows from the codec name.
    for w in weights:
        if len(w.shape) != 2 or w.shape[1] != K or w.codec != first.codec:
            return None
    for a, b in zip(weights, weights[1:]):
        if a.payload.untyped_storage().data_ptr() != b.payload.untyped_storage().data_ptr():
            return None
        if a.payload.data_ptr() + a.payload.numel() != b.payload.data_ptr():
            return None
        if a.scales.data_ptr() + 4 * a.scales.numel() != b.scales.data_ptr():
            return None
    N = sum(w.shape[0] for w in weights)
    payload = first.payload.as_strided((N * K // 2,), (1,))
    scales = first.scales.as_strided((N * K // 128,), (1,))
    return PackedWeight(payload, scales, first.lut, (N, K), first.codec)


def concat_lora(factors, out_features):
    """The LoRA factors of several projections over one input as one branch:
    A = [A_1; A_2; ...] ([sum r_i, K]) and B = blockdiag(B_1, B_2, ...)
    ([sum N_i, sum r_i]; a projection without LoRA contributes rows of zeros).
    Built with differentiable torch ops, so gradients reach every A_i and B_i
    and the zero blocks receive none.  `factors` is [(A_i, B_i) or None] in
    record order, `out_features` the N_i.  Returns (A, B) or (None, None)."""
    As, Bs = [], []
    for f, n in zip(factors, out_features):
        if f is None:
            continue
        As.append(f[0])
    if not As:
        return None, None
    for f, n in zip(factors, out_features):
        if f is None:
            Bs.append(As[0].new_zeros((n, 0)))
        else:
            Bs.append(f[1])
    return torch.cat(As, 0), torch.block_diag(*Bs)


def fused_lora_linears(x, weights, factors=None, scale=0.0):
    """Projections of one input x as one fused call when their records are
    adjacent (``concat_records``) and their LoRA branches share `scale`:
    returns the list of outputs, each x . W_i^T + scale * (x . A_i^T) . B_i^T,
    autograd-capable in x and every A_i, B_i.  Otherwise one call each.  The
    combined rank (sum of r_i) must be <= 64."""
    factors = factors or [None] * len(weights)
    outs = [w.shape[0] for w in weights]
    cat = concat_records(weights)
    ranks = sum(f[0].shape[0] for f in factors if f is not None)
    if cat is None or ranks > FL_MAX_RANK:
        return [frozen_lora_linear(x, w, *(f if f is not None else (None, None)), scale)
                for w, f in zip(weights, factors)]
    A, B = concat_lora(factors, outs)
    y = frozen_lora_linear(x, cat, A, B, scale)
    return list(y.split(outs, dim=-1))


def check_projection(proj, x, weight: PackedWeight):
    """The shape checks of LoRAProjection.forward (finetune/lora.py:207-216), same messages."""
    if tuple(weight.shape) != tuple(proj.base_weight_shape):
        raise ValueError(
            f"{proj.target_path} base weight shape mismatch: expected "
            f"{tuple(proj.base_weight_shape)}, got {tuple(weight.shape)}")
    if x.shape[-1] != proj.in_features:
        raise ValueError(
            f"{proj.target_path} input width mismatch: expected {proj.in_features}, got {x.shape[-1]}")


def lora_projection_forward(proj, x, weight: PackedWeight, base_bias=None):
    """``LoRAProjection.forward(x, base_weight, base_bias)`` with a packed base weight.

    Same argument meaning and error behaviour as finetune/lora.py:205-220
    (shape checks raise ValueError); bias-carrying projections are rejected
    because the fused kernels have no bias term.
    """
    check_projection(proj, x, weight)
    if base_bias is not None:
        raise ValueError("unsupported_capability: fused frozen linear has no bias term")
    return frozen_lora_linear(x, weight, proj.A, proj.B, proj.scale)
