"""Tiny-Llama LoRA streaming training for end-to-end parity -- test infrastructure.

The workload is the tiny-Llama training configuration run for 50 optimizer steps: a random Llama
(2 decoder layers, hidden 256, 4 heads of 64, 2 KV heads, SwiGLU 768, vocab
2048, RMSNorm eps 1e-6, RoPE theta 1e4), frozen decoder matrices stored
int4-sym-g128, LoRA rank 8 alpha 16 on the reference's default dense targets
(q, v, o), AdamW lr 1e-4 (weight decay 0), 16 seeded rows of 128 uniform
token ids (labels = ids) visited in order, two rows (micro-batches) per step.

``tests/golden/make_golden.py`` trains it with the reference's own engine
(``training/engine.py:run``, adapter ``llama``) and commits the per-step
losses and LoRA gradients / parameters (``tiny_llama_train.npz``).  This
module restates the reference's training step around a pluggable block
functional, weight reloader and terminal so that:

* on the CPU, with the block math of ``spilltune_b200.dense.block_forward``
  and the oracle's decode + ``LoRAProjection.forward`` as the projection, it
  reproduces the reference's fixture (the restatement is pinned);
* on the GPU, with ``spilltune_b200.dense.packed_dense_block`` (every
  projection one fused call on packed weights), ``PackedSlotSession`` streaming
  and the fused LM-head CE, it is the system under test.

Reference files restated here: ``training/engine.py:44-78`` (``microbatch``),
``:81-...`` (step loop: zero_grad, accumulate, step), ``training/recompute.py:
16-133`` (``StreamingBlockFunction``), ``adapters/dense.py:232-247``
(``positions_and_masks``), ``finetune/lora.py:319-388`` (LoRA creation order and
init), ``finetune/optimizer.py:231-341`` (``LoRAOptimizer``).
"""
import math
from contextlib import contextmanager

import torch
import torch.nn.functional as F

VOCAB, HIDDEN, LAYERS, HEADS, KV_HEADS, HEAD_DIM, INTER = 2048, 256, 2, 4, 2, 64, 768
EPS, THETA, MAX_POS = 1e-6, 10000.0, 256
SEQ, ROWS, STEPS, ACCUM = 128, 16, 50, 2
RANK, ALPHA, LR, SEED, TOKEN_CHUNK = 8, 16.0, 1e-4, 42, 64
MODEL_SEED, DATA_SEED = 1234, 99
TARGETS = ("self_attn.q_proj", "self_attn.v_proj", "self_attn.o_proj")  # reference adapters/targets.py:3-9
ALL7 = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
        "mlp.up_proj", "mlp.down_proj")  # the tiny-Llama configuration: LoRA on every projection
MATRICES = {"self_attn.q_proj": (HEADS * HEAD_DIM, HIDDEN), "self_attn.k_proj": (KV_HEADS * HEAD_DIM, HIDDEN),
            "self_attn.v_proj": (KV_HEADS * HEAD_DIM, HIDDEN), "self_attn.o_proj": (HIDDEN, HEADS * HEAD_DIM),
            "mlp.gate_proj": (INTER, HIDDEN), "mlp.up_proj": (INTER, HIDDEN), "mlp.down_proj": (HIDDEN, INTER)}


def model_state():
    """The model's FP32 tensors under their Llama checkpoint names (seeded)."""
    g = torch.Generator().manual_seed(MODEL_SEED)
    state = {"model.embed_tokens.weight": torch.randn(VOCAB, HIDDEN, generator=g) * 0.02}
    for i in range(LAYERS):
        p = f"model.layers.{i}."
        state[p + "input_layernorm.weight"] = 0.8 + 0.4 * torch.rand(HIDDEN, generator=g)
        for name, shape in MATRICES.items():
            state[p + name + ".weight"] = torch.randn(*shape, generator=g) * 0.02
        state[p + "post_attention_layernorm.weight"] = 0.8 + 0.4 * torch.rand(HIDDEN, generator=g)
    state["model.norm.weight"] = 0.8 + 0.4 * torch.rand(HIDDEN, generator=g)
    state["lm_head.weight"] = torch.randn(VOCAB, HIDDEN, generator=g) * 0.02
    return state


def token_rows():
    """ROWS rows of SEQ uniform token ids; every shifted token is supervised."""
    g = torch.Generator().manual_seed(DATA_SEED)
    ids = torch.randint(0, VOCAB, (ROWS, SEQ), generator=g)
    return [(ids[i:i + 1].clone(), ids[i:i + 1].clone()) for i in range(ROWS)]


# ----------------------------------------------------------------- LoRA state
class Projection:
    """The state of one reference ``LoRAProjection`` (finetune/lora.py:97-176):
    FP32 A [r, K] (randn * 0.02), B [N, r] (zeros), gradient buffers and Adam
    moments, scale alpha / r."""

    def __init__(self, name, out_features, in_features, A, device):
        self.name = self.target_path = name
        self.rank, self.alpha = RANK, ALPHA
        self.in_features, self.out_features = in_features, out_features
        self.A = A.detach().clone().to(device).requires_grad_(True)
        self.B = torch.zeros(out_features, RANK, device=device).requires_grad_(True)
        z = lambda t: torch.zeros_like(t.detach())
        self.grad_A, self.grad_B = z(self.A), z(self.B)
        self.m_A, self.v_A, self.m_B, self.v_B = z(self.A), z(self.A), z(self.B), z(self.B)

    @property
    def scale(self):
        return self.alpha / self.rank

    @property
    def base_weight_shape(self):
        return (self.out_features, self.in_features)

    def zero_grad(self):
        self.grad_A.zero_()
        self.grad_B.zero_()


def make_adapters(device, targets=TARGETS):
    """Per block, {target path: Projection}, with A drawn exactly as the
    reference's run does: torch.manual_seed(seed) at the start of
    engine.run, then randn(rank, in).mul_(0.02) block by block, target by
    target (create_lora_for_block)."""
    torch.manual_seed(SEED)
    blocks = []
    for _ in range(LAYERS):
        d = {}
        for t in targets:
            N, K = MATRICES[t]
            A = torch.randn(RANK, K, dtype=torch.float32).mul_(0.02)
            d[t] = Projection(t, N, K, A, device)
        blocks.append(d)
    return blocks


class AdamW:
    """``LoRAOptimizer`` (finetune/optimizer.py): bias-corrected FP32 AdamW in
    torch.optim.AdamW's single-tensor op order, weight decay 0."""

    def __init__(self, lr=LR, beta1=0.9, beta2=0.999, eps=1e-8):
        self.lr, self.beta1, self.beta2, self.eps = lr, beta1, beta2, eps
        self.step_count = 0

    def zero_grad(self, projections):
        for p in projections:
            p.grad_A.zero_()
            p.grad_B.zero_()
            p.A.grad = None
            p.B.grad = None

    def step(self, projections):
        n = self.step_count + 1
        step_size = self.lr / (1.0 - self.beta1 ** n)
        bc2 = math.sqrt(1.0 - self.beta2 ** n)
        with torch.no_grad():
            for p in projections:
                for param, grad, m, v in ((p.A, p.grad_A, p.m_A, p.v_A), (p.B, p.grad_B, p.m_B, p.v_B)):
                    m.lerp_(grad, 1.0 - self.beta1)
                    v.mul_(self.beta2).addcmul_(grad, grad, value=1.0 - self.beta2)
                    denom = (v.sqrt() / bc2).add_(self.eps)
                    param.addcdiv_(m, denom, value=-step_size)
        self.step_count = n


# ----------------------------------------------------------------- streaming block
@contextmanager
def _borrow(reloader, phase):
    borrow = getattr(reloader, "borrow", None)
    if borrow is None:
        yield reloader()
    else:
        with borrow(phase) as w:
            yield w


class StreamingBlock(torch.autograd.Function):
    """``StreamingBlockFunction``: keep the block input; forward under a
    'forward' borrow; backward reloads under a 'backward' borrow, recomputes the
    same functional and takes ``autograd.grad`` w.r.t. the input and every A/B
    (sorted by name), then replaces or accumulates grad_A/grad_B."""

    @staticmethod
    def forward(ctx, hidden, positions, mask, functional, kwargs, reloader, adapters, accumulate):
        ctx.functional, ctx.kwargs, ctx.reloader = functional, kwargs, reloader
        ctx.adapters, ctx.accumulate, ctx.positions, ctx.mask = adapters, accumulate, positions, mask
        ctx.save_for_backward(hidden.detach().clone())
        with _borrow(reloader, "forward") as weights:
            return functional(hidden_states=hidden, position_embeddings=positions, attention_mask=mask,
                              **weights, **kwargs)

    @staticmethod
    def backward(ctx, grad_output):
        hidden = ctx.saved_tensors[0].detach().requires_grad_(True)
        projs = sorted(ctx.adapters.values(), key=lambda p: p.name)
        inputs = [hidden] + [t for p in projs for t in (p.A, p.B)]
        with _borrow(ctx.reloader, "backward") as weights:
            with torch.enable_grad():
                out = ctx.functional(hidden_states=hidden, position_embeddings=ctx.positions,
                                     attention_mask=ctx.mask, **weights, **ctx.kwargs)
            grads = torch.autograd.grad(out, inputs, grad_output, allow_unused=True)
            for i, p in enumerate(projs):
                ga, gb = grads[1 + 2 * i], grads[2 + 2 * i]
                if ga is None or gb is None:
                    raise RuntimeError(f"adapter {p.name} is disconnected")
                if not ctx.accumulate:
                    p.zero_grad()
                p.grad_A.add_(ga.detach().to(p.grad_A))
                p.grad_B.add_(gb.detach().to(p.grad_B))
        return (grads[0],) + (None,) * 7


def positions_and_masks(batch, length, device, dtype=torch.bfloat16):
    """Full RoPE cos/sin and the causal additive mask (all-valid rows)."""
    positions = torch.arange(length, device=device).expand(batch, -1)
    inv = 1.0 / THETA ** (torch.arange(0, HEAD_DIM, 2, device=device).float() / HEAD_DIM)
    freq = (inv[None, :, None].expand(batch, -1, 1) @ positions[:, None].float()).transpose(1, 2)
    phase = torch.cat((freq, freq), -1)
    rotary = (phase.cos().to(dtype), phase.sin().to(dtype))
    blocked = torch.ones(length, length, dtype=torch.bool, device=device).triu(1)[None, None]
    blocked = blocked.expand(batch, 1, length, length)
    mask = torch.zeros(blocked.shape, dtype=dtype, device=device).masked_fill(blocked, torch.finfo(dtype).min)
    return rotary, mask


def reference_terminal(normalized, head, labels, normalization, token_chunk):
    """engine.py:58-78: per token chunk, bf16 logits, FP32 summed CE, the VJP of
    chunk / normalization; returns (loss_sum, d normalized)."""
    grad_n = torch.zeros_like(normalized)
    loss_sum = torch.zeros((), device=normalized.device)
    S = normalized.shape[1]
    for start in range(0, S - 1, token_chunk):
        end = min(start + token_chunk, S - 1)
        target = labels[:, start + 1:end + 1]
        if not (target != -100).any():
            continue
        h = normalized[:, start:end].detach().requires_grad_(True)
        logits = F.linear(h, head)
        chunk = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), target.reshape(-1),
                                ignore_index=-100, reduction="sum")
        (g,) = torch.autograd.grad(chunk / normalization, h)
        grad_n[:, start:end].copy_(g.detach())
        loss_sum += chunk.detach()
    return loss_sum, grad_n


def fused_terminal(normalized, head, labels, normalization, token_chunk):
    """The same terminal through spilltune_b200.head (fused LM head + CE)."""
    from spilltune_b200 import head as hd
    S = normalized.shape[1]
    lab = labels.cpu()
    chunks = tuple((s, min(s + token_chunk, S - 1)) for s in range(0, S - 1, token_chunk)
                   if bool((lab[:, s + 1:min(s + token_chunk, S - 1) + 1] != -100).any()))
    n = normalized.detach().requires_grad_(True)
    loss = hd.chunked_causal_loss(n, head, labels.to(normalized.device), normalization=normalization,
                                  token_chunk=token_chunk, supervised_chunks=chunks)
    (g,) = torch.autograd.grad(loss, n)
    return loss.detach() * normalization, g


class Block:
    def __init__(self, index, functional, kwargs, reloader, adapters):
        self.index, self.functional, self.kwargs = index, functional, kwargs
        self.reloader, self.adapters = reloader, adapters


def microbatch(blocks, embedding, norm_weight, head, ids, labels, *, normalization, accumulate, device, terminal):
    """engine.py:44-78 for one row."""
    from spilltune_b200.dense import rms
    positions, mask = positions_and_masks(ids.shape[0], ids.shape[1], device)
    embedded = F.embedding(ids.cpu(), embedding).to(device).detach().requires_grad_(True)
    hidden = embedded
    for b in blocks:
        hidden = StreamingBlock.apply(hidden, positions, mask, b.functional, b.kwargs, b.reloader, b.adapters,
                                      accumulate)
    terminal_input = hidden.detach().requires_grad_(True)
    normalized = rms(terminal_input, norm_weight, EPS)
    loss_sum, grad_n = terminal(normalized, head, labels.to(device), normalization, TOKEN_CHUNK)
    (gradient,) = torch.autograd.grad(normalized, terminal_input, grad_n)
    if not torch.isfinite(loss_sum) or not torch.isfinite(gradient).all():
        raise FloatingPointError("non-finite causal loss/gradient")
    hidden.backward(gradient)
    return float(loss_sum / normalization)


def train(blocks, embedding, norm_weight, head, *, device, terminal, steps=STEPS, on_step=None):
    """The engine's step loop: cyclic rows, ACCUM micro-batches per step, one
    global normalisation per window, zero_grad / accumulate / AdamW step."""
    rows = token_rows()
    projections = [p for b in blocks for _, p in sorted(b.adapters.items())]
    opt = AdamW()
    losses, cursor = [], 0
    for step in range(1, steps + 1):
        items = [rows[(cursor + i) % len(rows)] for i in range(ACCUM)]
        normalization = sum(int((lab[:, 1:] != -100).sum()) for _, lab in items)
        opt.zero_grad(projections)
        loss = 0.0
        for i, (ids, lab) in enumerate(items):
            loss += microbatch(blocks, embedding, norm_weight, head, ids, lab, normalization=normalization,
                               accumulate=i > 0, device=device, terminal=terminal)
        opt.step(projections)
        cursor += ACCUM
        losses.append(loss)
        if on_step is not None:
            on_step(step, blocks)
    return losses
