"""Generate the golden fixtures in this folder by importing the reference itself.

Run in a container where the SpillTune reference source is available:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

It writes small ``.npz`` files (a few KB each).  The tests never import the
reference; they only read these committed vectors.

* ``codec_int4.npz`` — ``codecs.encode(mode='int4-sym-g128')`` payload/scales and
  ``codecs.materialize`` BF16 bits for seeded tensors covering a tail group
  (129, 257 elements), an all-zero group (scale 1.0), the known-answer vector of
  the reference's ``tests/test_quantization.py:73-81`` and a 32x256 matrix.
* ``lora_small.npz`` — ``LoRAProjection.forward`` (``finetune/lora.py:205-220``)
  on the decoded matrix plus the autograd backward (dX, dA, dB) for a seeded
  problem with M=18 (ragged), K=256, N=384, rank 8, alpha 16.
* ``moe_small.npz`` — the reference's Qwen3-MoE ``moe_feed_forward``
  (``adapters/qwen3_moe.py:95-113``) on int4-sym-g128-encoded stacked experts
  (E=6, top-2, hidden 128, expert intermediate 128, 24 tokens, expert 5 never
  routed), its output and the autograd gradient of the hidden states.
* ``deepseek_route.npz`` — the reference's DeepSeek-V3 router
  (``adapters/deepseek.py:115-126``): 16 experts in 4 groups, 2 kept, top-4,
  normalised, scale 2.5; indices and weights sorted by expert id per token.
* ``head_small.npz`` — the reference's ``chunked_causal_loss``
  (``quantization/native_terminal.py:11-47``) on seeded bf16 hidden states,
  a bf16 head and labels with ignored (-100) positions: loss and the hidden
  states' gradient.
* ``tiny_llama_train.npz`` — the reference's own training engine
  (``training/engine.py:run``, adapter ``llama``, int4-sym-g128 storage, CPU)
  on the tiny Llama of ``tests/e2e_tiny.py`` for 50 AdamW steps: the per-step
  losses, every LoRA projection's gradients after steps 1 and 2, its A and B
  after step 50, and checksums of the initial A (to confirm the tests draw the
  same initial state).
* ``tiny_llama_train_all7.npz`` — the same with LoRA on all seven projections
  (the tiny-Llama training configuration) through a registered adapter (``_all7_factory``).
"""
import os
import sys

import numpy as np
import torch

from ram_vram_finetune.quantization import codecs
from ram_vram_finetune.finetune.lora import LoRAProjection
from ram_vram_finetune.adapters.qwen3_moe import moe_feed_forward
from ram_vram_finetune.adapters.deepseek import route as deepseek_route
from ram_vram_finetune.quantization.native_terminal import chunked_causal_loss

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))  # tests/: the shared tiny-Llama definition
import e2e_tiny  # noqa: E402


def bits(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def codec_cases():
    torch.manual_seed(43)
    cases = {}
    for length in (128, 129, 257):
        v = torch.randn(1, length) * 0.03
        v[:, :128] = 0
        cases[f"len{length}"] = v
    kat = torch.zeros(1, 128)
    kat[0, :6] = torch.tensor([-7, -1.5, -.5, .5, 1.5, 7])
    cases["kat"] = kat
    g = torch.Generator().manual_seed(7)
    cases["mat32x256"] = torch.randn(32, 256, generator=g) * 0.02
    out = {}
    for name, v in cases.items():
        rec = codecs.encode(v.contiguous(), "int4-sym-g128")
        codecs.validate_spec(rec.spec, rec.parts)
        out[f"{name}/input"] = v.numpy().astype(np.float32)
        out[f"{name}/payload"] = rec.parts["payload"].numpy()
        out[f"{name}/scales"] = rec.parts["scales"].numpy()
        out[f"{name}/decoded_bf16"] = bits(codecs.materialize(rec)).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "codec_int4.npz"), **out)


def lora_case():
    M, K, N, r, alpha = 18, 256, 384, 8, 16.0
    g = torch.Generator().manual_seed(11)
    w = torch.randn(N, K, generator=g) * 0.02
    rec = codecs.encode(w.contiguous(), "int4-sym-g128")
    W = codecs.materialize(rec)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    A = torch.randn(r, K, generator=g) * 0.05
    B = torch.randn(N, r, generator=g) * 0.05
    dY = torch.randn(M, N, generator=g).to(torch.bfloat16)
    z = lambda t: torch.zeros_like(t)
    proj = LoRAProjection(name="self_attn.q_proj", rank=r, alpha=alpha, in_features=K,
                          out_features=N, A=A.clone(), B=B.clone(), grad_A=z(A), grad_B=z(B),
                          m_A=z(A), v_A=z(A), m_B=z(B), v_B=z(B))
    xr = x.clone().requires_grad_(True)
    y = proj.forward(xr, W)
    dx, da, db = torch.autograd.grad(y, (xr, proj.A, proj.B), dY)
    np.savez_compressed(
        os.path.join(HERE, "lora_small.npz"),
        M=M, K=K, N=N, rank=r, alpha=alpha,
        payload=rec.parts["payload"].numpy(), scales=rec.parts["scales"].numpy(),
        x_bf16=bits(x), A=A.numpy(), B=B.numpy(), dY_bf16=bits(dY),
        Y_bf16=bits(y.detach()), dX_bf16=bits(dx), dA=da.numpy(), dB=db.numpy())


def moe_case():
    T, H, I, E, top_k = 24, 128, 128, 6, 2
    g = torch.Generator().manual_seed(23)
    hidden = torch.randn(2, T // 2, H, generator=g)
    hidden[..., 0] = 3.0
    hidden = hidden.to(torch.bfloat16)
    gate = torch.randn(E, H, generator=g) * 0.3
    gate[5, 0] = -5.0  # expert 5 never reaches the top-2
    gate = gate.to(torch.bfloat16)
    gate_up = torch.randn(E, 2 * I, H, generator=g) * 0.05
    down = torch.randn(E, H, I, generator=g) * 0.05
    rec_gu = codecs.encode(gate_up.contiguous(), "int4-sym-g128")
    rec_dn = codecs.encode(down.contiguous(), "int4-sym-g128")
    weights = {"mlp.gate.weight": gate, "mlp.experts.gate_up_proj": codecs.materialize(rec_gu),
               "mlp.experts.down_proj": codecs.materialize(rec_dn)}
    h = hidden.clone().requires_grad_(True)
    out = moe_feed_forward(h, weights, num_experts=E, top_k=top_k, norm_topk_prob=True)
    dout = torch.randn(out.shape, generator=g).to(torch.bfloat16)
    (dh,) = torch.autograd.grad(out, (h,), dout)
    np.savez_compressed(
        os.path.join(HERE, "moe_small.npz"),
        T=T, H=H, I=I, E=E, top_k=top_k, norm_topk_prob=1,
        hidden_bf16=bits(hidden), gate_bf16=bits(gate),
        gate_up_payload=rec_gu.parts["payload"].numpy(), gate_up_scales=rec_gu.parts["scales"].numpy(),
        down_payload=rec_dn.parts["payload"].numpy(), down_scales=rec_dn.parts["scales"].numpy(),
        out_bf16=bits(out.detach()), dout_bf16=bits(dout), dhidden_bf16=bits(dh))

    # DeepSeek-V3 router: 16 experts in 4 groups, 2 groups kept, top-4.
    T, H, E = 32, 64, 16
    flat = (torch.randn(T, H, generator=g)).to(torch.bfloat16)
    wr = torch.randn(E, H, generator=g) * 0.2
    bias = torch.randn(E, generator=g) * 0.1
    _, rw, ri = deepseek_route(flat, wr, bias, groups=4, group_k=2, top_k=4, normalize=True, scale=2.5)
    order = torch.argsort(ri, dim=-1)
    np.savez_compressed(
        os.path.join(HERE, "deepseek_route.npz"),
        flat_bf16=bits(flat), weight=wr.numpy(), bias=bias.numpy(), groups=4, group_k=2, top_k=4,
        scale=2.5, indices=torch.gather(ri, 1, order).numpy(), weights=torch.gather(rw, 1, order).numpy())


def head_case():
    Bsz, S, H, V, chunk = 2, 70, 128, 512, 32
    g = torch.Generator().manual_seed(31)
    normalized = torch.randn(Bsz, S, H, generator=g).to(torch.bfloat16)
    head = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16)
    labels = torch.randint(0, V, (Bsz, S), generator=g)
    labels[torch.rand(Bsz, S, generator=g) < 0.25] = -100
    labels[:, 33:50] = -100  # a whole chunk with no supervised token is skipped
    norm = float((labels[:, 1:] != -100).sum())
    x = normalized.clone().requires_grad_(True)
    loss = chunked_causal_loss(x, head, labels, normalization=norm, token_chunk=chunk)
    (dx,) = torch.autograd.grad(loss, (x,))
    np.savez_compressed(
        os.path.join(HERE, "head_small.npz"), B=Bsz, S=S, H=H, V=V, token_chunk=chunk, normalization=norm,
        normalized_bf16=bits(normalized), head_bf16=bits(head), labels=labels.numpy(),
        loss=np.float32(loss.detach()), dnormalized_bf16=bits(dx))


def _all7_factory():
    """A registered adapter (the reference's extension API, adapters/registry.py:6-14)
    that is the stock Llama adapter with LoRA on all seven projections: the
    reference's target list is switched to the seven targets while the adapter
    builds its blocks (create_lora_for_block, finetune/lora.py:319-388), and each
    block's functional becomes a restatement of dense_block (adapters/dense.py:
    120-153) that routes every projection through its LoRAProjection.forward."""
    import torch.nn.functional as F
    from ram_vram_finetune.adapters import targets as tg
    from ram_vram_finetune.adapters.dense import LlamaAdapter, rms

    def block7(hidden_states, position_embeddings, attention_mask, *, heads, kv_heads, head_dim, eps, lora_q,
               lora_k, lora_v, lora_o, lora_gate, lora_up, lora_down, qk_norm=False, **weights):
        def linear(x, path, lora):
            return lora.forward(x, weights[path + ".weight"], weights.get(path + ".bias"))
        residual = hidden_states
        x = rms(hidden_states, weights["input_layernorm.weight"], eps)
        shape = (*x.shape[:-1], -1, head_dim)
        q = linear(x, "self_attn.q_proj", lora_q).view(shape)
        k = linear(x, "self_attn.k_proj", lora_k).view(shape)
        v = linear(x, "self_attn.v_proj", lora_v).view(shape).transpose(1, 2)
        q, k = q.transpose(1, 2), k.transpose(1, 2)
        cos, sin = (value.unsqueeze(1) for value in position_embeddings)

        def rotate(t):
            left, right = t.chunk(2, dim=-1)
            return t * cos + torch.cat((-right, left), dim=-1) * sin
        q, k = rotate(q), rotate(k)

        def repeat(t):
            b, h, s_, d = t.shape
            return t[:, :, None].expand(b, h, heads // kv_heads, s_, d).reshape(b, heads, s_, d)
        k, v = repeat(k), repeat(v)
        scores = (q @ k.transpose(-2, -1)) * head_dim ** -0.5
        probabilities = torch.softmax(scores + attention_mask, dim=-1, dtype=torch.float32).to(q.dtype)
        attended = (probabilities @ v).transpose(1, 2).contiguous().reshape(*x.shape[:-1], heads * head_dim)
        x = residual + linear(attended, "self_attn.o_proj", lora_o)
        residual = x
        x = rms(x, weights["post_attention_layernorm.weight"], eps)
        return residual + linear(F.silu(linear(x, "mlp.gate_proj", lora_gate)) * linear(x, "mlp.up_proj", lora_up),
                                 "mlp.down_proj", lora_down)

    def factory(path, **kwargs):
        saved = tg.ATTENTION_TARGETS["full_attention"]
        tg.ATTENTION_TARGETS["full_attention"] = e2e_tiny.ALL7
        try:
            adapter = LlamaAdapter(path, **kwargs)
        finally:
            tg.ATTENTION_TARGETS["full_attention"] = saved
        for block in adapter.blocks:
            block.functional = block7
            for key, path_ in (("lora_k", "self_attn.k_proj"), ("lora_gate", "mlp.gate_proj"),
                               ("lora_up", "mlp.up_proj"), ("lora_down", "mlp.down_proj")):
                block.kwargs[key] = block.adapters[path_]
        return adapter
    return factory


def tiny_llama_training(targets="qvo"):
    """The reference engine on the tiny Llama (see tests/e2e_tiny.py); targets
    "qvo" uses the stock llama adapter (LoRA on q, v, o), "all7" a registered
    adapter with LoRA on all seven projections (the tiny-Llama training configuration)."""
    import json
    import tempfile
    from safetensors.torch import save_file
    from transformers.models.llama.configuration_llama import LlamaConfig
    from ram_vram_finetune.config import TrainConfig
    from ram_vram_finetune.training import engine
    t = e2e_tiny
    tmp = tempfile.mkdtemp(prefix="tiny_llama_")
    model = os.path.join(tmp, "model")
    os.makedirs(model)
    cfg = LlamaConfig(vocab_size=t.VOCAB, hidden_size=t.HIDDEN, intermediate_size=t.INTER,
                      num_hidden_layers=t.LAYERS, num_attention_heads=t.HEADS, num_key_value_heads=t.KV_HEADS,
                      head_dim=t.HEAD_DIM, max_position_embeddings=t.MAX_POS, rms_norm_eps=t.EPS,
                      attention_dropout=0.0, tie_word_embeddings=False, use_cache=False,
                      rope_parameters={"rope_type": "default", "rope_theta": t.THETA})
    with open(os.path.join(model, "config.json"), "w") as f:
        f.write(json.dumps(cfg.to_dict(), indent=2) + "\n")
    state = {k: v.contiguous() for k, v in t.model_state().items()}
    save_file(state, os.path.join(model, "model.safetensors"))
    dataset = os.path.join(tmp, "rows.jsonl")
    with open(dataset, "w") as f:
        for ids, labels in t.token_rows():
            f.write(json.dumps({"input_ids": ids[0].tolist(), "labels": labels[0].tolist()}) + "\n")
    adapter_name = "llama"
    if targets == "all7":
        from ram_vram_finetune.adapters.registry import register
        adapter_name = "tiny_llama_all7"
        register(adapter_name, _all7_factory())
    config = TrainConfig(model=model, dataset=dataset, output=os.path.join(tmp, "out"), adapter=adapter_name,
                         device="cpu", steps=t.STEPS, accumulation=t.ACCUM, rank=t.RANK, alpha=t.ALPHA,
                         learning_rate=t.LR, weight_decay=0.0, seed=t.SEED, token_chunk=t.TOKEN_CHUNK,
                         max_sequence_length=t.SEQ, checkpoint_every=10 ** 6, quantization="int4-sym-g128")
    out = {}

    def capture(event, data):
        adapter = data.get("adapter")
        projs = {f"{b.index}:{name}": p for b in adapter.blocks for name, p in b.adapters.items()} if adapter else {}
        if event == "adapter_ready":
            for k, p in projs.items():
                out[f"{k}/A0_sum"] = np.float64(p.A.detach().double().sum())
                out[f"{k}/A0_head"] = p.A.detach()[0, :8].numpy().copy()
        elif event == "step" and data["metrics"]["step"] in (1, 2):
            st = data["metrics"]["step"]
            for k, p in projs.items():
                out[f"{k}/step{st}_grad_A"] = p.grad_A.numpy().copy()
                out[f"{k}/step{st}_grad_B"] = p.grad_B.numpy().copy()
        elif event == "training_complete":
            for k, p in projs.items():
                out[f"{k}/final_A"] = p.A.detach().numpy().copy()
                out[f"{k}/final_B"] = p.B.detach().numpy().copy()

    report = engine.run(config, progress_callback=capture)
    assert report["status"] == "completed"
    losses = np.array([m["loss"] for m in report["metrics"]], dtype=np.float64)
    name = "tiny_llama_train.npz" if targets == "qvo" else "tiny_llama_train_all7.npz"
    np.savez_compressed(os.path.join(HERE, name), losses=losses, **out)
    print("tiny llama", targets, "losses", losses[:3], "...", losses[-3:], file=sys.stderr)


CASES = {"codec": codec_cases, "lora": lora_case, "moe": moe_case, "head": head_case,
         "tiny_llama": tiny_llama_training, "tiny_llama_all7": lambda: tiny_llama_training("all7")}

if __name__ == "__main__":
    # `make_golden.py [case ...]` regenerates only the named fixtures (all by default).
    torch.set_num_threads(1)
    for name in sys.argv[1:] or list(CASES):
        CASES[name]()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")), file=sys.stderr)
