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
"""
import os
import sys

import numpy as np
import torch

from ram_vram_finetune.quantization import codecs
from ram_vram_finetune.finetune.lora import LoRAProjection

HERE = os.path.dirname(os.path.abspath(__file__))


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


if __name__ == "__main__":
    torch.set_num_threads(1)
    codec_cases()
    lora_case()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")), file=sys.stderr)
