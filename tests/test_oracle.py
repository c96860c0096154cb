"""The CPU oracle is pinned to the reference before anything is checked against it.

Golden vectors come from importing the reference itself (tests/golden/make_golden.py);
the known-answer vector is the reference's own tests/test_quantization.py:73-81.
"""
import numpy as np
import pytest
import torch

import oracle.codec as oc
import oracle.linear as ol

GOLD = "tests/golden/"


def _load(name):
    import os
    return np.load(os.path.join(os.path.dirname(__file__), "golden", name))


def _bf16(a, shape):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).view(*shape)


def test_codec_matches_reference_golden():
    d = _load("codec_int4.npz")
    names = sorted({k.split("/")[0] for k in d.files})
    assert names == ["kat", "len128", "len129", "len257", "mat32x256"]
    for n in names:
        x = d[n + "/input"]
        p, s = oc.encode_int4_sym(x)
        assert np.array_equal(p, d[n + "/payload"]), n
        assert np.array_equal(s, d[n + "/scales"]), n
        assert np.array_equal(oc.decode(p, s, x.size), d[n + "/decoded_bf16"]), n
        assert oc.validate_int4_sym(p, s, x.size) == 0


def test_known_answer_vector():
    v = np.zeros(128, np.float32)
    v[:6] = [-7, -1.5, -.5, .5, 1.5, 7]
    p, s = oc.encode_int4_sym(v)
    assert p[:3].tolist() == [0x61, 0x88, 0xFA]
    assert s[0] == 1
    assert oc.bf16_bits_to_f32(oc.decode(p, s, 128))[:6].tolist() == [-7, -2, 0, 0, 2, 7]


def test_tail_zero_group_and_threaded_decode():
    rng = np.random.default_rng(3)
    for n in (1, 127, 128, 129, 1000, 70001):
        x = rng.standard_normal(n).astype(np.float32) * 0.02
        x[: min(n, 128)] = 0
        p, s = oc.encode_int4_sym(x)
        assert s[0] == 1.0
        a = oc.decode(p, s, n)
        assert np.array_equal(a, oc.decode(p, s, n, threads=4))
        # padding codes decode to zero (code 8)
        tail = (len(p) * 2) - n
        if tail:
            codes = np.stack([p & 15, p >> 4], 1).reshape(-1)
            assert (codes[n:] == 8).all()


def test_validate_rejections():
    p, s = oc.encode_int4_sym(np.ones(129, np.float32))
    assert oc.validate_int4_sym(p, s, 129) == 0
    bad = p.copy(); bad[0] = 0
    assert oc.validate_int4_sym(bad, s, 129) == 1
    bad = p.copy(); bad[-1] ^= 1
    assert oc.validate_int4_sym(bad, s, 129) == 2
    sc = s.copy(); sc[0] = 0
    assert oc.validate_int4_sym(p, sc, 129) == 3
    sc = s.copy(); sc[:] = 1e38
    assert oc.validate_int4_sym(p, sc, 129) == 4


def test_nf4_codebook_matches_published_construction():
    assert np.abs(oc.nf4_construction() - oc.NF4_LUT).max() < 1e-6
    assert oc.NF4_LUT[0] == -1 and oc.NF4_LUT[7] == 0 and oc.NF4_LUT[15] == 1


def test_nf4_encode_roundtrip():
    rng = np.random.default_rng(5)
    x = rng.standard_normal(4096).astype(np.float32) * 0.02
    p, s = oc.encode_nf4(x)
    dec = oc.bf16_bits_to_f32(oc.decode(p, s, x.size, lut=oc.NF4_LUT))
    # each element decodes to the nearest codebook point times the absmax scale
    assert np.abs(dec - x).max() <= 0.17 * np.abs(x).max() + 1e-6
    assert np.array_equal(s, np.abs(x.reshape(-1, 128)).max(1))


def test_lora_oracle_matches_reference_golden():
    g = _load("lora_small.npz")
    M, K, N, r, alpha = [g[k].item() for k in ("M", "K", "N", "rank", "alpha")]
    W = _bf16(oc.decode(g["payload"], g["scales"], N * K), (N, K))
    x = _bf16(g["x_bf16"], (M, K))
    dY = _bf16(g["dY_bf16"], (M, N))
    A, B = torch.from_numpy(g["A"]), torch.from_numpy(g["B"])
    y, dx, da, db = ol.lora_backward_reference(x, W, A, B, alpha / r, dY)
    assert torch.equal(y, _bf16(g["Y_bf16"], (M, N)))
    assert torch.equal(dx, _bf16(g["dX_bf16"], (M, K)))
    assert torch.equal(da, torch.from_numpy(g["dA"]))
    assert torch.equal(db, torch.from_numpy(g["dB"]))
    # The fp32 shadow the kernels are graded against agrees within the bar.
    dx32, da32, db32 = ol.lora_backward_fp32(x, W, A, B, alpha / r, dY)
    assert ol.rel_l2(dx, dx32) < 1e-2 and ol.rel_l2(da, da32) < 1e-5 and ol.rel_l2(db, db32) < 1e-5
    assert ol.rel_l2(y, ol.lora_forward_fp32(x, W, A, B, alpha / r)) < 1e-2


def test_torch_decode_matches_reference_golden():
    """oracle.codec.decode_torch (the reference's decode_into as torch ops, used
    as the reference path in bench.py) gives the reference's own decoded bits."""
    import torch
    g = _load("codec_int4.npz")
    for name in ("len128", "len129", "len257", "kat", "mat32x256"):
        x = g[f"{name}/input"]
        out = torch.empty(x.size, dtype=torch.bfloat16)
        oc.decode_torch(torch.from_numpy(g[f"{name}/payload"]), torch.from_numpy(g[f"{name}/scales"]), x.size,
                        torch.arange(16, dtype=torch.float32) - 8.0, out)
        assert np.array_equal(out.view(torch.int16).numpy().view(np.uint16), g[f"{name}/decoded_bf16"]), name
