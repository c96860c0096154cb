"""Host-side record handling of the product package, checked against the oracle."""
import numpy as np
import pytest
import torch

import oracle.codec as oc
from spilltune_b200 import codec


@pytest.mark.parametrize("shape", [(1, 128), (1, 129), (3, 257), (64, 384)])
def test_host_int4_encoder_matches_oracle(shape):
    g = torch.Generator().manual_seed(sum(shape))
    w = torch.randn(*shape, generator=g) * 0.03
    w[0, :64] = 0
    pw = codec.encode_int4_sym(w)
    p, s = oc.encode_int4_sym(w.numpy())
    assert np.array_equal(pw.payload.numpy(), p)
    assert np.array_equal(pw.scales.numpy(), s)


@pytest.mark.parametrize("shape", [(2, 256), (5, 129)])
def test_host_nf4_encoder_matches_oracle(shape):
    g = torch.Generator().manual_seed(7)
    w = torch.randn(*shape, generator=g) * 0.02
    pw = codec.encode_nf4(w)
    p, s = oc.encode_nf4(w.numpy())
    assert np.array_equal(pw.payload.numpy(), p)
    assert np.array_equal(pw.scales.numpy(), s)
    assert torch.equal(pw.lut, torch.from_numpy(oc.NF4_LUT))


def test_from_record_wraps_reference_layout():
    d = np.load("tests/golden/codec_int4.npz")
    spec = {"version": 1, "shape": [32, 256], "dtype": "bfloat16", "codec": "int4-sym-g128",
            "group_size": 128, "numel": 32 * 256}
    parts = {"payload": torch.from_numpy(d["mat32x256/payload"]), "scales": torch.from_numpy(d["mat32x256/scales"])}
    pw = codec.from_record(spec, parts)
    assert pw.shape == (32, 256) and pw.codec == codec.INT4_SYM
    assert pw.payload.data_ptr() == parts["payload"].data_ptr()
    with pytest.raises(ValueError, match="unsupported_quantization"):
        codec.from_record(dict(spec, codec="int8-sym-g128"), parts)
    with pytest.raises(ValueError, match="payload"):
        codec.PackedWeight(parts["payload"][:-1], parts["scales"], codec.INT4_SYM_LUT, (32, 256))


@pytest.mark.parametrize("name", ["int4-sym-g128", "nf4-g128"])
def test_host_encoders_reject_what_the_reference_rejects(name):
    """As the reference's encoder does (its tests/test_quantization.py:114-136): a
    nonfinite input, and a value whose decoded BF16 would overflow, raise ValueError."""
    from spilltune_b200 import codec
    x = torch.ones(1, 128)
    x[0, 0] = float("nan")
    with pytest.raises(ValueError, match="nonfinite"):
        codec.encode(x, name)
    with pytest.raises(ValueError, match="BF16"):
        codec.encode(torch.full((1, 128), 3.4e38), name)
    codec.encode(torch.full((1, 128), 3.3e38), name)  # the largest values that still fit are kept


@pytest.mark.parametrize("name", ["int4-sym-g128", "nf4-g128"])
def test_validate_restates_the_reference_record_checks(name):
    """codec.validate raises what the reference's validate_spec raises
    (quantization/codecs.py:119-156) and accepts what the encoder produces."""
    from spilltune_b200 import codec
    w = codec.encode(torch.randn(3, 43) * 0.02, name)  # 129 elements: a ragged second group
    codec.validate(w)

    def broken(fn):
        b = codec.PackedWeight(w.payload.clone(), w.scales.clone(), w.lut.clone(), w.shape, w.codec)
        fn(b)
        return b

    with pytest.raises(ValueError, match="invalid stored scales"):
        codec.validate(broken(lambda b: b.scales.__setitem__(0, 0.0)))
    with pytest.raises(ValueError, match="invalid stored scales"):
        codec.validate(broken(lambda b: b.scales.__setitem__(1, float("inf"))))
    with pytest.raises(ValueError, match="padding"):
        codec.validate(broken(lambda b: b.payload.__setitem__(-1, int(b.payload[-1]) ^ 0x10)))
    with pytest.raises(ValueError, match="BF16"):
        codec.validate(broken(lambda b: b.scales.fill_(3.4e38)))
    if name == "int4-sym-g128":
        with pytest.raises(ValueError, match="reserved"):
            codec.validate(broken(lambda b: b.payload.__setitem__(0, int(b.payload[0]) & 0xF0)))
        # Exact overflow rule: a scale at which code -8 would overflow is fine when the
        # group's largest stored magnitude (7) does not.
        ok = codec.encode(torch.full((1, 128), 3.0e38), name)
        codec.validate(ok)
