"""Slot-streaming host logic (victim choice, prefetch order, poisoning) without a GPU.

torch.cuda streams/events are replaced by recording fakes, as the reference's
tests/test_prefetch.py does with monkeypatch.
"""
import contextlib

import pytest
import torch

from spilltune_b200 import codec, streaming


class _FakeEvent:
    def __init__(self, *a, **k):
        self.recorded = 0

    def record(self, stream=None):
        self.recorded += 1

    def synchronize(self):
        pass

    def elapsed_time(self, other):
        return 1.0


class _FakeStream:
    def __init__(self, *a, **k):
        self.waits = []

    def wait_event(self, ev):
        self.waits.append(ev)

    def wait_stream(self, s):
        pass


@pytest.fixture
def fake_cuda(monkeypatch):
    compute = _FakeStream()
    monkeypatch.setattr(torch.cuda, "Stream", _FakeStream)
    monkeypatch.setattr(torch.cuda, "Event", _FakeEvent)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda device=None: compute)
    monkeypatch.setattr(torch.cuda, "stream", lambda s: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "device", lambda d: contextlib.nullcontext())
    monkeypatch.setattr(torch.cuda, "synchronize", lambda d=None: None)
    real_empty = torch.empty

    def empty(*a, device=None, **k):
        return real_empty(*a, **k)

    monkeypatch.setattr(torch, "empty", empty)
    monkeypatch.setattr(torch.Tensor, "is_pinned", lambda self: True)
    return compute


def _layers(n):
    out = []
    for i in range(n):
        w = codec.encode_int4_sym(torch.full((64, 256), float(i + 1)) * 0.01)
        out.append({"q": w})
    return out


def test_prefetch_order_and_reuse(fake_cuda):
    layers = _layers(4)
    sess = streaming.PackedSlotSession(layers, "cuda:0", slots=2)
    loaded = []
    orig = sess._enqueue

    def spy(idx, slot):
        loaded.append(idx)
        return orig(idx, slot)

    sess._enqueue = spy
    for l in range(4):
        with sess.borrow(l, "forward") as W:
            assert torch.equal(W["q"].payload, layers[l]["q"].payload)
    for l in reversed(range(4)):
        with sess.borrow(l, "backward") as W:
            assert torch.equal(W["q"].scales, layers[l]["q"].scales)
    # forward loads 0 and prefetches 1..3; backward reuses 3 and 2, reloads 1 and 0.
    assert loaded == [0, 1, 2, 3, 1, 0]
    assert sess.hits == 7 and sess.uploads == 6  # only the very first borrow misses


def test_reentrant_borrow_rejected_and_poison(fake_cuda):
    sess = streaming.PackedSlotSession(_layers(2), "cuda:0", slots=2)
    with sess.borrow(0, "forward"):
        with pytest.raises(RuntimeError, match="reentrant"):
            with sess.borrow(1, "forward"):
                pass
    with pytest.raises(ValueError):
        with sess.borrow(0, "forward"):
            raise ValueError("consumer failed")
    with pytest.raises(RuntimeError, match="poisoned"):
        with sess.borrow(0, "forward"):
            pass


def test_unpinned_sources_rejected(fake_cuda, monkeypatch):
    monkeypatch.setattr(torch.Tensor, "is_pinned", lambda self: False)
    with pytest.raises(ValueError, match="pinned"):
        streaming.PackedSlotSession(_layers(2), "cuda:0", slots=2)


def test_shard_images_reassemble_the_slot_image():
    """With a process group each rank keeps bytes [r*S, (r+1)*S) of a layer's slot image; the
    all-gathered shards must give back every part at the offset the slot views read it from."""
    from spilltune_b200 import codec
    from spilltune_b200.streaming import _parts, layer_bytes, shard_image
    g = torch.Generator().manual_seed(5)
    layer = {name: codec.encode(torch.randn(n, k, generator=g) * 0.02, "nf4-g128")
             for name, n, k in (("q", 256, 384), ("k", 128, 384), ("down", 384, 256))}
    for world in (2, 3, 8):
        step = world * 256
        cap = (layer_bytes(layer) + step - 1) // step * step
        shard = cap // world
        image = torch.cat([shard_image(layer, r * shard, shard) for r in range(world)])
        assert image.numel() == cap
        end = 0
        for off, b in _parts(layer):
            assert torch.equal(image[off:off + b.numel()], b)
            end = off + b.numel()
        assert int(image[end:].count_nonzero()) == 0  # padding past the last part
