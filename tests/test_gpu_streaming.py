"""PackedSlotSession on one GPU (the reference's SlotSession/PrefetchSession
contract, memory.py:188-275 and prefetch.py:47-252): every borrowed view holds
the host record byte for byte, in forward order (prefetch +1) and backward
order (prefetch -1), through slot reuse; and a fused projection computed from
a borrowed slot equals the same call on a resident copy of the record, which
shows the compute stream waited for the copy stream's ready event."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _layers(n_layers, seed=5):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n_layers):
        layer = {name: codec.encode(torch.randn(n, k, generator=g) * 0.02, "nf4-g128")
                 for name, n, k in (("q", 512, 384), ("k", 128, 384), ("down", 384, 2048))}
        out.append({k: w.to("cpu").pin_memory() for k, w in layer.items()})
    return out


def test_slot_views_match_host_records_and_feed_the_kernels(cuda_lib):
    from spilltune_b200 import ops
    from spilltune_b200.streaming import PackedSlotSession
    n = 5
    layers = _layers(n)
    resident = [{k: w.to("cuda") for k, w in layer.items()} for layer in layers]
    x = {k: torch.randn(64, w.shape[1]).to(torch.bfloat16).cuda() for k, w in layers[0].items()}
    sess = PackedSlotSession(layers, torch.device("cuda"), slots=2)
    order = [(i, "forward") for i in range(n)] + [(i, "backward") for i in reversed(range(n))]
    mismatches = []
    for idx, phase in order:
        with sess.borrow(idx, phase) as views:
            # Work enqueued on the compute stream right after the borrow reads the slot.
            outs = {k: ops.fwd(x[k], views[k]) for k in views}
            for name, w in layers[idx].items():
                v = views[name]
                if not (torch.equal(v.payload.cpu(), w.payload) and torch.equal(v.scales.cpu(), w.scales)
                        and torch.equal(v.lut.cpu(), w.lut)):
                    mismatches.append((idx, phase, name))
            for k, y in outs.items():
                if not torch.equal(y, ops.fwd(x[k], resident[idx][k])):
                    mismatches.append((idx, phase, k, "output"))
    torch.cuda.synchronize()
    assert not mismatches
    # Only layer 0's first borrow loads on demand; every other borrow finds its
    # layer already prefetched.  Uploads: layer 0 + four forward prefetches +
    # three backward prefetches (layers 3 and 4 are still in the two slots
    # when the backward starts).
    assert sess.hits == len(order) - 1
    assert sess.uploads == 2 * n - 2
    sess.close()
