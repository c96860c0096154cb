"""Sharded slot streaming (PackedSlotSession with a process group): every rank copies
1/W of each layer from pinned host memory and the slot is all-gathered over NCCL.
Checked on two GPUs: every borrowed view equals the host record byte for byte, in
forward and backward order (prefetch, slot reuse).  Skipped with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layers(n_layers):
    from spilltune_b200 import codec
    g = torch.Generator().manual_seed(11)
    out = []
    for _ in range(n_layers):
        layer = {name: codec.encode(torch.randn(n, k, generator=g) * 0.02, "nf4-g128")
                 for name, n, k in (("q", 512, 384), ("k", 128, 384), ("down", 384, 640))}
        out.append({k: w.to("cpu").pin_memory() for k, w in layer.items()})
    return out


def _worker(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    from spilltune_b200.streaming import PackedSlotSession
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = True
    try:
        layers = _layers(5)
        group = dist.new_group(backend="nccl")
        sess = PackedSlotSession(layers, torch.device("cuda", rank), slots=2, group=group)
        order = [(i, "forward") for i in range(5)] + [(i, "backward") for i in reversed(range(5))]
        for idx, phase in order:
            with sess.borrow(idx, phase) as views:
                for name, w in layers[idx].items():
                    v = views[name]
                    ok &= torch.equal(v.payload.cpu(), w.payload)
                    ok &= torch.equal(v.scales.cpu(), w.scales)
                    ok &= torch.equal(v.lut.cpu(), w.lut)
        ok &= sess.h2d_bytes == sess.uploads * sess.shard
        sess.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write("ok" if ok else "mismatch")


def test_sharded_slots_match_host_records(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert [(tmp_path / f"rank{r}").read_text() for r in range(2)] == ["ok", "ok"]
