"""Data-parallel host logic on two CPU ranks (gloo), no GPU.

Checks that the per-layer LoRA gradient buckets are summed across ranks, that
micro-batches are sharded without overlap, that the global token count
normalises the loss so the DP gradient equals the single-process gradient of
the whole window, and that a rank that dies is detected by the others through
a short process-group timeout rather than hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _worker_reduce(rank, world, port, q):
    try:
        _init(rank, world, port)
        from spilltune_b200.dp import LoRAGradReducer, shard_microbatches, global_token_count
        torch.manual_seed(0)
        # Per-layer buckets of grad_A [r, K] / grad_B [N, r]: rank-dependent values.
        layers = [[torch.full((4, 16), float(rank + 1 + l)), torch.full((24, 4), float(10 * (rank + 1) + l))]
                  for l in range(3)]
        red = LoRAGradReducer()
        for grads in reversed(layers):
            red.reduce(grads)
        red.finish()
        out = {"grads": [[g.clone() for g in gl] for gl in layers], "buckets": red.buckets, "bytes": red.bytes}
        # Sharding + global normalisation: window of 5 micro-batches, token counts differ.
        counts = [7, 3, 11, 5, 2]
        mine = shard_microbatches(len(counts), rank, world)
        out["mine"] = mine
        out["global_tokens"] = global_token_count(sum(counts[i] for i in mine))
        # DP gradient of a linear loss w.x summed over tokens / global tokens.
        w = torch.zeros(8, requires_grad=True)
        g_data = torch.Generator().manual_seed(1)
        xs = [torch.randn(c, 8, generator=g_data) for c in counts]
        loss = sum((xs[i] @ w).sum() for i in mine) / out["global_tokens"]
        loss.backward()
        dist.all_reduce(w.grad)
        out["dp_grad"] = w.grad.clone()
        out["ref_grad"] = torch.cat(xs).sum(0) / sum(counts)
        # Plain NumPy copies: torch tensors put on a queue travel as shared-memory
        # handles, which vanish if this process exits before the parent reads them.
        out["grads"] = [[g.numpy() for g in gl] for gl in out["grads"]]
        out["dp_grad"], out["ref_grad"] = out["dp_grad"].numpy(), out["ref_grad"].numpy()
        q.put((rank, out))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_two_rank_gradient_reduction_sharding_and_normalisation():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_reduce, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in (0, 1):
        out = res[r]
        assert out["buckets"] == 3 and out["bytes"] == 3 * 4 * (64 + 96)
        for l, (ga, gb) in enumerate(out["grads"]):
            assert torch.equal(torch.from_numpy(ga), torch.full((4, 16), float(1 + l + 2 + l)))  # (1+l) + (2+l)
            assert torch.equal(torch.from_numpy(gb), torch.full((24, 4), float(10 + l + 20 + l)))
        assert out["global_tokens"] == 28
        assert torch.allclose(torch.from_numpy(out["dp_grad"]), torch.from_numpy(out["ref_grad"]), atol=1e-6)
    assert sorted(res[0]["mine"] + res[1]["mine"]) == [0, 1, 2, 3, 4]
    assert not set(res[0]["mine"]) & set(res[1]["mine"])


def _worker_dead_peer(rank, world, port, q):
    _init(rank, world, port, timeout_s=3)
    # One complete step first, so the group is fully connected before a rank
    # leaves (a rank that leaves during rendezvous tests something else).
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == 1:
        # This rank leaves between steps without joining the next collective.
        os._exit(0)
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # gloo reports the missing peer (timeout / connection closed)
        q.put((rank, type(e).__name__))
    finally:
        # Queue.put hands the item to a feeder thread: flush it before the
        # hard exit, or the parent may never receive it.
        q.close()
        q.join_thread()
        os._exit(0)


def test_dead_peer_is_detected_by_timeout():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_dead_peer, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, what = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
    assert rank == 0 and what != "no error"


def test_shard_rejects_bad_rank():
    from spilltune_b200.dp import shard_microbatches
    with pytest.raises(ValueError):
        shard_microbatches(4, 2, 2)
    assert shard_microbatches(4, 0, 1) == [0, 1, 2, 3]
