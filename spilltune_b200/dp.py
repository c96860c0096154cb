"""Data parallelism over the token batch for the frozen-linear trainer.

The reference trains on one device (config accepts ``cpu|cuda:0``,
ram_vram_finetune/config.py:52-53) and normalises the loss per accumulation
window (training/engine.py:166-167).  Across N data-parallel ranks:

* every rank streams the same frozen layers and runs its own micro-batches:
  rank r takes micro-batches r, r+N, r+2N, ... of the accumulation window
  (``shard_microbatches``);
* the loss is normalised by the GLOBAL supervised-token count
  (``global_token_count``), so the summed gradients equal the single-device
  gradient of the whole window;
* the only exchange is the LoRA gradients (FP32 grad_A / grad_B): one bucket
  per layer, all-reduced (sum) as soon as that layer's backward has produced
  it, on a side stream that overlaps the next layer's recompute and backward
  (``LoRAGradReducer``).  AdamW then runs replicated on identical gradients.

The frozen weights and the fused kernels need no collective.  With NCCL the
all-reduce runs over NVLink / NVSwitch; the same code runs on CPU ranks with
gloo (synchronously), which is how the host logic is tested.
"""
import torch
import torch.distributed as dist


def world():
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


def rank():
    return dist.get_rank() if dist.is_available() and dist.is_initialized() else 0


def shard_microbatches(n_micro, rank_, world_):
    """Indices of the micro-batches of one accumulation window that `rank_` runs."""
    if world_ < 1 or not 0 <= rank_ < world_:
        raise ValueError("invalid data-parallel rank/world")
    return list(range(rank_, n_micro, world_))


def global_token_count(local_count, group=None, device=None):
    """Sum of supervised tokens over all ranks (the loss normaliser)."""
    if world() == 1:
        return int(local_count)
    t = torch.tensor([int(local_count)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return int(t.item())


class LoRAGradReducer:
    """Sums (or averages) LoRA gradient buckets across ranks, one bucket per call.

    ``reduce(grads)`` enqueues the reduction of a list of gradient tensors
    (e.g. every grad_A / grad_B of one layer) and returns immediately on CUDA;
    ``finish()`` makes the current stream wait for every pending bucket.  On
    CPU tensors (gloo) the reduction completes inside ``reduce``.
    """

    def __init__(self, group=None, average=False):
        self.group = group
        self.average = average
        self.world = world() if group is None else dist.get_world_size(group)
        self._stream = None
        self._pending = []
        self.buckets = 0
        self.bytes = 0

    def _comm_stream(self, device):
        if self._stream is None:
            self._stream = torch.cuda.Stream(device=device)
        return self._stream

    def reduce(self, grads):
        grads = [g for g in grads if g is not None]
        if not grads or self.world == 1:
            return
        dev = grads[0].device
        n = sum(g.numel() for g in grads)
        self.buckets += 1
        self.bytes += 4 * n
        if dev.type == "cuda":
            stream = self._comm_stream(dev)
            stream.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(stream):
                flat = torch.cat([g.reshape(-1).float() for g in grads])
                dist.all_reduce(flat, group=self.group)
                if self.average:
                    flat.div_(self.world)
                off = 0
                for g in grads:
                    g.copy_(flat[off:off + g.numel()].view_as(g))
                    off += g.numel()
            # Keep the bucket alive until the stream is done with it.
            flat.record_stream(stream)
            self._pending.append(flat)
        else:
            flat = torch.cat([g.reshape(-1).float() for g in grads])
            dist.all_reduce(flat, group=self.group)
            if self.average:
                flat.div_(self.world)
            off = 0
            for g in grads:
                g.copy_(flat[off:off + g.numel()].view_as(g))
                off += g.numel()

    def finish(self):
        if self._stream is not None:
            torch.cuda.current_stream(self._stream.device).wait_stream(self._stream)
        self._pending.clear()
