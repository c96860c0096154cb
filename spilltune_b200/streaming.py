"""Packed-weight layer-slot streaming: pinned host records -> bounded VRAM slots.

B200 counterpart of the reference's ``SlotSession.load`` (ram_vram_finetune/
memory.py:188-275) and ``PrefetchSession`` (ram_vram_finetune/prefetch.py:47-252),
extended to the compressed blocks ``PrefetchSession`` refuses today
(prefetch.py:57-60):

* the packed parts (payload + scales + codebook per projection) are copied as
  they are stored — no decoded BF16 slot, no ``decode_into``: the fused
  kernels read the slot directly;
* copies run on a dedicated copy stream from pinned host memory, one layer
  ahead of the consumer (forward: +1, backward: -1, prefetch.py:203-207);
* a slot's ``ready`` event admits use on the compute stream (prefetch.py:197);
  its ``consumed`` event, recorded after the whole consumer scope, admits the
  next overwrite (prefetch.py:217-218);
* no device-wide synchronize on the load path (memory.py:204-206 does one per load).

With a process group (data parallel over the GPUs of one box), a rank keeps and
copies only its 1/W byte range of each layer's slot image, and the slot is
completed by an in-place NCCL all-gather over NVLink on the copy stream: host
traffic (and pinned host memory) per GPU drops W-fold, which matters because the
GPUs of a box share the host's memory bandwidth.  The group should be one of
its own (``torch.distributed.new_group``), so weight gathers never interleave
with other collectives on the same communicator.

Failures poison the session, like the reference's (prefetch.py:94-101).
"""
from contextlib import contextmanager
import threading

import torch

from .codec import PackedWeight, validate

_ALIGN = 256   # slot buffers and shard boundaries
_PART = 16     # parts inside a layer image (the kernels' operand alignment)


def _align(n, a=_ALIGN):
    return (n + a - 1) // a * a


def _layout(layer):
    """Slot-image layout of one layer (dict name -> PackedWeight), in order:
    every matrix's payload, then every matrix's scales, then every codebook,
    each part 16-byte aligned.  Group-128 records with K % 128 == 0 have
    payloads of N * K / 2 and scales of N * K / 32 bytes (multiples of 16), so
    matrices that follow each other in the layer (q, k, v; gate, up) sit back to
    back: their concatenation is itself a valid stacked record [N1 + N2 + ..., K]
    that one fused call can read (``ops.concat_records``).
    Returns [(name, part, offset, tensor)] and the image size (256-aligned)."""
    out, off = [], 0
    for part in ("payload", "scales", "lut"):
        for name, w in layer.items():
            t = getattr(w, part)
            off = _align(off, _PART)
            out.append((name, part, off, t))
            off += t.numel() * t.element_size()
    return out, _align(off)


def layer_bytes(layer):
    """Slot bytes for one layer (dict name -> PackedWeight)."""
    return _layout(layer)[1]


def _parts(layer):
    """(slot offset, byte view) of every part of a layer, in slot-image order."""
    return [(off, t.reshape(-1).view(torch.uint8)) for _name, _part, off, t in _layout(layer)[0]]


def layer_views(buf, layer):
    """{name: PackedWeight} views of a layer image in `buf` (uint8, any device)."""
    parts = {}
    for name, part, off, t in _layout(layer)[0]:
        n = t.numel() * t.element_size()
        parts.setdefault(name, {})[part] = buf.narrow(0, off, n).view(t.dtype)
    return {name: PackedWeight(parts[name]["payload"], parts[name]["scales"], parts[name]["lut"], w.shape, w.codec)
            for name, w in layer.items()}


def pack_layer(layer, device):
    """One layer copied into a single device buffer laid out like a slot image;
    returns (buffer, {name: PackedWeight views}).  Resident layers packed this
    way can run fused calls over adjacent matrices, like streamed slots."""
    buf = torch.empty(layer_bytes(layer), dtype=torch.uint8, device=device)
    for off, b in _parts(layer):
        buf.narrow(0, off, b.numel()).copy_(b, non_blocking=True)
    return buf, layer_views(buf, layer)


def shard_image(layer, start, size, out=None):
    """Bytes [start, start + size) of the layer's slot image (zero past its parts), as a CPU tensor."""
    if out is None:
        out = torch.zeros(size, dtype=torch.uint8)
    else:
        out.zero_()
    for off, b in _parts(layer):
        lo, hi = max(off, start), min(off + b.numel(), start + size)
        if lo < hi:
            out[lo - start:hi - start].copy_(b[lo - off:hi - off])
    return out


class PackedSlotSession:
    """Two (or more) device slots fed from pinned host layers on a copy stream."""

    def __init__(self, layers, device, *, slots=2, copy_stream=None, group=None):
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("unsupported_capability: slot streaming needs a CUDA device")
        if not layers:
            raise ValueError("slot streaming needs a nonempty ordered layer plan")
        if slots < 2 and len(layers) > 1:
            raise MemoryError("resource_budget: prefetch requires two slots for a multi-layer plan")
        for layer in layers:
            for name, w in layer.items():
                if not isinstance(w, PackedWeight):
                    raise TypeError(f"{name}: slot layers hold PackedWeight records")
                for t in (w.payload, w.scales, w.lut):
                    if t.device.type != "cpu" or not t.is_pinned() or not t.is_contiguous():
                        raise ValueError("host records must be contiguous pinned CPU tensors")
                # The reference validates every stored record when its session is
                # built (memory.py:128); same checks, same errors.
                validate(w)
        self.layers = list(layers)
        self.capacity = max(layer_bytes(layer) for layer in self.layers)
        self.group = group
        self.world, self.rank = 1, 0
        if group is not None:
            import torch.distributed as dist
            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.host_shards = None
        if self.world > 1:
            # Equal 256-byte-aligned shards; this rank's range of every layer, pinned.
            step = self.world * _ALIGN
            self.capacity = (self.capacity + step - 1) // step * step
            self.shard = self.capacity // self.world
            self.host_shards = [shard_image(layer, self.rank * self.shard, self.shard).pin_memory()
                                for layer in self.layers]
        with torch.cuda.device(self.device):
            self.copy_stream = copy_stream or torch.cuda.Stream(device=self.device)
            self.slots = []
            for i in range(min(slots, len(self.layers))):
                buf = torch.empty(self.capacity, dtype=torch.uint8, device=self.device)
                self.slots.append({"id": i, "buffer": buf, "layer": None, "ready": None, "consumed": None,
                                   "active": False, "views": None})
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        self.poisoned = False
        self.closed = False
        self.h2d_bytes = 0
        self.uploads = 0
        self.hits = 0
        self.copy_events = []  # (start, end, bytes) per upload, for H2D GB/s
        self._lock = threading.Lock()

    # -------------------------------------------------------------- internals
    def _views(self, slot, idx):
        return layer_views(slot["buffer"], self.layers[idx])

    def _find(self, idx):
        return next((s for s in self.slots if s["layer"] == idx), None)

    def _victim(self, keep=None):
        free = [s for s in self.slots if not s["active"] and (keep is None or s["layer"] != keep)]
        if not free:
            raise RuntimeError("no inactive slot available")
        # Prefer an empty slot, then the one consumed longest ago (lowest id tie-break).
        return min(free, key=lambda s: (s["layer"] is not None, s.get("last_use", -1), s["id"]))

    def _enqueue(self, idx, slot):
        if slot["active"]:
            raise RuntimeError("cannot overwrite an active consumer slot")
        views = self._views(slot, idx)
        src = self.layers[idx]
        nbytes = 0
        with torch.cuda.stream(self.copy_stream):
            if slot["consumed"] is not None:
                self.copy_stream.wait_event(slot["consumed"])
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(self.copy_stream)
            if self.host_shards is not None:
                import torch.distributed as dist
                buf = slot["buffer"]
                mine = buf.narrow(0, self.rank * self.shard, self.shard)
                mine.copy_(self.host_shards[idx], non_blocking=True)
                nbytes = self.shard
                # In place: every rank's chunk of the slot -> the whole slot on every rank.
                dist.all_gather_into_tensor(buf, mine, group=self.group, async_op=True).wait()
            else:
                buf = slot["buffer"]
                for off, b in _parts(src):
                    buf.narrow(0, off, b.numel()).copy_(b, non_blocking=True)
                    nbytes += b.numel()
            end.record(self.copy_stream)
        slot.update(layer=idx, ready=end, views=views)
        self.copy_events.append((start, end, nbytes))
        self.h2d_bytes += nbytes
        self.uploads += 1

    # -------------------------------------------------------------- public
    @contextmanager
    def borrow(self, idx, phase):
        """Yield {name: PackedWeight} device views of layer `idx` for the current stream.

        phase 'forward' prefetches idx+1, 'backward' prefetches idx-1.
        """
        if self.closed or self.poisoned:
            raise RuntimeError("slot session is closed or poisoned")
        if phase not in ("forward", "backward"):
            raise ValueError("unknown slot consumer phase")
        if not self._lock.acquire(blocking=False):
            raise RuntimeError("concurrent/reentrant slot borrow is unsupported")
        slot = None
        try:
            compute = torch.cuda.current_stream(self.device)
            slot = self._find(idx)
            if slot is None:
                slot = self._victim()
                self._enqueue(idx, slot)
            else:
                self.hits += 1
            slot["active"] = True
            compute.wait_event(slot["ready"])
            nxt = idx + (1 if phase == "forward" else -1)
            if 0 <= nxt < len(self.layers) and self._find(nxt) is None and len(self.slots) > 1:
                self._enqueue(nxt, self._victim(keep=idx))
            yield slot["views"]
        except BaseException:
            self.poisoned = True
            raise
        finally:
            try:
                if slot is not None and slot["active"]:
                    ev = torch.cuda.Event()
                    ev.record(torch.cuda.current_stream(self.device))
                    slot["consumed"] = ev
                    slot["active"] = False
                    self._clock = getattr(self, "_clock", 0) + 1
                    slot["last_use"] = self._clock
            finally:
                self._lock.release()

    def h2d_seconds(self):
        """Sum of copy-stream durations of completed uploads (synchronizes their events; with a
        group this includes the all-gather)."""
        total = 0.0
        for s, e, _ in self.copy_events:
            e.synchronize()
            total += s.elapsed_time(e) / 1e3
        return total

    def reset_stats(self):
        self.copy_events.clear()
        self.h2d_bytes = 0
        self.uploads = 0
        self.hits = 0

    def close(self):
        if self._lock.locked():
            raise RuntimeError("cannot close an active slot session")
        if not self.closed:
            torch.cuda.synchronize(self.device)
            self.slots.clear()
            self.closed = True
