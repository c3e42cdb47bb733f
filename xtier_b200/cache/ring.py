"""Swap ring of the hot-slot pool: residency changes applied on the GPU, weight copies off the decode stream.

`SwapRing` owns a command ring in mapped pinned memory and a side copy stream (csrc/cuda/pool_ring.cu). A swap
posts UNMAP(victim) and applies it at once with a one-thread commit kernel on the compute stream (the victim's routes
go to the CPU tier from the next kernel on), makes the copy stream wait for that commit, copies the incoming expert's
bytes into the freed slot on the copy stream, stamps the ring's `landed` word there, and posts MAP(incoming, slot).
The commit kernel the captured decode step runs first applies the MAP in the first step after the copy landed; until
then the incoming expert routes to the CPU tier as before. No decode step waits for a PCIe copy, and the slot is
mapped by no table while it is rewritten. The host-side residency (`table_host`, `hot`, the prefill staging indices)
follows the posted commands; `sync()` (before a prefill) waits for the copies and applies everything.

Reference parity: csrc/mailbox/mailbox.cpp:144-360 (mapped command ring with posted / applied / landed sequence
words), xtier/cache/pool.py:112-142 (GPU-side commit of landed swaps).
"""
from __future__ import annotations

import torch

from .. import ops


class SwapRing:
    def __init__(self, layers, device, capacity: int = 4096):
        """layers: the TieredMoE layers of one GPU whose swaps go through this ring (ring layer id = index)."""
        ops.load()
        self.layers = list(layers)
        self.device = torch.device(device)
        self.index = {id(l): i for i, l in enumerate(self.layers)}
        self.h = torch.ops.xtier.pool_ring_create(capacity)
        self.capacity = capacity
        self.tables = torch.tensor([l.table.data_ptr() for l in self.layers], dtype=torch.int64, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.seq = 0
        self._synced = 0     # last sequence number a sync() covered
        self.stream = torch.cuda.Stream(self.device)
        self._inflight: list[tuple[object, torch.cuda.Event]] = []   # host sources kept alive until copied
        for l in self.layers:
            l.ring = self

    def commit(self):
        """Applies every posted command whose copy has landed (current stream; graph capturable)."""
        torch.ops.xtier.pool_ring_commit(self.h, self.tables, self.err)

    def _post(self, layer_id: int, expert: int, slot: int) -> int:
        self.seq += 1
        rc = torch.ops.xtier.pool_ring_post(self.h, self.seq, layer_id, expert, slot)
        if rc:
            self.seq -= 1
            raise RuntimeError('swap ring full: call sync() between rounds' if rc == -3 else f'swap ring post {rc}')
        return self.seq

    def place(self, layer, incoming: int, slot: int, src, victim: int | None = None):
        """Copies expert `incoming` (host ExpertWeights [1, ...], pinned) into `slot` off the decode stream; with a
        victim, that expert is unmapped first (its routes go to the CPU tier until further notice)."""
        li = self.index[id(layer)]
        if victim is not None:
            self._post(li, victim, -1)
            self.commit()                               # the unmap takes effect before anything launched later
        ready = torch.cuda.Event()
        ready.record()
        map_seq = self.seq + 1
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                getattr(layer.pool, f)[slot].copy_(getattr(src, f)[0], non_blocking=True)
            torch.ops.xtier.pool_ring_landed(self.h, map_seq, self.err)
            done = torch.cuda.Event()
            done.record()
        self._inflight.append((src, done))
        assert self._post(li, incoming, slot) == map_seq
        self._inflight = [(s, e) for s, e in self._inflight if not e.query()]

    def applied(self) -> int:
        """Sequence number of the last command the GPU applied in order."""
        return int(torch.ops.xtier.pool_ring_applied(self.h))

    def sync(self):
        """The current stream waits for every copy in flight, then applies every posted command."""
        if self._synced == self.seq:
            return
        self._synced = self.seq
        torch.cuda.current_stream().wait_stream(self.stream)
        self.commit()
        self._inflight = [(s, e) for s, e in self._inflight if not e.query()]

    def check(self):
        if int(self.err.item()):
            raise RuntimeError('swap ring: a command named a layer or expert outside the tables')

    def close(self):
        if self.h:
            torch.cuda.synchronize(self.device)
            torch.ops.xtier.pool_ring_destroy(self.h)
            self.h = 0
            for l in self.layers:
                l.ring = None
