"""Elastic hot-expert cache: extra GPU slots in memory that only a prefill needs (XTIER_CACHE_ELASTIC=1).

Between prefills, the memory their activations and workspaces take lies idle. A partly cached layer gets address
space for `extra` slots behind its base and shared slots (`VmmArena`: a reserved device address range whose prefix is
backed by memory, csrc/cuda/vmm.cu); free memory backs extra slots, which the adaptive policy fills with the most
routed experts the GPU does not hold (no victim needed). The arena base never moves, so captured decode graphs stay
valid; only the physical backing of the tail comes and goes.

`Governor` sizes the extra slots of every elastic layer together ("levels": one extra slot in every layer):
* it learns what a forward that allocates (a prefill) needs -- peak allocated memory over the amount before it -- per
  (tokens, context) and predicts a new forward's need as the tightest bound among the needs seen: a seen need bounds
  any forward no larger in either; scaled by both ratios (up to XTIER_CACHE_ELASTIC_EXTRAPOLATE, 2x) it bounds a
  larger one; with no bound every extra slot goes back;
* `before_alloc` releases levels until free memory covers need x MARGIN (1.25) + RESERVE_GIB (2);
* `after_decode`: every CHECK (16) decode steps, free memory under CRITICAL_GIB (1) releases every level and stops
  growth for COOLDOWN_S; after IDLE (32) decode steps without an allocating forward, it grows a few levels while free
  memory stays above the reserve plus the usual small prefill's need;
* `guarded(fn)`: an out-of-memory error while levels are held releases them all, empties the allocator's cache,
  turns elastic growth off for the process and runs the forward once more.
Releasing a slot first unpublishes its expert from the residency table on the compute stream, synchronizes the
device, then unmaps the granules: no queued or running kernel can read a released slot.

Reference parity: xtier/cache/elastic.py:1-56 (the design), :140-415 (Governor: predict, learn, release, grow,
before_alloc, after_decode, emergency), :472-512 (OOM retry). The need table, the level accounting and the arena
(csrc/cuda/vmm.cu) are this project's own.
"""
from __future__ import annotations

import ctypes as C
import logging
import math
import time

import torch

from .. import config

logger = logging.getLogger('xtier_b200')
GIB = 2 ** 30
FIELDS = ('w13', 'w2', 's13', 's2')


def _lib():
    from .. import ops
    L = ops.cdll()
    L.xt_vmm_granularity.restype = C.c_size_t
    L.xt_vmm_granularity.argtypes = [C.c_int]
    L.xt_vmm_reserve.argtypes = [C.c_int, C.c_size_t, C.c_void_p, C.c_void_p]
    L.xt_vmm_map.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t]
    L.xt_vmm_unmap.argtypes = [C.c_void_p, C.c_size_t, C.c_size_t]
    L.xt_vmm_mapped.restype = C.c_longlong
    L.xt_vmm_mapped.argtypes = [C.c_void_p]
    L.xt_vmm_free.argtypes = [C.c_void_p]
    return L


class _CudaArray:
    """Exposes a raw device range to torch (`__cuda_array_interface__`); the tensor keeps this object alive."""

    def __init__(self, ptr: int, nbytes: int, owner):
        self.__cuda_array_interface__ = dict(shape=(nbytes,), typestr='|u1', data=(ptr, False), version=3,
                                             strides=None)
        self.owner = owner


class VmmArena:
    """`capacity` bytes of reserved device address space; `ensure(n)` backs the first n bytes (whole granules),
    `shrink(n)` gives back the granules past them."""

    def __init__(self, capacity: int, device):
        self.device = torch.device(device)
        self.L = _lib()
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.index = idx
        self.granule = int(self.L.xt_vmm_granularity(idx))
        if self.granule == 0:
            raise RuntimeError('VMM: the driver does not offer cuMemCreate / cuMemMap')
        base, got = C.c_void_p(), C.c_size_t()
        with torch.cuda.device(self.device):
            rc = self.L.xt_vmm_reserve(idx, capacity, C.byref(base), C.byref(got))
        if rc != 0:
            raise RuntimeError(f'VMM: reserving {capacity} bytes failed ({rc})')
        self.base, self.capacity = int(base.value), int(got.value)
        self.granules = 0          # mapped prefix, in granules

    def tensor(self) -> torch.Tensor:
        """The whole range as a uint8 tensor (only the mapped prefix may be touched)."""
        return torch.as_tensor(_CudaArray(self.base, self.capacity, self), device=self.device)

    def ensure(self, nbytes: int):
        g = min(self.capacity // self.granule, math.ceil(nbytes / self.granule))
        if g > self.granules:
            with torch.cuda.device(self.device):
                rc = self.L.xt_vmm_map(C.c_void_p(self.base), self.granules, g)
            if rc != 0:
                raise torch.cuda.OutOfMemoryError(f'VMM: mapping {(g - self.granules) * self.granule} bytes failed '
                                                  f'({rc})')
            self.granules = g

    def shrink(self, nbytes: int):
        g = math.ceil(nbytes / self.granule)
        if g < self.granules:
            rc = self.L.xt_vmm_unmap(C.c_void_p(self.base), g, self.granules)
            if rc != 0:
                raise RuntimeError(f'VMM: unmapping failed ({rc})')
            self.granules = g

    @property
    def mapped_bytes(self) -> int:
        return self.granules * self.granule

    def close(self):
        if self.base:
            self.L.xt_vmm_free(C.c_void_p(self.base))
            self.base = 0


class ElasticSlots:
    """Extra slots of one TieredMoE layer: its pool's code and scale tensors move into VMM arenas with room for
    `extra` more slots behind the base and shared ones (global scales: plain tensors at full capacity)."""

    def __init__(self, moe, extra: int):
        self.moe = moe
        pool = moe.pool
        self.first = pool.experts                    # base hot slots + shared slots
        self.cap = int(extra)
        C_ = self.first + self.cap
        self.rows = {f: getattr(pool, f)[0].numel() * getattr(pool, f).element_size() for f in FIELDS}
        self.arenas = {}
        for f in FIELDS:
            old = getattr(pool, f)
            a = VmmArena(C_ * self.rows[f], moe.device)
            a.ensure(self.first * self.rows[f])
            t = a.tensor()[:C_ * self.rows[f]].view(old.dtype).view(C_, *old.shape[1:])
            t[:self.first].copy_(old)
            self.arenas[f] = a
            setattr(pool, f, t)
        for f in ('g13', 'g2'):
            old = getattr(pool, f)
            t = torch.ones((C_,) + tuple(old.shape[1:]), dtype=old.dtype, device=old.device)
            t[:self.first].copy_(old)
            setattr(pool, f, t)
        self.mapped = 0                              # extra slots backed by memory
        self.occupant = [-1] * self.cap              # expert in each extra slot (-1: empty)
        moe.elastic = self

    def slot_bytes(self) -> int:
        return sum(self.rows.values())

    def mapped_bytes(self) -> int:
        return sum(a.mapped_bytes for a in self.arenas.values())

    def free_slot(self) -> int | None:
        for j in range(self.mapped):
            if self.occupant[j] < 0:
                return self.first + j
        return None

    def occupants(self) -> list[int]:
        return [e for e in self.occupant[:self.mapped] if e >= 0]

    def grow(self, n: int):
        """Backs extra slots [0, n) with memory (the new ones empty)."""
        n = min(n, self.cap)
        if n <= self.mapped:
            return
        for f in FIELDS:
            self.arenas[f].ensure((self.first + n) * self.rows[f])
        self.mapped = n

    def release(self, n: int):
        """Keeps extra slots [0, n): the experts of the others leave the residency table (stream-ordered), the device
        is synchronized, then their granules are unmapped."""
        n = max(0, n)
        if n >= self.mapped:
            return
        moe = self.moe
        if moe.ring is not None:   # no MAP into a released slot may still be pending
            moe.ring.sync()
        for j in range(n, self.mapped):
            e = self.occupant[j]
            if e >= 0:
                moe.table[e] = -1
                moe.table_host[e] = -1
                self.occupant[j] = -1
        torch.cuda.synchronize(moe.device)
        for f in FIELDS:
            self.arenas[f].shrink((self.first + n) * self.rows[f])
        self.mapped = n

    def close(self):
        self.release(0)
        for a in self.arenas.values():
            a.close()


def install(model, extra: int | None = None) -> list[ElasticSlots]:
    """Gives every partly cached MoE layer of `model` room for extra slots (XTIER_CACHE_ELASTIC_MAX x its base hot
    slots, at most every expert it does not hold). Call before any CUDA graph capture."""
    out = []
    for L in model.layers:
        moe = L['moe']
        if moe.all_hot or moe.pool is None or getattr(moe, 'slotless', False) or not moe.can_refill:
            continue
        n = extra if extra is not None else int(round((config.get('XTIER_CACHE_ELASTIC_MAX') - 1.0) * len(moe.hot)))
        n = max(0, min(n, moe.E - len(moe.hot)))
        if n:
            out.append(ElasticSlots(moe, n))
    return out


class Governor:
    """Sizes the extra slots of `layers` (ElasticSlots) against free device memory; all layers move together."""

    def __init__(self, layers, mem_info=None, reserve_gib=None, critical_gib=None, margin=None, idle=None,
                 every=None, cooldown_s=None, extrapolate=None, step=None, clock=time.monotonic):
        self.layers = list(layers)
        self.mem_info = mem_info or (lambda: torch.cuda.mem_get_info())
        g = lambda n, v: config.get(n) if v is None else v
        self.reserve = g('XTIER_CACHE_ELASTIC_RESERVE_GIB', reserve_gib) * GIB
        self.critical = g('XTIER_CACHE_ELASTIC_CRITICAL_GIB', critical_gib) * GIB
        self.margin = g('XTIER_CACHE_ELASTIC_MARGIN', margin)
        self.idle = int(g('XTIER_CACHE_ELASTIC_IDLE', idle))
        self.every = max(1, int(g('XTIER_CACHE_ELASTIC_CHECK', every)))
        self.cooldown = g('XTIER_CACHE_ELASTIC_COOLDOWN_S', cooldown_s)
        self.extrapolate = g('XTIER_CACHE_ELASTIC_EXTRAPOLATE', extrapolate)
        self.step = int(step if step is not None else 4)
        self.clock = clock
        self.cap = max((l.cap for l in self.layers), default=0)
        self.level = sum(l.slot_bytes() for l in self.layers)     # bytes of one extra slot in every layer
        self.extra = 0
        self.needs: dict[tuple[int, int], float] = {}
        self.enabled = bool(self.layers)
        self.since_alloc = 0
        self.decodes = 0
        self.frozen_until = 0.0
        self.events: list[tuple[str, int, str]] = []

    # ---------------------------------------------------------------- learning
    def learn(self, tokens: int, ctx: int, need: float):
        k = (int(tokens), int(ctx))
        self.needs[k] = max(self.needs.get(k, 0.0), float(need))

    def predict(self, tokens: int, ctx: int) -> float | None:
        best = None
        for (t, c), n in self.needs.items():
            rt, rc = tokens / max(t, 1), ctx / max(c, 1)
            if rt <= 1 and rc <= 1:
                bound = n
            elif max(rt, 1) * max(rc, 1) <= self.extrapolate:
                bound = n * max(rt, 1) * max(rc, 1)
            else:
                continue
            best = bound if best is None else min(best, bound)
        return best

    # ---------------------------------------------------------------- resizing
    def _set(self, n: int, why: str):
        n = max(0, min(n, self.cap))
        if n == self.extra:
            return
        if n < self.extra:
            for l in self.layers:
                l.release(n)
        else:
            for l in self.layers:
                l.grow(n)
        self.events.append(('release' if n < self.extra else 'grow', n, why))
        logger.debug('elastic: %s -> %d extra slots per layer (%s)', self.events[-1][0], n, why)
        self.extra = n

    def release_all(self, why: str):
        self._set(0, why)

    def before_alloc(self, tokens: int, ctx: int = 0) -> int:
        """Call before a forward that allocates; returns the levels released."""
        self.since_alloc = 0
        if self.extra == 0:
            return 0
        need = self.predict(tokens, ctx)
        if need is None:
            n0 = self.extra
            self.release_all(f'no need known for {tokens} tokens')
            return n0
        free, _ = self.mem_info()
        deficit = need * self.margin + self.reserve - free
        if deficit <= 0:
            return 0
        drop = min(self.extra, math.ceil(deficit / max(self.level, 1)))
        self._set(self.extra - drop, f'{tokens} tokens need {need / GIB:.2f} GiB')
        return drop

    def after_forward(self, tokens: int, ctx: int, before_bytes: int, peak_bytes: int):
        self.learn(tokens, ctx, max(0, peak_bytes - before_bytes))

    def after_decode(self) -> int:
        """Call after a decode step; returns the levels added (negative: released)."""
        self.decodes += 1
        self.since_alloc += 1
        if not self.enabled:
            return 0
        if self.decodes % self.every == 0:
            free, _ = self.mem_info()
            if free < self.critical and self.extra:
                n0 = self.extra
                self.release_all('free memory critical')
                self.frozen_until = self.clock() + self.cooldown
                return -n0
        if self.since_alloc < self.idle or self.clock() < self.frozen_until or self.extra >= self.cap:
            return 0
        free, _ = self.mem_info()
        small = [n for (t, _), n in self.needs.items() if t <= 4096]
        keep = self.reserve + (sorted(small)[int(0.75 * (len(small) - 1))] * self.margin if small else 0.0)
        room = int((free - keep) // max(self.level, 1))
        add = max(0, min(self.step, room, self.cap - self.extra))
        if add:
            self._set(self.extra + add, 'idle decode')
        return add

    def guarded(self, fn, *args, **kw):
        """Runs fn; on an out-of-memory error with extra slots held: release them all, empty the cache, switch growth
        off and run it once more."""
        try:
            return fn(*args, **kw)
        except torch.cuda.OutOfMemoryError:
            if self.extra == 0:
                raise
            logger.warning('elastic: out of memory with %d extra slots per layer held; releasing them and retrying '
                           'once (elastic growth is off from now on)', self.extra)
            self.release_all('out of memory')
            self.enabled = False
            torch.cuda.empty_cache()
            return fn(*args, **kw)

    def stats(self) -> dict:
        return dict(extra=self.extra, cap=self.cap, level_bytes=self.level, needs=len(self.needs),
                    enabled=self.enabled, events=len(self.events))
