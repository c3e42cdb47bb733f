"""ctypes bindings of the native host libraries: the CPU expert engine (`CpuEngine`) and the cold-expert store
(`ColdStore`). The mailbox that lets CUDA graphs call the engine lives in xtier_b200.engine.mailbox.

Reference parity: xtier/engine/__init__.py (CpuPlan :79, ColdStore :231; library lookup via XTIER_ENGINE_LIB :21).
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

import numpy as np
import torch

from .. import config
from ..formats import MXFP4, NVFP4, ExpertWeights

_LIBDIR = Path(__file__).resolve().parent.parent / '_lib'
_lib = None

_P = C.c_void_p
_I = C.c_int
_F = C.c_float


def lib_path() -> Path:
    override = config.get('XTIER_ENGINE_LIB')
    return Path(override) if override else _LIBDIR / 'libxt_engine.so'


def lib():
    """The engine library, built in-tree on first use if missing."""
    global _lib
    if _lib is None:
        path = lib_path()
        if not path.exists():
            from .. import _build
            _build.build(cuda=False, verbose=False)
        L = C.CDLL(str(path))
        L.xt_engine_create.restype = _P
        L.xt_engine_create.argtypes = [_I, _I, _I, _I, _I, _I, _F, _I, _P, _P, _P, _P, _P, _P, _P]
        for name in ('xt_engine_forward', 'xt_engine_forward_decode'):
            getattr(L, name).restype = _I
            getattr(L, name).argtypes = [_P, _I, _I, _P, _P, _P, _P]
        L.xt_engine_read_probe.argtypes = [_P, _I, _I, _P]
        L.xt_engine_destroy.argtypes = [_P]
        L.xt_engine_set_swiglu.argtypes = [_P, _F, _F]
        L.xt_engine_shape.argtypes = [_P, _P]
        L.xt_engine_last_timings.argtypes = [_P, _P]
        L.xt_engine_tail_stats.argtypes = [_P, _P]
        L.xt_engine_slot_table.argtypes = [_P, _P]
        L.xt_engine_place.argtypes = [_P, _I, _I]
        L.xt_engine_expert_scales.argtypes = [_P, _P, _P]
        L.xt_engine_slot_pin.argtypes = [_P, _I]
        L.xt_engine_slot_unpin.argtypes = [_P, _I]
        L.xt_engine_slot_pieces.argtypes = [_P, _I, _I, _P, _P]
        L.xt_engine_nodes.argtypes = [_P]
        L.xt_engine_shard.argtypes = [_P, _I, _P, _P, _P, _P, _P]
        L.xt_engine_cold_attach.argtypes = [_P, _P, _P, _P, _P, _F]
        L.xt_engine_cold_attach_pieces.argtypes = [_P, _P, _P, _P, _P, _F]
        L.xt_engine_cold_stats.argtypes = [_P, _P]
        L.xt_engine_worker_cpus.argtypes = [_I, _P, _I]
        L.xt_engine_isa.restype = C.c_char_p
        L.xt_engine_error.restype = C.c_char_p
        L.xt_cold_open.restype = _P
        L.xt_cold_open.argtypes = [_P, _I, _I, _I]
        L.xt_cold_write.argtypes = [_P, _I, C.c_longlong, _P, _P, _I]
        L.xt_cold_read.argtypes = [_P, _I, _P, _P, _P, _P, _I]
        L.xt_cold_submit.restype = _P
        L.xt_cold_submit.argtypes = [_P, _I, _P, _P, _P, _P, _I, _P, _I]
        L.xt_cold_wait.argtypes = [_P, _P, _I, _I]
        L.xt_cold_finish.argtypes = [_P, _P]
        L.xt_cold_stats.argtypes = [_P, _P]
        L.xt_cold_close.argtypes = [_P]
        L.xt_cold_error.restype = C.c_char_p
        _lib = L
    return _lib


def isa() -> str:
    return lib().xt_engine_isa().decode()


def _ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def default_threads() -> int:
    n = config.get('XTIER_THREADS')
    if n and n > 0:
        return n
    return max(1, len(os.sched_getaffinity(0)) - 1)


class CpuEngine:
    """One MoE layer's routed (and shared) experts on the CPU.

    `experts` holds the routed experts (ids 0..E-1); `shared` optional shared experts applied to every token with
    weight 1. With `slots` < E only `resident` experts are in RAM; the others must come from an attached cold store.
    With `total_experts`, `experts` holds exactly the `resident` experts in slot order (ids of a larger set of
    `total_experts`), so the caller never materializes the experts this engine does not keep.
    """

    def __init__(self, experts: ExpertWeights, shared: ExpertWeights | None = None, threads: int | None = None,
                 limit: float = 0.0, slots: int | None = None, resident=None, fill: bool = True,
                 total_experts: int | None = None):
        L = lib()
        self.H, self.I = experts.hidden, experts.inter
        self.E = experts.experts if total_experts is None else total_experts
        self.fmt = experts.fmt
        self.shared = 0 if shared is None else shared.experts
        self.slots = self.E if slots is None else slots
        ew = experts.to('cpu')
        if resident is not None:
            res = torch.as_tensor(resident, dtype=torch.int32).contiguous()
            if total_experts is not None:
                if (fill and len(res) != experts.experts) or self.slots < len(res):
                    raise ValueError('engine: the given experts must be the resident ones, one per slot')
                src = ew if fill else None
            else:
                src = ew.select(res.clamp_min(0).long()) if fill else None
        else:
            res = None
            src = ew.select(torch.arange(self.slots)) if self.slots < self.E else ew
        arrays = None
        if fill:
            parts = [src] + ([shared.to('cpu')] if shared is not None else [])
            fields = ('w13', 'w2', 's13', 's2', 'g13', 'g2')
            if len(parts) == 1:   # no concatenation copy
                arrays = [getattr(src, f).contiguous() for f in fields]
            else:
                arrays = [torch.cat([getattr(p, f) for p in parts]).contiguous() for f in fields]
            arrays[4] = arrays[4].float().contiguous()
            arrays[5] = arrays[5].float().contiguous()
        self._keep = arrays
        self.plan = L.xt_engine_create(self.H, self.I, self.E, self.shared, self.slots,
                                       threads if threads is not None else default_threads(), limit,
                                       0 if self.fmt == NVFP4 else 1,
                                       *([_ptr(a) for a in arrays] if arrays else [None] * 6),
                                       _ptr(res))
        self._keep = None
        if not self.plan:
            raise RuntimeError(f'xtier_b200 engine: {L.xt_engine_error().decode()}')

    def close(self):
        if getattr(self, 'plan', None):
            lib().xt_engine_destroy(self.plan)
            self.plan = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_swiglu(self, alpha: float, beta: float):
        lib().xt_engine_set_swiglu(self.plan, alpha, beta)

    def shape(self) -> dict:
        out = (C.c_int * 7)()
        lib().xt_engine_shape(self.plan, out)
        return dict(zip(('hidden', 'inter', 'experts', 'shared', 'slots', 'nodes', 'threads'), list(out)))

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, out: torch.Tensor | None = None,
                decode: bool = False) -> torch.Tensor:
        """x bf16 [m, H], ids int32 [m, k] (-1 skips), weights fp32 [m, k] -> fp32 [m, H] (CPU tensors)."""
        x = x.to(torch.bfloat16).contiguous()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.to(torch.float32).contiguous()
        m, k = ids.shape
        if out is None:
            out = torch.empty(m, self.H, dtype=torch.float32)
        fn = lib().xt_engine_forward_decode if decode else lib().xt_engine_forward
        rc = fn(self.plan, m, k, _ptr(x), _ptr(ids), _ptr(weights), _ptr(out))
        if rc < 0:
            raise RuntimeError(f'xtier_b200 engine: {lib().xt_engine_error().decode()}')
        return out

    def read_probe(self, ids: torch.Tensor) -> int:
        ids = ids.to(torch.int32).contiguous()
        return lib().xt_engine_read_probe(self.plan, ids.shape[0], ids.shape[1], _ptr(ids))

    def last_timings(self) -> tuple[float, float]:
        out = (C.c_double * 2)()
        lib().xt_engine_last_timings(self.plan, out)
        return out[0], out[1]

    def tail_stats(self):
        out = (C.c_double * 3)()
        lib().xt_engine_tail_stats(self.plan, out)
        return tuple(out)

    def slot_table(self) -> np.ndarray:
        t = np.empty(self.E, dtype=np.int32)
        lib().xt_engine_slot_table(self.plan, t.ctypes.data)
        return t

    def pin(self, expert: int) -> int:
        """Keeps `expert` in its RAM slot (no miss evicts it) until `unpin`; returns the slot, -1 when not in RAM."""
        return lib().xt_engine_slot_pin(self.plan, expert)

    def unpin(self, slot: int):
        lib().xt_engine_slot_unpin(self.plan, slot)

    def place(self, expert: int, slot: int) -> int:
        """Slot `slot` now holds `expert` (-1: nothing); returns the expert it held before (-1: none)."""
        return lib().xt_engine_place(self.plan, expert, slot)

    def set_expert_scales(self, g13: torch.Tensor, g2: torch.Tensor):
        """Global scales of every routed expert (g13 [E, 2], g2 [E]); a slot then takes the scales of whichever expert
        is placed or read into it (needed with a cold store, whose records hold only codes and block scales)."""
        a = g13.detach().float().cpu().contiguous()
        b = g2.detach().float().cpu().contiguous()
        if a.numel() != 2 * self.E or b.numel() != self.E:
            raise ValueError('expert scales: g13 [E, 2] and g2 [E] expected')
        if lib().xt_engine_expert_scales(self.plan, _ptr(a), _ptr(b)) != 0:
            raise RuntimeError('xtier_b200 engine: expert scales refused (a forward is running?)')

    def nodes(self) -> int:
        return lib().xt_engine_nodes(self.plan)

    def slot_pieces(self, slot: int, node: int):
        ptrs = (C.c_void_p * 6)()
        sizes = (C.c_size_t * 6)()
        if lib().xt_engine_slot_pieces(self.plan, slot, node, ptrs, sizes) != 0:
            raise IndexError(f'slot {slot} node {node}')
        return list(ptrs), list(sizes)

    def shard(self, node: int) -> dict:
        """Node `node`'s shard: base address, bytes, slot stride, the six pieces' offsets and sizes in a slot."""
        base, nbytes, stride = C.c_void_p(), C.c_size_t(), C.c_size_t()
        off, sizes = (C.c_size_t * 6)(), (C.c_size_t * 6)()
        if lib().xt_engine_shard(self.plan, node, C.byref(base), C.byref(nbytes), C.byref(stride), off, sizes) != 0:
            raise IndexError(f'node {node}')
        return dict(base=base.value or 0, bytes=nbytes.value, stride=stride.value, piece_off=list(off),
                    piece_bytes=list(sizes))

    def write_slot(self, slot: int, ew: ExpertWeights, e: int):
        """Copies expert e of `ew` into RAM slot `slot` (all nodes), e.g. after reading it from a checkpoint."""
        N = self.nodes()
        I, H = self.I, self.H
        gr, dr = I // N, H // N
        w13, s13, w2, s2 = ew.w13[e], ew.s13[e], ew.w2[e], ew.s2[e]
        for n in range(N):
            ptrs, sizes = self.slot_pieces(slot, n)
            pieces = [w13[n * gr:(n + 1) * gr], w13[I + n * gr:I + (n + 1) * gr], s13[n * gr:(n + 1) * gr],
                      s13[I + n * gr:I + (n + 1) * gr], w2[n * dr:(n + 1) * dr], s2[n * dr:(n + 1) * dr]]
            for p, ptr, sz in zip(pieces, ptrs, sizes):
                p = p.contiguous()
                if p.numel() * p.element_size() != sz:
                    raise ValueError(f'engine slot piece: {p.numel() * p.element_size()} bytes, slot holds {sz}')
                C.memmove(ptr, p.data_ptr(), sz)

    def attach_cold(self, store: 'ColdStore', files, offsets, scores=None, half_life: float = 64.0):
        f = np.ascontiguousarray(files, dtype=np.int32)
        o = np.ascontiguousarray(offsets, dtype=np.int64)
        s = None if scores is None else np.ascontiguousarray(scores, dtype=np.float32)
        rc = lib().xt_engine_cold_attach(self.plan, store.handle, f.ctypes.data, o.ctypes.data,
                                         None if s is None else s.ctypes.data, half_life)
        if rc != 0:
            raise RuntimeError('xtier_b200 engine: cold attach failed')
        self._cold = (store, f, o, s)

    def attach_cold_pieces(self, store: 'ColdStore', files, offsets, scores=None, half_life: float = 64.0):
        """As attach_cold with one (file, offset) per piece: arrays [experts * nodes * 6]."""
        f = np.ascontiguousarray(files, dtype=np.int32)
        o = np.ascontiguousarray(offsets, dtype=np.int64)
        s = None if scores is None else np.ascontiguousarray(scores, dtype=np.float32)
        rc = lib().xt_engine_cold_attach_pieces(self.plan, store.handle, f.ctypes.data, o.ctypes.data,
                                                None if s is None else s.ctypes.data, half_life)
        if rc != 0:
            raise RuntimeError('xtier_b200 engine: cold attach failed')
        self._cold = (store, f, o, s)

    def cold_stats(self):
        out = (C.c_double * 4)()
        lib().xt_engine_cold_stats(self.plan, out)
        return dict(zip(('forwards', 'reads', 'wait_s', 'decode_forwards'), list(out)))


class ColdStore:
    """O_DIRECT expert records on one file per drive (see csrc/cold/store.cpp)."""

    def __init__(self, paths, threads: int = 4, writable: bool = False):
        self.paths = [str(p) for p in paths]
        arr = (C.c_char_p * len(self.paths))(*[p.encode() for p in self.paths])
        self.handle = lib().xt_cold_open(arr, len(self.paths), threads, int(writable))
        if not self.handle:
            raise OSError(lib().xt_cold_error().decode())

    def write(self, file: int, offset: int, pieces: list[bytes | np.ndarray]):
        bufs = [np.frombuffer(bytes(p), dtype=np.uint8) if not isinstance(p, np.ndarray) else p for p in pieces]
        ptrs = (C.c_void_p * len(bufs))(*[b.ctypes.data for b in bufs])
        sizes = (C.c_size_t * len(bufs))(*[b.nbytes for b in bufs])
        if lib().xt_cold_write(self.handle, file, offset, ptrs, sizes, len(bufs)) != 0:
            raise OSError(lib().xt_cold_error().decode())

    def read(self, files, offsets, dst_ptrs, sizes, n: int):
        f = np.ascontiguousarray(files, dtype=np.int32)
        o = np.ascontiguousarray(offsets, dtype=np.int64)
        d = (C.c_void_p * len(dst_ptrs))(*dst_ptrs)
        s = (C.c_size_t * len(sizes))(*sizes)
        if lib().xt_cold_read(self.handle, len(f), f.ctypes.data, o.ctypes.data, d, s, n) != 0:
            raise OSError(lib().xt_cold_error().decode())

    def submit(self, files, offsets, dst_ptrs, sizes, n: int, groups=None, group_count: int = 1):
        f = np.ascontiguousarray(files, dtype=np.int32)
        o = np.ascontiguousarray(offsets, dtype=np.int64)
        d = (C.c_void_p * len(dst_ptrs))(*dst_ptrs)
        s = (C.c_size_t * len(sizes))(*sizes)
        g = None if groups is None else np.ascontiguousarray(groups, dtype=np.int32)
        t = lib().xt_cold_submit(self.handle, len(f), f.ctypes.data, o.ctypes.data, d, s, n,
                                 None if g is None else g.ctypes.data, group_count)
        if not t:
            raise OSError(lib().xt_cold_error().decode())
        return _Ticket(self, t, (f, o, d, s, g))

    def stats(self):
        out = (C.c_double * 4)()
        lib().xt_cold_stats(self.handle, out)
        return dict(zip(('bytes_read', 'bytes_written', 'jobs', 'seconds'), list(out)))

    def close(self):
        if self.handle:
            lib().xt_cold_close(self.handle)
            self.handle = None


class _Ticket:
    def __init__(self, store, handle, keep):
        self.store, self.handle, self._keep = store, handle, keep

    def wait(self, g0: int, g1: int):
        if lib().xt_cold_wait(self.store.handle, self.handle, g0, g1) != 0:
            raise OSError('cold store: a read of the ticket failed')

    def finish(self):
        rc = lib().xt_cold_finish(self.store.handle, self.handle)
        self.handle = None
        if rc != 0:
            raise OSError('cold store: a read of the ticket failed')


__all__ = ['CpuEngine', 'ColdStore', 'isa', 'lib', 'NVFP4', 'MXFP4', 'default_threads']
