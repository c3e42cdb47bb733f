"""Row-table lookups inside a CUDA graph.

`GraphLookup` turns a RowStore lookup into three stream operations that a CUDA graph can capture and replay with no
host code on the replay path: a device->host copy of the step's ids into pinned memory, a host-function node that runs
the C++ lookup (csrc/tables/rows.cpp: xt_rows_host_fn; page cache, NVMe reads, row cache) into pinned rows, and a
host->device copy of the rows into a fixed device buffer the model reads. With `fp8_block`, the table holds FP8 (E4M3)
rows with one E8M0 scale per `fp8_block` values (DeepSeek Engram rows) and a fourth operation decodes them into BF16
rows (`rows_bf16`, csrc/cuda/fp8.cu fp8_rows; reference xtier/packs/deepseek_v4/engram_gather.py). The ids buffer has a
fixed capacity; the
number looked up per call is fixed at construction (pad unused ids with any valid row). A failed lookup leaves zero
rows and sets an error word that `check()` reports between replays.
(Reference parity: xtier/tables/lookup.py:47-93, GraphLookup.fetch through cudaLaunchHostFunc.)
"""
from __future__ import annotations

import ctypes as C

import torch

from . import RowStore, lib as rows_lib


class _Ctx(C.Structure):
    _fields_ = [('store', C.c_void_p), ('ids', C.c_void_p), ('n', C.c_int), ('rows', C.c_void_p),
                ('scales', C.c_void_p), ('error', C.c_int)]


class GraphLookup:
    def __init__(self, store: RowStore, n: int, device='cuda', fp8_block: int = 0):
        from .. import ops
        self.store, self.n = store, n
        self.fp8_block = fp8_block
        self.device = torch.device(device)
        self.ids_host = torch.zeros(n, dtype=torch.int64).pin_memory()
        self.rows_host = torch.zeros(n, store.row_bytes, dtype=torch.uint8).pin_memory()
        self.scales_host = (torch.zeros(n, store.scale_bytes, dtype=torch.uint8).pin_memory()
                            if store.scale_bytes else None)
        self.rows = torch.zeros(n, store.row_bytes, dtype=torch.uint8, device=self.device)
        self.scales = (torch.zeros(n, store.scale_bytes, dtype=torch.uint8, device=self.device)
                       if store.scale_bytes else None)
        self.rows_bf16 = None
        if fp8_block:
            if store.scale_bytes * fp8_block != store.row_bytes:
                raise ValueError('fp8 rows: one scale byte per fp8_block payload bytes expected')
            self.rows_bf16 = torch.zeros(n, store.row_bytes, dtype=torch.bfloat16, device=self.device)
        self.ctx = _Ctx(store.handle, self.ids_host.data_ptr(), n, self.rows_host.data_ptr(),
                        self.scales_host.data_ptr() if self.scales_host is not None else None, 0)
        self._fn = C.cast(rows_lib().xt_rows_host_fn, C.c_void_p).value
        cu = ops.cdll()
        cu.xt_launch_host_fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p]
        self._launch = cu.xt_launch_host_fn

    def fetch(self, ids: torch.Tensor):
        """Enqueues the lookup of ids [n] (int64, on the device) on the current stream; returns the device rows
        (and scales). Capturable."""
        self.ids_host.copy_(ids, non_blocking=True)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        if self._launch(C.c_void_p(stream), C.c_void_p(self._fn), C.byref(self.ctx)) != 0:
            raise RuntimeError('cudaLaunchHostFunc failed')
        self.rows.copy_(self.rows_host, non_blocking=True)
        if self.scales is not None:
            self.scales.copy_(self.scales_host, non_blocking=True)
        if self.fp8_block:
            from .. import ops
            return ops.fp8_rows(self.rows, self.scales, self.rows_bf16, block=self.fp8_block)
        return (self.rows, self.scales) if self.scales is not None else self.rows

    def check(self):
        if self.ctx.error:
            self.ctx.error = 0
            raise IndexError('row table lookup failed inside the graph: ' + rows_lib().xt_rows_error().decode())
