"""Symmetric peer memory: one device buffer per rank, of the same size, mapped into every rank's address space
through CUDA IPC handles (exchanged over the host group). Kernels get the W base addresses as a device array and load
from / store to peers directly over NVLink; the layout inside the buffer is the same on every rank.

(The reference has no peer path: its second GPU is reached through host memory, xtier/cache/second.py:1-16.)
"""
from __future__ import annotations

import ctypes as C

import torch

from . import dist as xdist


class SymmetricBuffer:
    """`ptrs[r]`: rank r's buffer as mapped in this process; `peer_table`: the same as a device int64 tensor."""

    def __init__(self, nbytes: int, device=None):
        from .. import ops
        env = xdist.get()
        self.device = device or env.device or torch.device('cuda')
        self.nbytes = (nbytes + 4095) // 4096 * 4096
        L = ops.cdll()
        L.xt_ipc_alloc.argtypes = [C.c_size_t, C.c_void_p]
        L.xt_ipc_free.argtypes = [C.c_void_p]
        L.xt_ipc_export.argtypes = [C.c_void_p, C.c_void_p]
        L.xt_ipc_open.argtypes = [C.c_void_p, C.c_void_p]
        L.xt_ipc_close.argtypes = [C.c_void_p]
        self._L = L
        base = C.c_void_p()
        with torch.cuda.device(self.device):
            rc = L.xt_ipc_alloc(self.nbytes, C.byref(base))
        if rc != 0:
            raise RuntimeError(f'symmetric buffer: cudaMalloc of {self.nbytes} bytes failed ({rc})')
        self.base = base.value
        hb = L.xt_ipc_handle_bytes()
        handle = (C.c_uint8 * hb)()
        if env.world > 1:
            rc = L.xt_ipc_export(C.c_void_p(self.base), handle)
            if rc != 0:
                raise RuntimeError(f'cudaIpcGetMemHandle failed ({rc})')
        infos = xdist.all_gather_bytes(bytes(handle))
        self.ptrs = []
        self._opened = []
        for r, inf in enumerate(infos):
            if r == env.rank:
                self.ptrs.append(self.base)
                continue
            p = C.c_void_p()
            with torch.cuda.device(self.device):
                rc = L.xt_ipc_open((C.c_uint8 * hb).from_buffer_copy(inf), C.byref(p))
            if rc != 0:
                raise RuntimeError(f'cudaIpcOpenMemHandle of rank {r} failed ({rc})')
            self._opened.append(p.value)
            self.ptrs.append(p.value)
        self.peer_table = torch.tensor(self.ptrs, dtype=torch.int64, device=self.device)

    def close(self):
        for p in self._opened:
            self._L.xt_ipc_close(C.c_void_p(p))
        self._opened = []
        if getattr(self, 'base', None):
            self._L.xt_ipc_free(C.c_void_p(self.base))
            self.base = None
