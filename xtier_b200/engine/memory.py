"""Large pinned host tables: exact-size anonymous mappings interleaved over NUMA nodes and page-locked for the GPU.

`pinned_interleaved(nbytes, nodes)` maps `nbytes` (rounded up to whole pages, no allocator slack), asks the kernel to
interleave its pages over `nodes` (mbind MPOL_INTERLEAVE, so a table read by every socket's cores is not stuck on one
memory controller), advises huge pages, then registers it with CUDA (cudaHostRegister) so that copies to the GPU run
at full PCIe speed and kernels can read it through its mapped address. It returns a uint8 tensor over the mapping; the
mapping is unregistered and unmapped when the tensor's storage goes away. Where the kernel refuses mbind (containers
without CAP_SYS_NICE, single-node machines) the memory is still returned, with `policy_applied` False in `info`.
(Reference parity: xtier/engine/memory.py:43 pinned_interleaved -- exact-size mmap + mbind(INTERLEAVE) +
cudaHostRegister for huge pinned tables.)
"""
from __future__ import annotations

import ctypes as C
import mmap
import os
import weakref

import numpy as np
import torch

_SYS_MBIND = 237            # x86-64
_MPOL_INTERLEAVE = 3
_MADV_HUGEPAGE = 14
_libc = C.CDLL(None, use_errno=True)
_libc.mmap.restype = C.c_void_p
_libc.mmap.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_long]
_libc.munmap.argtypes = [C.c_void_p, C.c_size_t]
_libc.madvise.argtypes = [C.c_void_p, C.c_size_t, C.c_int]
_libc.syscall.restype = C.c_long


class _Mapping:
    def __init__(self, ptr: int, size: int, registered: bool):
        self.ptr, self.size, self.registered = ptr, size, registered

    def close(self):
        if self.ptr:
            if self.registered:
                try:
                    torch.cuda.cudart().cudaHostUnregister(self.ptr)
                except Exception:
                    pass
            _libc.munmap(C.c_void_p(self.ptr), self.size)
            self.ptr = 0


def pinned_interleaved(nbytes: int, nodes: list[int] | None = None, register: bool | None = None):
    """-> (uint8 tensor [nbytes] over the mapping, info dict). nodes None: every NUMA node with memory."""
    page = mmap.PAGESIZE
    size = max(page, (nbytes + page - 1) // page * page)
    ptr = _libc.mmap(None, size, mmap.PROT_READ | mmap.PROT_WRITE, mmap.MAP_PRIVATE | mmap.MAP_ANONYMOUS, -1, 0)
    if ptr in (None, C.c_void_p(-1).value):
        raise MemoryError(f'mmap of {size} bytes failed: {os.strerror(C.get_errno())}')
    if nodes is None:
        nodes = sorted(int(d[4:]) for d in os.listdir('/sys/devices/system/node')
                       if d.startswith('node') and d[4:].isdigit()) if os.path.isdir('/sys/devices/system/node') else [0]
    mask = 0
    for n in nodes:
        mask |= 1 << n
    maskbuf = (C.c_ulong * 16)(*([mask & ((1 << 64) - 1)] + [0] * 15))
    applied = len(nodes) > 1 and _libc.syscall(C.c_long(_SYS_MBIND), C.c_void_p(ptr), C.c_ulong(size),
                                               C.c_int(_MPOL_INTERLEAVE), maskbuf, C.c_ulong(64 * 16),
                                               C.c_uint(0)) == 0
    _libc.madvise(C.c_void_p(ptr), size, _MADV_HUGEPAGE)
    if register is None:
        register = torch.cuda.is_available()
    registered = False
    if register:
        rc = torch.cuda.cudart().cudaHostRegister(ptr, size, 0)
        registered = int(rc) == 0 if not isinstance(rc, tuple) else int(rc[0]) == 0
    mp = _Mapping(ptr, size, registered)
    arr = np.ctypeslib.as_array((C.c_uint8 * size).from_address(ptr))
    t = torch.from_numpy(arr)[:nbytes]
    weakref.finalize(arr, mp.close)
    return t, dict(bytes=size, nodes=list(nodes), policy_applied=bool(applied), registered=registered, mapping=mp)
