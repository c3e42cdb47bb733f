"""NVMe row tables (libxt_rows.so): huge embedding-like tables kept on NVMe and looked up by row id.

`RowStore` opens a table made of segments (a checkpoint tensor split over files, or a relayout file) and returns rows
(and their optional scale bytes) for a batch of ids; misses are read with O_DIRECT, deduplicated per page, and kept in
a direct-mapped row cache. `GraphLookup` (xtier_b200.tables.lookup) performs the lookup inside a CUDA graph.

Reference parity: xtier/tables/__init__.py:48-129 (RowStore, Segment, tensor_locations), csrc/tables/rows.cpp.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
from pathlib import Path

import numpy as np

from .. import config

_LIB = Path(__file__).resolve().parent.parent / '_lib' / 'libxt_rows.so'
_lib = None


def lib():
    global _lib
    if _lib is None:
        if not _LIB.exists():
            from .. import _build
            _build.build(cuda=False, verbose=False)
        L = C.CDLL(str(_LIB))
        L.xt_rows_open.restype = C.c_void_p
        L.xt_rows_open.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_longlong, C.c_longlong, C.c_int, C.c_longlong, C.c_int]
        L.xt_rows_lookup.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]
        L.xt_rows_prefetch.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
        L.xt_rows_range.argtypes = [C.c_void_p, C.c_longlong, C.c_longlong]
        L.xt_rows_stats.argtypes = [C.c_void_p, C.c_void_p]
        L.xt_rows_close.argtypes = [C.c_void_p]
        L.xt_rows_error.restype = C.c_char_p
        _lib = L
    return _lib


@dataclasses.dataclass
class Segment:
    """Rows [first, first + count) of the table, stored at byte `offset` of `path` (scales at `scale_offset`)."""
    path: str
    first: int
    count: int
    offset: int
    scale_offset: int = -1


class RowStore:
    def __init__(self, segments: list[Segment], row_bytes: int, scale_bytes: int = 0, io_threads: int | None = None,
                 cache_rows: int | None = None, mode: str | None = None):
        self.row_bytes, self.scale_bytes = row_bytes, scale_bytes
        n = len(segments)
        paths = (C.c_char_p * n)(*[s.path.encode() for s in segments])
        arr = lambda v: np.ascontiguousarray(v, dtype=np.int64)
        self._keep = [arr([s.first for s in segments]), arr([s.count for s in segments]),
                      arr([s.offset for s in segments]), arr([s.scale_offset for s in segments])]
        io = io_threads if io_threads is not None else config.get('XTIER_ROWS_IO_THREADS')
        if cache_rows is None:
            cache_rows = config.get('XTIER_ROWS_CACHE_MB') * (1 << 20) // max(1, row_bytes + scale_bytes)
        mode = mode or config.get('XTIER_ROWS_MODE')
        self.handle = lib().xt_rows_open(paths, *[a.ctypes.data for a in self._keep], n, row_bytes, scale_bytes, io,
                                         cache_rows, 1 if mode == 'ram' else 0)
        if not self.handle:
            raise OSError(lib().xt_rows_error().decode())
        self.rows = max(s.first + s.count for s in segments)

    def lookup(self, ids, rows_out: np.ndarray | None = None, scales_out: np.ndarray | None = None):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        n = ids.size
        if rows_out is None:
            rows_out = np.empty((n, self.row_bytes), dtype=np.uint8)
        if self.scale_bytes and scales_out is None:
            scales_out = np.empty((n, self.scale_bytes), dtype=np.uint8)
        rc = lib().xt_rows_lookup(self.handle, ids.ctypes.data, n, rows_out.ctypes.data,
                                  scales_out.ctypes.data if scales_out is not None else None)
        if rc != 0:
            raise IndexError(lib().xt_rows_error().decode())
        return (rows_out, scales_out) if self.scale_bytes else rows_out

    def lookup_ptr(self, ids_ptr: int, n: int, rows_ptr: int, scales_ptr: int | None = None):
        if lib().xt_rows_lookup(self.handle, ids_ptr, n, rows_ptr, scales_ptr) != 0:
            raise IndexError(lib().xt_rows_error().decode())

    def prefetch(self, ids):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        lib().xt_rows_prefetch(self.handle, ids.ctypes.data, ids.size)

    def set_range(self, lo: int, hi: int):
        """Tensor parallelism: rows outside [lo, hi) read as zeros on this rank."""
        lib().xt_rows_range(self.handle, lo, hi)

    def stats(self) -> dict:
        out = (C.c_double * 6)()
        lib().xt_rows_stats(self.handle, out)
        return dict(zip(('lookups', 'rows', 'hits', 'misses', 'pages', 'bytes'), list(out)))

    def close(self):
        if self.handle:
            lib().xt_rows_close(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def write_table(path: str | Path, data: np.ndarray, scales: np.ndarray | None = None, segments: int = 1,
                align: int = 4096) -> list[Segment]:
    """Writes `data` [rows, row_bytes] (uint8) into `segments` files named path.N and returns their Segment list
    (each segment's rows, then its scales, every part aligned to `align`)."""
    rows = data.shape[0]
    per = (rows + segments - 1) // segments
    segs = []
    for s in range(segments):
        lo, hi = s * per, min(rows, (s + 1) * per)
        if lo >= hi:
            break
        p = f'{path}.{s}'
        with open(p, 'wb') as f:
            f.write(b'\0' * 512)   # a header gap, so segments do not start at offset 0
            off = 512
            f.write(data[lo:hi].tobytes())
            soff = -1
            if scales is not None:
                pos = off + (hi - lo) * data.shape[1]
                pad = (-pos) % align
                f.write(b'\0' * pad)
                soff = pos + pad
                f.write(scales[lo:hi].tobytes())
        segs.append(Segment(p, lo, hi - lo, off, soff))
    return segs
