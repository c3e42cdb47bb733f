"""Hashed bigram embedding rows from an NVMe row table, added to the residual stream (the lookup of DeepSeek V4's
Engram memory, and of the three-tier benchmark's 32 GiB table).

Each token t at a position with previous token p reads row hash(p, t) mod rows of the table: the 64-bit key
(p << 32) | t goes through the SplitMix64 finalizer (Steele, Lea and Flood, "Fast splittable pseudorandom number
generators", 2014: xor-shift 30, multiply, xor-shift 27, multiply, xor-shift 31), computed on the device in int64
with logical shifts, so the ids never leave the GPU before the lookup. The BF16 rows [dim] come from `RowStore` (page
cache, NVMe with O_DIRECT, row cache); in decode the lookup runs inside the CUDA
graph (`GraphLookup`: device->host ids, a host-function node running the C++ lookup, host->device rows) and the rows
are projected to the hidden size when the table's width differs (a BF16 [hidden, dim] matrix) and added to the
token's embedding. Prefill looks its rows up directly.
(Reference parity: xtier/tables/lookup.py:47-93 and xtier/packs/deepseek_v4/__init__.py (Engram `_init`,
`_owned_rows`, `_prefetch`): rows of an NVMe table looked up inside the graph with a row cache.)
"""
from __future__ import annotations

import numpy as np
import torch

_M1 = -4658895280553007687    # 0xbf58476d1ce4e5b9 as a signed 64-bit integer
_M2 = -7723592293110705685    # 0x94d049bb133111eb


def _lsr(x: torch.Tensor, k: int) -> torch.Tensor:
    """Logical right shift of int64 lanes."""
    return (x >> k) & ((1 << (64 - k)) - 1)


def bigram_rows(prev: torch.Tensor, cur: torch.Tensor, rows: int, seed: int = 0) -> torch.Tensor:
    """Row ids (int64) of the (previous, current) token pairs: SplitMix64 finalizer of (prev << 32 | cur) ^ seed."""
    z = (prev.long() << 32) | (cur.long() & 0xFFFFFFFF)
    z = z ^ seed
    z = (z ^ _lsr(z, 30)) * _M1
    z = (z ^ _lsr(z, 27)) * _M2
    z = z ^ _lsr(z, 31)
    return (z & 0x7FFFFFFFFFFFFFFF) % rows


def bigram_rows_reference(prev, cur, rows: int, seed: int = 0) -> np.ndarray:
    """The same hash in Python integers (the tests' oracle)."""
    out = []
    mask = (1 << 64) - 1
    for p, c in zip(np.asarray(prev).tolist(), np.asarray(cur).tolist()):
        z = (((p << 32) | (c & 0xFFFFFFFF)) ^ seed) & mask
        z = ((z ^ (z >> 30)) * 0xbf58476d1ce4e5b9) & mask
        z = ((z ^ (z >> 27)) * 0x94d049bb133111eb) & mask
        z = z ^ (z >> 31)
        out.append((z & 0x7FFFFFFFFFFFFFFF) % rows)
    return np.asarray(out, dtype=np.int64)


class BigramTable:
    """An NVMe table of `rows` BF16 rows of width `dim`, added (through `proj` [hidden, dim] when dim != hidden) to
    the embeddings of `batch` decode tokens inside the graph, and of whole prompts in prefill."""

    def __init__(self, store, rows: int, dim: int, hidden: int, batch: int = 1, device='cuda', seed: int = 0,
                 proj: torch.Tensor | None = None):
        from .lookup import GraphLookup
        if store.row_bytes != dim * 2 or store.scale_bytes:
            raise ValueError('BigramTable: BF16 rows of width dim expected')
        if dim != hidden and proj is None:
            raise ValueError('BigramTable: a [hidden, dim] projection is needed when dim != hidden')
        self.store, self.rows, self.dim, self.hidden, self.seed = store, rows, dim, hidden, seed
        self.device = torch.device(device)
        self.proj = None if proj is None else proj.to(self.device, torch.bfloat16).contiguous()
        self.lookup = GraphLookup(store, batch, self.device)
        self.ids = torch.zeros(batch, dtype=torch.int64, device=self.device)
        self.delta = torch.empty(batch, hidden, dtype=torch.bfloat16, device=self.device)

    def _project(self, r: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from .. import ops
        if self.proj is None:
            return r if out is None else out.copy_(r)
        return ops.linear(r, self.proj, out=out)

    def add_decode(self, x: torch.Tensor, prev: torch.Tensor, cur: torch.Tensor):
        """x [batch, hidden] += rows of (prev, cur); graph-capturable."""
        self.ids.copy_(bigram_rows(prev, cur, self.rows, self.seed))
        raw = self.lookup.fetch(self.ids)
        r = raw.view(torch.bfloat16).view(-1, self.dim)
        x.add_(self._project(r, self.delta))

    def rows_host(self, prev, cur) -> torch.Tensor:
        """BF16 [n, dim] rows of the pairs, looked up directly (prefill, reference)."""
        ids = bigram_rows(torch.as_tensor(prev).cpu(), torch.as_tensor(cur).cpu(), self.rows, self.seed)
        raw = self.store.lookup(ids.numpy())
        return torch.from_numpy(np.ascontiguousarray(raw)).view(torch.bfloat16).view(-1, self.dim)

    def prefetch_rows(self, tokens: torch.Tensor, prev0: int):
        """Starts reading the rows of a later prompt chunk on a thread (the look-ahead of a chunked prefill); returns a
        future whose result `add_prefill(..., rows=)` takes."""
        import concurrent.futures as cf
        if not hasattr(self, '_ahead'):
            self._ahead = cf.ThreadPoolExecutor(1, thread_name_prefix='xtier-engram-ahead')
        t = tokens.detach().cpu().long()
        prev = torch.cat([torch.tensor([prev0]), t[:-1]])
        return self._ahead.submit(self.rows_host, prev, t)

    def add_prefill(self, x: torch.Tensor, tokens: torch.Tensor, prev0: int = 0, rows: torch.Tensor | None = None):
        """x [T, hidden] += rows of the prompt's pairs (the first token's previous one is prev0); `rows`: the BF16
        rows already read (prefetch_rows)."""
        if rows is None:
            t = tokens.detach().cpu().long()
            prev = torch.cat([torch.tensor([prev0]), t[:-1]])
            rows = self.rows_host(prev, t)
        x.add_(self._project(rows.to(x.device)))

    def check(self):
        self.lookup.check()


def synthetic_table(path, rows: int, dim: int, std: float = 0.02, seed: int = 0, segments: int = 1,
                    chunk_rows: int = 65536, device=None) -> list:
    """Writes a [rows, dim] BF16 table of N(0, std) values into `segments` files path.N, chunk by chunk (a 32 GiB
    table never sits in memory), in the layout of `tables.write_table` (a 512-byte header gap, then the rows), and
    returns its Segment list. The chunk starting at row r is drawn from a generator seeded by (seed, r) (on
    `device`, default the GPU when there is one), so the table's bytes depend on its shape and seed only. A table
    written before with the same shape, std and seed (a sidecar path.json) is reused."""
    import json
    import os
    from . import Segment
    if device is None:
        device = 'cuda' if torch.cuda.is_available() else 'cpu'
    meta = dict(rows=rows, dim=dim, std=std, seed=seed, segments=segments, chunk_rows=chunk_rows)
    per = (rows + segments - 1) // segments
    bounds = [(s * per, min(rows, (s + 1) * per)) for s in range(segments) if s * per < rows]
    segs = [Segment(f'{path}.{s}', lo, hi - lo, 512) for s, (lo, hi) in enumerate(bounds)]
    side = f'{path}.json'
    try:
        with open(side) as f:
            same = json.load(f) == meta
    except (OSError, ValueError):
        same = False
    if same and all(os.path.exists(g.path) and os.path.getsize(g.path) == 512 + g.count * dim * 2 for g in segs):
        return segs
    for g in segs:
        with open(g.path, 'wb') as f:
            f.write(b'\0' * 512)
            for lo in range(g.first, g.first + g.count, chunk_rows):
                hi = min(g.first + g.count, lo + chunk_rows)
                gen = torch.Generator(device=device).manual_seed(seed * 1000003 + lo)
                x = (torch.randn(hi - lo, dim, generator=gen, device=device) * std).bfloat16()
                f.write(x.view(torch.uint8).cpu().numpy().tobytes())
    with open(side, 'w') as f:
        json.dump(meta, f)
    return segs
