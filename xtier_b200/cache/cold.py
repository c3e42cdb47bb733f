"""Cold experts: relayout files on NVMe drives, read on demand with O_DIRECT, and the manifest a restart reuses.

A record is one expert's shard for one node of the CPU engine, in the order of the engine's RAM slot: gate rows, up
rows, gate block scales, up block scales, down rows, down block scales, each piece padded to 512 bytes. That is the
order the C++ store writes (csrc/cold/store.cpp `xt_cold_write`) and the order the engine's miss path reads back into
a victim slot in one job (csrc/engine/engine.cpp `cold_ensure`). Records start on 4 KiB boundaries. The node shards of
one expert are dealt over the drives by weight (`parts`, e.g. 5:5:2 for two fast drives and a slower one), so one miss
reads from every drive at once.

Files: `<dir>/<key>.xtc` on every drive directory; the manifest `<first dir>/<key>.json`:

    {"version": 1, "key": ..., "drives": [...], "parts": [...], "end": [next free byte per drive],
     "layers": {"<layer>": {"shape": [H, I, fmt, nodes], "experts": E, "record": bytes,
                            "units": 1 or 3, "unit_bytes": [...],
                            "loc": [[drive, offset] for every (expert, node, unit), in that order],
                            "crc": [[crc32 of the first 4 KiB, of the last 4 KiB] per unit],
                            "source": [[name, size, mtime_ns] per checkpoint file], "g13": [...], "g2": [...]}}}

The manifest is rewritten (temporary file + rename) only after a layer's records are on the drives: the store
`fdatasync`s every record it writes. On restart a layer is reused when its shape, its layout and its source match and
the CRCs of its records check out; otherwise its records are written again. `<key>.ranges` beside the manifest keeps,
per layer, where each expert tensor sits in the checkpoint file it was loaded from (for `tools/cold_punch.py`).

Reference parity: docs/design-cold-experts.md (record = the engine slot's six pieces per NUMA shard, shards dealt over
drives by XTIER_COLD_PARTS, KEY.json with per-record CRC of the first / last 4 KiB and the checkpoint source id,
KEY.ranges, fill RAM slots from the store at start, decayed-use victim choice, XTIER_COLD_UNITS=3 records cut into
gate / up / rest units dealt over the drives), xtier/cache/cold.py:142-240 (manifest reuse), :248 LayerPlan, :454
attach. The byte-weighted dealing and the JSON fields are this project's.
"""
from __future__ import annotations

import json
import os
import zlib
from pathlib import Path

import numpy as np
import torch

from ..formats import NVFP4, ExpertWeights

VERSION = 1
ALIGN = 4096


def _pad(n: int, a: int = 512) -> int:
    return (n + a - 1) // a * a


def piece_bytes(H: int, I: int, fmt: str, nodes: int) -> list[int]:
    """Unpadded bytes of the six pieces of one node's shard (the engine's `slot_pieces` sizes)."""
    bs = 16 if fmt == NVFP4 else 32
    gr, dr = I // nodes, H // nodes
    return [gr * H // 2, gr * H // 2, gr * H // bs, gr * H // bs, dr * I // 2, dr * I // bs]


def record_bytes(H: int, I: int, fmt: str, nodes: int) -> int:
    return sum(_pad(b) for b in piece_bytes(H, I, fmt, nodes))


# A record can be cut into units dealt to drives of their own: 1 unit (the whole shard) or 3 (gate rows, up rows, the
# scales and down rows: about a third each), for drive sets whose speeds or count do not divide the shards evenly.
UNIT_GROUPS = {1: [[0, 1, 2, 3, 4, 5]], 3: [[0], [1], [2, 3, 4, 5]]}


def _dir_list(dirs) -> list:
    """Drive directories from a comma separated string, one path, or a list of paths."""
    if isinstance(dirs, str):
        return [d for d in dirs.split(',') if d]
    if isinstance(dirs, os.PathLike):
        return [dirs]
    return list(dirs)


def unit_bytes(H: int, I: int, fmt: str, nodes: int, units: int) -> list[int]:
    pb = piece_bytes(H, I, fmt, nodes)
    return [sum(_pad(pb[q]) for q in g) for g in UNIT_GROUPS[units]]


def shard_pieces(ew: ExpertWeights, e: int, n: int, nodes: int) -> list[np.ndarray]:
    """Expert e's pieces for node n as uint8 arrays (the bytes of the engine's RAM slot)."""
    I, H = ew.inter, ew.hidden
    gr, dr = I // nodes, H // nodes
    w13, s13, w2, s2 = (getattr(ew, f)[e].detach().cpu().contiguous() for f in ('w13', 's13', 'w2', 's2'))
    ps = [w13[n * gr:(n + 1) * gr], w13[I + n * gr:I + (n + 1) * gr], s13[n * gr:(n + 1) * gr],
          s13[I + n * gr:I + (n + 1) * gr], w2[n * dr:(n + 1) * dr], s2[n * dr:(n + 1) * dr]]
    return [p.contiguous().view(torch.uint8).numpy().reshape(-1) for p in ps]


def source_id(paths) -> list:
    """Identity of the checkpoint files a layer came from: [name, size, mtime_ns] each."""
    out = []
    for p in paths or []:
        st = os.stat(p)
        out.append([Path(p).name, st.st_size, st.st_mtime_ns])
    return out


def _aligned(n: int) -> np.ndarray:
    raw = np.empty(n + ALIGN, dtype=np.uint8)
    o = (-raw.ctypes.data) % ALIGN
    return raw[o:o + n]


def _crc_pair(buf: np.ndarray) -> list[int]:
    k = min(ALIGN, buf.size)
    return [zlib.crc32(buf[:k].tobytes()), zlib.crc32(buf[buf.size - k:].tobytes())]


def parse_parts(spec: str | None, drives: int) -> list[float]:
    """'5:5:2' -> weights per drive (default: equal)."""
    if not spec:
        return [1.0] * drives
    w = [float(x) for x in str(spec).split(':')]
    if len(w) != drives or min(w) <= 0:
        raise ValueError(f'cold parts {spec!r}: one positive weight per drive ({drives}) expected')
    return w


class ColdPool:
    """The cold-expert store of a model: record files on `dirs` (one per drive) and their manifest."""

    def __init__(self, dirs, key: str = 'xtier-cold', parts=None, threads: int = 4, units: int | None = None):
        from ..engine import ColdStore
        if units is None:
            from .. import config
            units = config.get('XTIER_COLD_UNITS')
        if units not in UNIT_GROUPS:
            raise ValueError(f'cold store: units must be one of {sorted(UNIT_GROUPS)}, got {units}')
        self.units = units
        self.dirs = [Path(d) for d in _dir_list(dirs)]
        if not self.dirs:
            raise ValueError('cold store: no directories')
        for d in self.dirs:
            d.mkdir(parents=True, exist_ok=True)
        self.key = key
        self.files = self.files_for(self.dirs, key)
        self.manifest_path = self.dirs[0] / f'{key}.json'
        self.ranges_path = self.dirs[0] / f'{key}.ranges'
        self.parts = parts if isinstance(parts, list) else parse_parts(parts, len(self.dirs))
        self.manifest = self._load_manifest()
        if self.manifest is None or self.manifest.get('drives') != self.files:
            # no manifest, or the drives changed: nothing on them can be trusted for this key
            self.manifest = dict(version=VERSION, key=key, drives=self.files, parts=self.parts,
                                 end=[0] * len(self.files), layers={})
        self.store = ColdStore(self.files, threads=threads, writable=True)

    @staticmethod
    def files_for(dirs, key: str) -> list[str]:
        return [str(Path(d) / f'{key}.xtc') for d in _dir_list(dirs)]

    # ---------------------------------------------------------------- manifest
    def _load_manifest(self):
        try:
            m = json.loads(self.manifest_path.read_text())
        except (OSError, ValueError):
            return None
        return m if m.get('version') == VERSION and m.get('key') == self.key else None

    def _save_manifest(self):
        tmp = self.manifest_path.with_suffix('.json.tmp')
        tmp.write_text(json.dumps(self.manifest))
        with open(tmp, 'rb') as f:
            os.fsync(f.fileno())
        os.replace(tmp, self.manifest_path)

    def layers(self) -> list[int]:
        return sorted(int(k) for k in self.manifest['layers'])

    def entry(self, layer: int) -> dict:
        return self.manifest['layers'][str(layer)]

    # ---------------------------------------------------------------- layout
    def _deal(self, E: int, nodes: int, usizes: list[int]) -> list[int]:
        """Drive of every (expert, node, unit): the drive that stays furthest below its weighted share of the bytes
        takes the next unit."""
        load = [0.0] * len(self.files)
        out = []
        for _ in range(E * nodes):
            for b in usizes:
                d = min(range(len(self.files)), key=lambda i: ((load[i] + b) / self.parts[i], i))
                load[d] += b
                out.append(d)
        return out

    def _allocate(self, layer: int, E: int, nodes: int, usizes: list[int]) -> list[list[int]]:
        old = self.manifest['layers'].get(str(layer))
        drives = self._deal(E, nodes, usizes)
        if old is not None and old.get('unit_bytes', [old['record']]) == usizes and len(old['loc']) == len(drives) \
                and [d for d, _ in old['loc']] == drives:
            return [list(x) for x in old['loc']]     # same sizes and dealing: rewrite in place
        loc = []
        for i, d in enumerate(drives):
            loc.append([d, self.manifest['end'][d]])
            self.manifest['end'][d] += _pad(usizes[i % len(usizes)], ALIGN)
        return loc

    @staticmethod
    def _units_of(ent: dict) -> tuple[int, list[int]]:
        return ent.get('units', 1), ent.get('unit_bytes', [ent['record']])

    # ---------------------------------------------------------------- write / check
    def write_layer(self, layer: int, ew: ExpertWeights, nodes: int, source=None, checkpoint: str | None = None,
                    tensor_ranges: dict | None = None):
        """Writes every record of the layer, then the manifest entry (and the checkpoint ranges when given)."""
        E, H, I = ew.experts, ew.hidden, ew.inter
        rec = record_bytes(H, I, ew.fmt, nodes)
        usizes = unit_bytes(H, I, ew.fmt, nodes, self.units)
        groups = UNIT_GROUPS[self.units]
        loc = self._allocate(layer, E, nodes, usizes)
        crc = []
        for e in range(E):
            for n in range(nodes):
                pieces = shard_pieces(ew, e, n, nodes)
                for u, g in enumerate(groups):
                    d, off = loc[(e * nodes + n) * len(groups) + u]
                    ps = [pieces[q] for q in g]
                    self.store.write(d, off, ps)
                    buf = np.zeros(usizes[u], dtype=np.uint8)
                    o = 0
                    for p in ps:
                        buf[o:o + p.size] = p
                        o += _pad(p.size)
                    crc.append(_crc_pair(buf))
        self.manifest['layers'][str(layer)] = dict(
            shape=[H, I, ew.fmt, nodes], experts=E, record=rec, units=self.units, unit_bytes=usizes, loc=loc,
            crc=crc, source=source or [],
            g13=ew.g13.detach().float().cpu().reshape(-1).tolist(), g2=ew.g2.detach().float().cpu().reshape(-1).tolist())
        self._save_manifest()
        if checkpoint is not None and tensor_ranges is not None:
            self._save_ranges(layer, checkpoint, tensor_ranges)

    def _save_ranges(self, layer: int, checkpoint: str, tensor_ranges: dict):
        try:
            r = json.loads(self.ranges_path.read_text())
        except (OSError, ValueError):
            r = {}
        r[str(layer)] = dict(file=str(checkpoint), tensors=tensor_ranges)
        tmp = self.ranges_path.with_suffix('.ranges.tmp')
        tmp.write_text(json.dumps(r))
        os.replace(tmp, self.ranges_path)

    def ranges(self) -> dict:
        try:
            return json.loads(self.ranges_path.read_text())
        except (OSError, ValueError):
            return {}

    def read_record(self, layer: int, e: int, n: int) -> np.ndarray:
        """The whole (expert, node) record (its units put back together in piece order)."""
        ent = self.entry(layer)
        N = ent['shape'][3]
        U, usizes = self._units_of(ent)
        buf = _aligned(ent['record'])
        files, offs, dst = [], [], []
        o = 0
        for u in range(U):
            d, off = ent['loc'][(e * N + n) * U + u]
            files.append(d)
            offs.append(off)
            dst.append(buf[o:].ctypes.data)
            o += usizes[u]
        self.store.read(files, offs, dst, usizes, 1)
        return buf

    def check_layer(self, layer: int) -> list[int]:
        """Indices ((expert * nodes + node) * units + unit) of the units whose first / last 4 KiB do not match their
        CRCs."""
        ent = self.entry(layer)
        U, usizes = self._units_of(ent)
        ks = [min(ALIGN, usizes[i % U]) for i in range(len(ent['loc']))]
        bad = []
        heads = [_aligned(k) for k in ks]
        tails = [_aligned(k) for k in ks]
        files = [d for d, _ in ent['loc']] * 2
        offs = [o for _, o in ent['loc']] + [o + usizes[i % U] - ks[i] for i, (_, o) in enumerate(ent['loc'])]
        try:
            self.store.read(files, offs, [b.ctypes.data for b in heads + tails], ks + ks, 1)
        except OSError:
            return list(range(len(ent['loc'])))
        for i, (h, t) in enumerate(zip(heads, tails)):
            if [zlib.crc32(h.tobytes()), zlib.crc32(t.tobytes())] != ent['crc'][i]:
                bad.append(i)
        return bad

    def layer_ok(self, layer: int, H: int, I: int, fmt: str, nodes: int, E: int, source=None) -> bool:
        ent = self.manifest['layers'].get(str(layer))
        if ent is None or ent['shape'] != [H, I, fmt, nodes] or ent['experts'] != E:
            return False
        if ent['record'] != record_bytes(H, I, fmt, nodes):
            return False
        U, usizes = self._units_of(ent)
        if U != self.units or usizes != unit_bytes(H, I, fmt, nodes, U):
            return False
        if source is not None and ent['source'] != source:
            return False
        if [d for d, _ in ent['loc']] != self._deal(E, nodes, usizes):
            return False
        return not self.check_layer(layer)

    def ensure_layer(self, layer: int, ew: ExpertWeights, nodes: int, source=None, checkpoint: str | None = None,
                     tensor_ranges: dict | None = None) -> bool:
        """True when the existing records were reused, False when they were (re)written."""
        if self.layer_ok(layer, ew.hidden, ew.inter, ew.fmt, nodes, ew.experts, source):
            if checkpoint is not None and tensor_ranges is not None:
                self._save_ranges(layer, checkpoint, tensor_ranges)
            return True
        self.write_layer(layer, ew, nodes, source, checkpoint, tensor_ranges)
        return False

    # ---------------------------------------------------------------- engine side
    def locations(self, layer: int) -> tuple[np.ndarray, np.ndarray]:
        """(file, offset) of every piece, [experts * nodes * 6] in (expert, node, piece) order."""
        ent = self.entry(layer)
        H, I, fmt, N = ent['shape']
        U, _ = self._units_of(ent)
        pb = piece_bytes(H, I, fmt, N)
        files, offs = [], []
        for i, (d, off) in enumerate(ent['loc']):
            o = off
            for q in UNIT_GROUPS[U][i % U]:
                files.append(d)
                offs.append(o)
                o += _pad(pb[q])
        return np.asarray(files, dtype=np.int32), np.asarray(offs, dtype=np.int64)

    def scales(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        ent = self.entry(layer)
        return (torch.tensor(ent['g13'], dtype=torch.float32).view(-1, 2),
                torch.tensor(ent['g2'], dtype=torch.float32))

    def attach(self, engine, layer: int, scores=None, half_life: float = 50.0):
        """Makes the engine read its misses of this layer from the store (and take each expert's global scales)."""
        ent = self.entry(layer)
        if engine.nodes() != ent['shape'][3]:
            raise ValueError(f'cold layer {layer}: records are for {ent["shape"][3]} nodes, the engine has '
                             f'{engine.nodes()}')
        g13, g2 = self.scales(layer)
        engine.set_expert_scales(g13, g2)
        files, offs = self.locations(layer)
        engine.attach_cold_pieces(self.store, files, offs, scores, half_life)

    def fill_engine(self, engine, layer: int, resident):
        """Reads the resident experts' records straight into the engine's RAM slots (start-up without the
        checkpoint's expert tensors): slot s <- expert resident[s]."""
        ent = self.entry(layer)
        N = ent['shape'][3]
        pf, po = self.locations(layer)
        files, offs, dst, sizes = [], [], [], []
        for s, e in enumerate(resident):
            if e < 0:
                engine.place(-1, s)
                continue
            engine.place(int(e), s)
            for n in range(N):
                ptrs, szs = engine.slot_pieces(s, n)
                base = (int(e) * N + n) * 6
                files += pf[base:base + 6].tolist()
                offs += po[base:base + 6].tolist()
                dst += ptrs
                sizes += [_pad(b) for b in szs]
        if files:
            self.store.read(files, offs, dst, sizes, 1)

    def load_layer(self, layer: int) -> ExpertWeights:
        """The layer's experts rebuilt from the records (the only copy once the checkpoint's tensors are punched)."""
        ent = self.entry(layer)
        H, I, fmt, N = ent['shape']
        E = ent['experts']
        bs = 16 if fmt == NVFP4 else 32
        w13 = np.empty((E, 2 * I, H // 2), np.uint8)
        s13 = np.empty((E, 2 * I, H // bs), np.uint8)
        w2 = np.empty((E, H, I // 2), np.uint8)
        s2 = np.empty((E, H, I // bs), np.uint8)
        sz = piece_bytes(H, I, fmt, N)
        gr, dr = I // N, H // N
        for e in range(E):
            for n in range(N):
                buf = self.read_record(layer, e, n)
                o, parts = 0, []
                for b in sz:
                    parts.append(buf[o:o + b])
                    o += _pad(b)
                w13[e, n * gr:(n + 1) * gr] = parts[0].reshape(gr, -1)
                w13[e, I + n * gr:I + (n + 1) * gr] = parts[1].reshape(gr, -1)
                s13[e, n * gr:(n + 1) * gr] = parts[2].reshape(gr, -1)
                s13[e, I + n * gr:I + (n + 1) * gr] = parts[3].reshape(gr, -1)
                w2[e, n * dr:(n + 1) * dr] = parts[4].reshape(dr, -1)
                s2[e, n * dr:(n + 1) * dr] = parts[5].reshape(dr, -1)
        g13, g2 = self.scales(layer)
        return ExpertWeights(fmt, torch.from_numpy(w13), torch.from_numpy(w2), torch.from_numpy(s13),
                             torch.from_numpy(s2), g13, g2)

    def stats(self) -> dict:
        return self.store.stats()

    def close(self):
        if self.store is not None:
            self.store.close()
            self.store = None


_HOST_STAGE: dict = {}   # (experts, H, I, fmt, parity, pinned) -> [host staging, event of its last upload or None]


class ColdPrefill:
    """The host side of a GPU prefill of a layer whose CPU-tier experts live in a cold-backed engine (RAM slots plus
    the drive store), so that no full host copy of the layer is kept.

    The layer's non-GPU experts (`cold`, in staging order) are gathered into a host staging buffer in the expert
    layout the GPU staging pool uses: an expert in one of the engine's RAM slots is copied from the slot (pinned
    while it is copied, so a concurrent miss cannot evict it), any other one is read from its records with O_DIRECT
    straight into its rows (through a bounce buffer when a piece is not a whole number of 512-byte blocks). Two host
    buffers per shape are shared by all layers (layer parity); a fill first waits until the previous upload out of
    its buffer is done. `start()` runs the fill on a thread (the next layer's read-ahead while this layer computes);
    `stage()` waits for it (or fills now) and returns the buffer.
    (Reference parity: xtier/cache/cold.py:646-790 PrefillCold -- cold experts read into a pinned staging by layer
    parity, the next layer read ahead; here RAM-slot experts come from the engine, and every non-GPU expert is staged
    since the routes of the next layer are not known yet.)
    """

    def __init__(self, pool: ColdPool, layer: int, engine, cold):
        ent = pool.entry(layer)
        self.H, self.I, self.fmt, self.N = ent['shape']
        self.pool, self.layer, self.engine = pool, layer, engine
        self.cold = [int(e) for e in cold]
        self.K = len(self.cold)
        self.bs = 16 if self.fmt == NVFP4 else 32
        self.files, self.offs = pool.locations(layer)
        self.g13, self.g2 = pool.scales(layer)     # every expert's global scales
        self.pb = piece_bytes(self.H, self.I, self.fmt, self.N)
        self.pinned = torch.cuda.is_available()
        self._thread = None
        self._box: dict = {}
        self.stats = dict(fills=0, from_ram=0, from_drive=0, bytes_read=0, wait_s=0.0)

    # ------------------------------------------------------------------ buffers
    def _key(self):
        return (self.K, self.H, self.I, self.fmt, self.layer % 2, self.pinned)

    def _buffer(self) -> list:
        cur = _HOST_STAGE.get(self._key())
        if cur is None:
            K, H, I, bs = self.K, self.H, self.I, self.bs
            shapes = [('w13', (K, 2 * I, H // 2), torch.uint8), ('w2', (K, H, I // 2), torch.uint8),
                      ('s13', (K, 2 * I, H // bs), torch.uint8), ('s2', (K, H, I // bs), torch.uint8),
                      ('g13', (K, 2), torch.float32), ('g2', (K,), torch.float32)]
            sizes = [_pad(int(np.prod(sh)) * torch.tensor([], dtype=dt).element_size(), ALIGN) for _, sh, dt in shapes]
            raw = torch.empty(sum(sizes) + ALIGN, dtype=torch.uint8, pin_memory=self.pinned)
            o = (-raw.data_ptr()) % ALIGN
            fields = {}
            for (name, sh, dt), n in zip(shapes, sizes):
                nb = int(np.prod(sh)) * torch.tensor([], dtype=dt).element_size()
                fields[name] = raw[o:o + nb].view(dt).view(sh)
                o += n
            cur = _HOST_STAGE[self._key()] = [ExpertWeights(self.fmt, *(fields[f] for f in
                                                                         ('w13', 'w2', 's13', 's2', 'g13', 'g2'))),
                                              None]
        return cur

    def uploaded(self, event):
        """The upload out of this layer's host buffer was enqueued; `event` completes with it."""
        self._buffer()[1] = event

    # ------------------------------------------------------------------ fill
    def _dests(self, st: ExpertWeights, i: int, n: int) -> list[int]:
        """Addresses of staging row i's six pieces for node n (the rows a node shard covers are contiguous)."""
        H, I, N, bs = self.H, self.I, self.N, self.bs
        gr, dr = I // N, H // N
        w13, s13, w2, s2 = st.w13.data_ptr(), st.s13.data_ptr(), st.w2.data_ptr(), st.s2.data_ptr()
        return [w13 + (i * 2 * I + n * gr) * (H // 2), w13 + (i * 2 * I + I + n * gr) * (H // 2),
                s13 + (i * 2 * I + n * gr) * (H // bs), s13 + (i * 2 * I + I + n * gr) * (H // bs),
                w2 + (i * H + n * dr) * (I // 2), s2 + (i * H + n * dr) * (I // bs)]

    def fill(self, st: ExpertWeights, experts=None):
        """Gathers `experts` (default: every non-GPU expert, in staging order) into rows 0.. of `st` (synchronous)."""
        import ctypes
        experts = list(self.cold) if experts is None else [int(e) for e in experts]
        files, offs, dst, sizes, bounce = [], [], [], [], []
        for i, e in enumerate(experts):
            slot = self.engine.pin(e) if self.engine is not None else -1
            try:
                if slot >= 0:
                    for n in range(self.N):
                        ptrs, szs = self.engine.slot_pieces(slot, n)
                        for d, sp, b in zip(self._dests(st, i, n), ptrs, szs):
                            ctypes.memmove(d, sp, b)
                    self.stats['from_ram'] += 1
                    continue
            finally:
                if slot >= 0:
                    self.engine.unpin(slot)
            for n in range(self.N):
                base = (e * self.N + n) * 6
                for q, d in enumerate(self._dests(st, i, n)):
                    b = self.pb[q]
                    files.append(int(self.files[base + q]))
                    offs.append(int(self.offs[base + q]))
                    if b % 512 == 0 and d % 512 == 0:
                        dst.append(d)
                    else:   # a ragged piece: read its padded bytes aside, copy the piece
                        buf = _aligned(_pad(b))
                        bounce.append((d, buf, b))
                        dst.append(buf.ctypes.data)
                    sizes.append(_pad(b))
            self.stats['from_drive'] += 1
        if files:
            self.pool.store.read(files, offs, dst, sizes, 1)
            self.stats['bytes_read'] += sum(sizes)
        for d, buf, b in bounce:
            ctypes.memmove(d, buf.ctypes.data, b)
        idx = torch.tensor(experts, dtype=torch.long)
        st.g13[:len(experts)].copy_(self.g13[idx])
        st.g2[:len(experts)].copy_(self.g2[idx])
        self.stats['fills'] += 1

    def read_experts(self, experts) -> ExpertWeights:
        """The given experts gathered into fresh host tensors (e.g. the source of a GPU slot swap)."""
        n, H, I, bs = len(experts), self.H, self.I, self.bs
        st = ExpertWeights(self.fmt, torch.empty(n, 2 * I, H // 2, dtype=torch.uint8),
                           torch.empty(n, H, I // 2, dtype=torch.uint8),
                           torch.empty(n, 2 * I, H // bs, dtype=torch.uint8),
                           torch.empty(n, H, I // bs, dtype=torch.uint8),
                           torch.empty(n, 2, dtype=torch.float32), torch.empty(n, dtype=torch.float32))
        self.fill(st, experts)
        return st

    def _run(self, cur: list):
        import time
        t0 = time.perf_counter()
        try:
            st, ev = cur
            if ev is not None:   # the previous layer of this parity has its upload out of the buffer done
                dev = getattr(ev, 'device', None)
                if dev is not None:
                    torch.cuda.set_device(dev)   # this thread's current device is the event's
                ev.synchronize()
            self.fill(st)
        except BaseException as ex:   # re-raised by stage()
            self._box['err'] = ex
        self._box['s'] = time.perf_counter() - t0

    def start(self):
        """Starts the fill on a thread (no-op while one runs)."""
        import threading
        if self._thread is None:
            self._box = {}
            cur = list(self._buffer())   # allocated (pinned) on the caller's thread and device
            self._thread = threading.Thread(target=self._run, args=(cur,), daemon=True,
                                            name=f'xtier-cold-prefill-{self.layer}')
            self._thread.start()

    def stage(self) -> ExpertWeights:
        """The filled host buffer: waits for a started fill, or fills now."""
        import time
        t0 = time.perf_counter()
        if self._thread is None:
            self.start()
        self._thread.join()
        self._thread = None
        self.stats['wait_s'] += time.perf_counter() - t0
        if 'err' in self._box:
            raise self._box['err']
        return self._buffer()[0]


def open_layer(pool: ColdPool, layer: int, path, nodes: int, prefix: str = 'experts.') -> ExpertWeights:
    """One layer's experts for a cold-backed engine: read from its checkpoint file (the records are written or
    checked against it and the tensor ranges kept for punching), or, once the file's expert tensors were punched out,
    rebuilt from the store alone (whose records must then check out)."""
    from ..checkpoint import cold_only, expert_ranges, load_experts
    if cold_only(path):
        if str(layer) not in pool.manifest['layers'] or pool.check_layer(layer):
            raise RuntimeError(f'{path}: expert tensors were punched out but the cold store has no intact records of '
                               f'layer {layer}; restore the file with tools/cold_punch.py --restore')
        return pool.load_layer(layer)
    ew = load_experts(path, prefix)
    pool.ensure_layer(layer, ew, nodes, source_id([path]), checkpoint=str(path),
                      tensor_ranges=expert_ranges(path, prefix))
    return ew


def ram_resident(E: int, slots: int, popularity, gpu_hot=()) -> list[int]:
    """Experts kept in the engine's RAM slots: the most popular experts the GPU does not serve first (the CPU
    computes those), then GPU-hot ones; `popularity` is any per-expert score (router bias, measured counts)."""
    pop = np.asarray(popularity, dtype=np.float64)
    hot = set(int(e) for e in gpu_hot)
    order = sorted(range(E), key=lambda e: (e in hot, -pop[e], e))
    return order[:slots]


def cold_engine(layer: int, host: ExpertWeights, pool: ColdPool, cold_fraction: float, popularity, gpu_hot=(),
                threads: int | None = None, source=None, half_life: float | None = None):
    """A CPU engine whose RAM holds (1 - cold_fraction) of the layer's experts, the rest read on demand from `pool`
    (records written or reused first)."""
    from ..engine import CpuEngine
    E = host.experts
    slots = max(1, E - int(round(cold_fraction * E)))
    resident = ram_resident(E, slots, popularity, gpu_hot)
    probe = CpuEngine(host.select(torch.arange(1)), threads=threads, slots=1, fill=False)
    nodes = probe.nodes()
    probe.close()
    pool.ensure_layer(layer, host, nodes, source)
    eng = CpuEngine(host, threads=threads, slots=slots, resident=resident)
    scores = np.zeros(E, np.float32)
    scores[resident] = np.linspace(1.0, 0.5, len(resident), dtype=np.float32)   # initial use counts by rank
    for e in gpu_hot:
        scores[int(e)] = 0.0
    if half_life is None:
        from .. import config
        half_life = config.get('XTIER_COLD_HALF_LIFE')
    pool.attach(eng, layer, scores, half_life)
    return eng
