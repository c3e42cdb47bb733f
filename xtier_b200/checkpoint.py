"""Expert checkpoints in safetensors files, and the fast loader.

`save_experts` writes one MoE layer's quantized experts (the engine layout: `w13 [E, 2I, H/2]`, `w2 [E, H, I/2]`,
block scales `s13`, `s2`, global scales `g13 [E, 2]`, `g2 [E]`) as a standard safetensors file (8-byte little-endian
header length, JSON header of dtype / shape / data_offsets, then the tensor bytes), with an `xtier.fmt` entry in the
metadata.

`load_experts(..., direct=True)` is the fast path: it parses the header, then reads every tensor with O_DIRECT through
the C++ cold store's reader threads (csrc/cold/store.cpp) straight into page-aligned buffers -- the 512-byte-aligned
window around each tensor, in 64 MiB pieces spread over the threads -- bypassing the page cache, so a multi-GB layer
streams at the drive's bandwidth instead of through one Python read. `direct=False` is the plain reader (numpy from
an mmap) and the oracle of the tests.
(Reference parity: xtier/backend/direct.py:90-315 -- locate each expert tensor's byte range in the checkpoint files and
read them with O_DIRECT into the engine's memory; check_scales, digest.)
"""
from __future__ import annotations

import json
import struct

import numpy as np
import torch

from .formats import ExpertWeights

_DT = {'U8': (np.uint8, torch.uint8), 'F32': (np.float32, torch.float32), 'BF16': (np.uint16, torch.bfloat16),
       'I32': (np.int32, torch.int32)}
_NAMES = ('w13', 'w2', 's13', 's2', 'g13', 'g2')
PIECE = 64 << 20


def _st_dtype(t: torch.Tensor) -> str:
    return {torch.uint8: 'U8', torch.float32: 'F32', torch.bfloat16: 'BF16', torch.int32: 'I32'}[t.dtype]


def save_experts(path, ew: ExpertWeights, prefix: str = 'experts.'):
    """One layer's experts -> a safetensors file (tensors `<prefix>w13`, ...)."""
    tensors = {prefix + n: getattr(ew, n).detach().to('cpu').contiguous() for n in _NAMES}
    header, off = {'__metadata__': {'xtier.fmt': ew.fmt}}, 0
    for name, t in tensors.items():
        nb = t.numel() * t.element_size()
        header[name] = {'dtype': _st_dtype(t), 'shape': list(t.shape), 'data_offsets': [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(',', ':')).encode()
    hb += b' ' * ((8 - len(hb) % 8) % 8)
    with open(path, 'wb') as f:
        f.write(struct.pack('<Q', len(hb)))
        f.write(hb)
        for t in tensors.values():
            f.write(t.view(torch.uint8).numpy().tobytes() if t.dtype != torch.bfloat16 else
                    t.view(torch.int16).numpy().tobytes())


def read_header(path) -> tuple[dict, int]:
    """(header dict, byte offset of the data section)."""
    with open(path, 'rb') as f:
        n = struct.unpack('<Q', f.read(8))[0]
        return json.loads(f.read(n)), 8 + n


MARKER = 'XTIER-COLD-ONLY'


def expert_ranges(path, prefix: str = 'experts.') -> dict:
    """Where each expert tensor of a layer file sits: {name: [absolute byte offset, bytes per expert]} for the four
    tensors a cold record holds (codes and block scales; the global scales stay in the file)."""
    header, data0 = read_header(path)
    out = {}
    for n in ('w13', 's13', 'w2', 's2'):
        h = header[prefix + n]
        a, b = h['data_offsets']
        out[n] = [data0 + a, (b - a) // h['shape'][0]]
    return out


def cold_only(path) -> bool:
    """True when `path` is listed in the punch marker beside it: its expert tensors live only in the cold store."""
    import os
    from pathlib import Path
    m = Path(path).parent / MARKER
    if not m.exists():
        return False
    try:
        files = json.loads(m.read_text()).get('files', {})
    except ValueError:
        return True     # an unreadable marker: refuse rather than read zeros
    return Path(path).name in files or str(path) in files


def _aligned(nbytes: int) -> np.ndarray:
    raw = np.empty(nbytes + 4096, dtype=np.uint8)
    o = (-raw.ctypes.data) % 4096
    return raw[o:o + nbytes]


def load_experts(path, prefix: str = 'experts.', direct: bool | None = None, threads: int = 8) -> ExpertWeights:
    """direct=None follows XTIER_FAST_LOAD."""
    if cold_only(path):
        raise RuntimeError(f'{path}: its expert tensors were punched out (marker {MARKER}); load this layer from the '
                           'cold store (ColdPool.load_layer / fill_engine) or restore it with tools/cold_punch.py '
                           '--restore')
    if direct is None:
        from . import config
        direct = bool(config.get('XTIER_FAST_LOAD'))
    header, data0 = read_header(path)
    fmt = header.get('__metadata__', {}).get('xtier.fmt')
    out = {}
    if not direct:
        mm = np.memmap(path, dtype=np.uint8, mode='r')
        for n in _NAMES:
            h = header[prefix + n]
            a, b = h['data_offsets']
            npdt, tdt = _DT[h['dtype']]
            arr = np.array(mm[data0 + a:data0 + b]).view(npdt).reshape(h['shape'])
            out[n] = torch.from_numpy(arr).view(tdt) if tdt == torch.bfloat16 else torch.from_numpy(arr)
        return ExpertWeights(fmt, *[out[n] for n in _NAMES])
    import os
    from .engine import ColdStore
    fsz = os.path.getsize(path)
    full = fsz // 512 * 512          # O_DIRECT covers whole 512-byte sectors; the file's last partial one is read plainly
    tails = []
    store = ColdStore([str(path)], threads=threads, writable=False)
    try:
        jobs = []   # (file offset, size, destination array)
        for n in _NAMES:
            h = header[prefix + n]
            a, b = h['data_offsets']
            lo = (data0 + a) // 512 * 512
            hi = (data0 + b + 511) // 512 * 512
            buf = _aligned(hi - lo)
            out[n] = (buf, data0 + a - lo, b - a, h)
            dhi = min(hi, full)
            for p in range(0, max(0, dhi - lo), PIECE):
                jobs.append((lo + p, min(PIECE, dhi - lo - p), buf[p:]))
            if hi > dhi:
                tails.append((max(lo, dhi), buf[max(lo, dhi) - lo:]))
        if jobs:
            store.read([0] * len(jobs), [j[0] for j in jobs], [j[2].ctypes.data for j in jobs],
                       [j[1] for j in jobs], 1)
    finally:
        store.close()
    if tails:
        with open(path, 'rb') as f:
            for off, dst in tails:
                f.seek(off)
                chunk = f.read(fsz - off)
                dst[:len(chunk)] = np.frombuffer(chunk, dtype=np.uint8)
    res = []
    for n in _NAMES:
        buf, skip, nb, h = out[n]
        npdt, tdt = _DT[h['dtype']]
        arr = buf[skip:skip + nb].view(npdt).reshape(h['shape']).copy()
        res.append(torch.from_numpy(arr).view(tdt) if tdt == torch.bfloat16 else torch.from_numpy(arr))
    return ExpertWeights(fmt, *res)


def check_scales(ew: ExpertWeights) -> bool:
    """Sanity check of a loaded layer: finite, positive global scales and block-scale bytes that decode to finite
    values (NaN E4M3 codes 0x7F / 0xFF are rejected)."""
    ok = bool(torch.isfinite(ew.g13.float()).all() and (ew.g13.float() > 0).all() and torch.isfinite(ew.g2.float()).all())
    if ew.fmt == 'nvfp4':
        s = torch.cat([ew.s13.flatten(), ew.s2.flatten()])
        ok = ok and not bool(((s & 0x7F) == 0x7F).any())
    return ok
