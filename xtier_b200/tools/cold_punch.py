"""Give the checkpoint's copy of the expert tensors back to the drive once the cold store holds them (and undo it).

    python -m xtier_b200.tools.cold_punch --cold DIR[,DIR...] [--key K] --dry-run   # compare only
    python -m xtier_b200.tools.cold_punch --cold DIR[,DIR...] [--key K]             # compare, then punch
    python -m xtier_b200.tools.cold_punch --cold DIR[,DIR...] [--key K] --restore   # write the tensors back

The store's `<key>.ranges` says where every layer's expert tensors (codes and block scales) sit in the checkpoint
file they were loaded from. Punching first compares every byte of those tensors with the experts rebuilt from the
cold records and stops on any difference; then it writes the marker `XTIER-COLD-ONLY` beside the files (their size
and mtime, the layers), frees the whole 4 KiB blocks inside each tensor with fallocate(PUNCH_HOLE | KEEP_SIZE) (not a
byte outside a tensor is touched: the range is rounded inward) and restores the file's mtime. The file keeps its
size, header and other tensors; `checkpoint.load_experts` refuses a marked file, so a layer is then loaded from the
store. `--restore` writes the tensors back from the records, compares again, restores the mtime and removes the
marker (also the way to recover from a punch that stopped half way).
(Reference parity: tools/cold_punch.py, docs/design-cold-experts.md "only one copy": compare, marker, inward-aligned
punch, mtime kept, --restore.)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys
from pathlib import Path

import numpy as np

FALLOC_FL_KEEP_SIZE = 0x01
FALLOC_FL_PUNCH_HOLE = 0x02
BLOCK = 4096


def _layer_tensors(pool, layer: int) -> dict:
    ew = pool.load_layer(layer)
    return {n: getattr(ew, n).contiguous().numpy().reshape(-1).view(np.uint8) for n in ('w13', 's13', 'w2', 's2')}


def _by_file(ranges: dict) -> dict:
    out: dict = {}
    for layer, r in ranges.items():
        out.setdefault(r['file'], []).append((int(layer), r['tensors']))
    return out


def compare(pool, ranges: dict) -> list[str]:
    """Differences between the checkpoint tensors and the cold records (empty: identical)."""
    bad = []
    for path, layers in _by_file(ranges).items():
        with open(path, 'rb') as f:
            for layer, tensors in layers:
                want = _layer_tensors(pool, layer)
                for name, (off, stride) in tensors.items():
                    f.seek(off)
                    got = np.frombuffer(f.read(want[name].size), dtype=np.uint8)
                    if got.size != want[name].size or not np.array_equal(got, want[name]):
                        bad.append(f'{path}: layer {layer} {name}')
    return bad


def _punch(fd: int, off: int, n: int) -> int:
    lo = (off + BLOCK - 1) // BLOCK * BLOCK
    hi = (off + n) // BLOCK * BLOCK
    if hi <= lo:
        return 0
    libc = ctypes.CDLL(None, use_errno=True)
    libc.fallocate.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_longlong, ctypes.c_longlong]
    if libc.fallocate(fd, FALLOC_FL_PUNCH_HOLE | FALLOC_FL_KEEP_SIZE, lo, hi - lo) != 0:
        e = ctypes.get_errno()
        raise OSError(e, f'fallocate(PUNCH_HOLE): {os.strerror(e)}')
    return hi - lo


def punch(pool, ranges: dict, log=print) -> int:
    files = _by_file(ranges)
    bad = compare(pool, ranges)
    if bad:
        raise SystemExit('cold_punch: the cold store differs from the checkpoint, nothing punched:\n  ' +
                         '\n  '.join(bad))
    for path, layers in files.items():
        marker = Path(path).parent / 'XTIER-COLD-ONLY'
        m = json.loads(marker.read_text()) if marker.exists() else {'files': {}}
        st = os.stat(path)
        m['files'][Path(path).name] = dict(size=st.st_size, mtime_ns=st.st_mtime_ns, atime_ns=st.st_atime_ns,
                                           layers=sorted(l for l, _ in layers), store=pool.key)
        marker.write_text(json.dumps(m))
    freed = 0
    for path, layers in files.items():
        st = os.stat(path)
        fd = os.open(path, os.O_RDWR)
        try:
            for layer, tensors in layers:
                for off, stride in tensors.values():
                    n = stride * pool.entry(layer)['experts']
                    freed += _punch(fd, off, n)
            os.fsync(fd)
        finally:
            os.close(fd)
        os.utime(path, ns=(st.st_atime_ns, st.st_mtime_ns))
        log(f'[xtier] cold_punch: {path}: {len(layers)} layer(s) punched')
    return freed


def restore(pool, ranges: dict, log=print) -> int:
    files = _by_file(ranges)
    written = 0
    for path, layers in files.items():
        marker = Path(path).parent / 'XTIER-COLD-ONLY'
        m = json.loads(marker.read_text()) if marker.exists() else {'files': {}}
        rec = m['files'].get(Path(path).name)
        st = os.stat(path)
        if rec is not None and rec['size'] != st.st_size:
            raise SystemExit(f'cold_punch: {path} changed size since it was punched; not restoring')
        fd = os.open(path, os.O_RDWR)
        try:
            for layer, tensors in layers:
                want = _layer_tensors(pool, layer)
                for name, (off, _) in tensors.items():
                    os.pwrite(fd, want[name].tobytes(), off)
                    written += want[name].size
            os.fsync(fd)
        finally:
            os.close(fd)
        t = (rec['atime_ns'], rec['mtime_ns']) if rec else (st.st_atime_ns, st.st_mtime_ns)
        os.utime(path, ns=t)
        if rec is not None:
            del m['files'][Path(path).name]
            if m['files']:
                marker.write_text(json.dumps(m))
            else:
                marker.unlink()
        log(f'[xtier] cold_punch: {path}: restored')
    sub = {k: v for k, v in ranges.items()}
    bad = compare(pool, sub)
    if bad:
        raise SystemExit('cold_punch: restored tensors do not match the cold store:\n  ' + '\n  '.join(bad))
    return written


def main(argv=None):
    from ..cache.cold import ColdPool
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--cold', required=True, help='cold store drive directories, comma separated')
    ap.add_argument('--key', default='xtier-cold')
    g = ap.add_mutually_exclusive_group()
    g.add_argument('--dry-run', action='store_true')
    g.add_argument('--restore', action='store_true')
    a = ap.parse_args(argv)
    pool = ColdPool(a.cold, key=a.key)
    try:
        ranges = pool.ranges()
        if not ranges:
            raise SystemExit(f'cold_punch: no {a.key}.ranges beside the manifest (layers never loaded from a checkpoint)')
        log = lambda s: print(s, file=sys.stderr)
        if a.dry_run:
            bad = compare(pool, ranges)
            print(json.dumps({'identical': not bad, 'differences': bad}))
            return 1 if bad else 0
        if a.restore:
            print(json.dumps({'restored_bytes': restore(pool, ranges, log)}))
        else:
            print(json.dumps({'punched_bytes': punch(pool, ranges, log)}))
        return 0
    finally:
        pool.close()


if __name__ == '__main__':
    sys.exit(main())
