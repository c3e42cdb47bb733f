"""Move a cold-expert store to a new layout: other drives, other drive weights, another engine node count, or records
cut into another number of units.

    python -m xtier_b200.tools.cold_relayout --src DIR[,DIR...] --dst DIR[,DIR...] [--key K] [--dst-key K2]
        [--parts 5:5:2] [--nodes N] [--units 1|3] [--layers 0,1,...]

Every layer of the source manifest is read back expert by expert, re-sharded when --nodes differs, written into the
new layout, read back again and compared byte for byte with the source; only when every layer matches is the new
manifest kept (the checkpoint ranges are carried over). The source store is never written. This is the only way to
change the layout of a store whose checkpoint tensors were punched out.
(Reference parity: tools/cold_relayout.py -- verified relayout into a new store; the old one untouched.)
"""
from __future__ import annotations

import argparse
import json
import sys

import torch


def relayout(src_dirs, dst_dirs, key: str = 'xtier-cold', dst_key: str | None = None, parts=None,
             nodes: int | None = None, layers=None, threads: int = 4, log=print, units: int | None = None) -> dict:
    from ..cache.cold import ColdPool
    dst_key = dst_key or key
    src = ColdPool(src_dirs, key=key, threads=threads, units=1)
    if not src.manifest['layers']:
        src.close()
        raise SystemExit(f'cold_relayout: no manifest with layers for key {key!r} in {src_dirs}')
    if [str(p) for p in src.files] == [str(p) for p in ColdPool.files_for(dst_dirs, dst_key)]:
        src.close()
        raise SystemExit('cold_relayout: source and destination are the same store')
    dst = ColdPool(dst_dirs, key=dst_key, parts=parts, threads=threads, units=units)
    dst.manifest['layers'] = {}
    dst.manifest['end'] = [0] * len(dst.files)
    todo = [int(x) for x in layers] if layers else src.layers()
    report = {}
    try:
        for layer in todo:
            ent = src.entry(layer)
            ew = src.load_layer(layer)
            N = nodes or ent['shape'][3]
            dst.write_layer(layer, ew, N, ent['source'])
            back = dst.load_layer(layer)
            same = all(torch.equal(getattr(ew, f), getattr(back, f)) for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'))
            if not same or dst.check_layer(layer):
                raise SystemExit(f'cold_relayout: layer {layer} does not read back identically; new manifest dropped')
            de = dst.entry(layer)
            report[layer] = dict(units=len(de['loc']), record_bytes=de['record'])
            log(f'[xtier] cold_relayout: layer {layer} ok ({report[layer]["units"]} units)')
        ranges = src.ranges()
        if ranges:
            for layer, r in ranges.items():
                if int(layer) in report:
                    dst._save_ranges(int(layer), r['file'], r['tensors'])
    except BaseException:
        dst.manifest_path.unlink(missing_ok=True)
        raise
    finally:
        src.close()
        dst.close()
    return report


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--src', required=True, help='source drive directories, comma separated')
    ap.add_argument('--dst', required=True, help='destination drive directories, comma separated')
    ap.add_argument('--key', default='xtier-cold')
    ap.add_argument('--dst-key', default=None)
    ap.add_argument('--parts', default=None, help='destination drive weights, e.g. 5:5:2')
    ap.add_argument('--nodes', type=int, default=None, help='re-shard for an engine with this many nodes')
    ap.add_argument('--units', type=int, default=None, choices=(1, 3), help='units per record (default XTIER_COLD_UNITS)')
    ap.add_argument('--layers', default=None, help='comma separated layer ids (default: all)')
    ap.add_argument('--threads', type=int, default=4)
    a = ap.parse_args(argv)
    rep = relayout(a.src, a.dst, a.key, a.dst_key, a.parts, a.nodes,
                   a.layers.split(',') if a.layers else None, a.threads, log=lambda s: print(s, file=sys.stderr),
                   units=a.units)
    print(json.dumps({'layers': len(rep)}))


if __name__ == '__main__':
    main()
