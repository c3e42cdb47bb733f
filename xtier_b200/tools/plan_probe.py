"""Measure the planner's cost coefficients on this machine (CPU engine, and the GPU kernels when a GPU is present).

    python -m xtier_b200.tools.plan_probe --hidden 2048 --inter 768 [--fmt nvfp4] [--threads N] --out probe.json
(reference parity: tools/plan_probe.py)"""
import argparse
import json

from ..planner.probe import measure


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--hidden', type=int, required=True)
    ap.add_argument('--inter', type=int, required=True)
    ap.add_argument('--fmt', default='nvfp4')
    ap.add_argument('--threads', type=int, default=None)
    ap.add_argument('--no-gpu', action='store_true')
    ap.add_argument('--out', required=True)
    a = ap.parse_args(argv)
    res = measure(a.hidden, a.inter, a.fmt, a.threads, gpu=not a.no_gpu)
    with open(a.out, 'w') as f:
        json.dump(res, f, indent=1)
    print(json.dumps(res['coeffs']))


if __name__ == '__main__':
    main()
