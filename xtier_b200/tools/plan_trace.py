"""Route trace (XTIER_ROUTE_TRACE) -> route profile for the planner.

    python -m xtier_b200.tools.plan_trace TRACE --experts 128 --out profile.json   (reference parity: tools/plan_trace.py)"""
import argparse
import json

from ..planner.trace import profile_from_trace


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('trace')
    ap.add_argument('--experts', type=int, required=True)
    ap.add_argument('--out', required=True)
    a = ap.parse_args(argv)
    prof = profile_from_trace(a.trace, a.experts)
    with open(a.out, 'w') as f:
        json.dump(prof, f)
    print(f'{len(prof["layers"])} layers, tokens per layer: {sorted(set(prof["tokens"].values()))[:4]}')


if __name__ == '__main__':
    main()
