"""Fit the CPU coefficients of the cost model from measured mailbox statistics (per-layer calls, CPU microseconds and
cold routes, e.g. a json dump of Mailbox.layer_stats over a run) and update a probe file.

    python -m xtier_b200.tools.plan_calibrate --stats stats.json --probe probe.json   (reference parity:
    tools/plan_calibrate.py)"""
import argparse
import json

from ..planner.cost import fit


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--stats', required=True, help='{"layers": {layer: {"calls", "cpu_us", "cpu_routes"}}}')
    ap.add_argument('--probe', required=True)
    a = ap.parse_args(argv)
    with open(a.stats) as f:
        st = json.load(f)
    pts = [(v['cpu_routes'] / v['calls'], v['cpu_us'] / v['calls']) for v in st['layers'].values() if v['calls']]
    c0, c1 = fit(pts) if len(pts) >= 2 else (pts[0][1], 0.0)
    with open(a.probe) as f:
        probe = json.load(f)
    probe.setdefault('coeffs', {})
    probe['coeffs']['c0'], probe['coeffs']['c1'] = max(c0, 1.0), max(c1, 0.1)
    with open(a.probe, 'w') as f:
        json.dump(probe, f, indent=1)
    print(json.dumps(probe['coeffs']))


if __name__ == '__main__':
    main()
