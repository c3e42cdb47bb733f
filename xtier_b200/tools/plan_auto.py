"""Route profile + probe coefficients + GPU budget -> per-layer slot plan ({"slots": {layer: n}}, XTIER_CACHE_PLAN).

    python -m xtier_b200.tools.plan_auto --profile profile.json [--probe probe.json]
        (--budget-slots N | --budget-gib G --expert-bytes B) [--granularity 4] --write plan.json
(reference parity: tools/plan_auto.py)"""
import argparse
import json

from ..planner.auto import make_plan


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--profile', required=True)
    ap.add_argument('--probe', default=None)
    ap.add_argument('--budget-slots', type=int, default=0)
    ap.add_argument('--budget-gib', type=float, default=0.0)
    ap.add_argument('--expert-bytes', type=int, default=0)
    ap.add_argument('--granularity', type=int, default=1)
    ap.add_argument('--write', required=True)
    a = ap.parse_args(argv)
    with open(a.profile) as f:
        prof = json.load(f)
    probe = None
    if a.probe:
        with open(a.probe) as f:
            probe = json.load(f)
    slots = a.budget_slots or int(a.budget_gib * (1 << 30) // max(1, a.expert_bytes))
    plan = make_plan(prof, probe, slots, a.granularity)
    with open(a.write, 'w') as f:
        json.dump(plan, f, indent=1)
    print(f'predicted {plan["predicted_us"]:.1f} us/token-step vs uniform {plan["uniform_us"]:.1f} us '
          f'({sum(plan["slots"].values())} of {slots} slots)')


if __name__ == '__main__':
    main()
