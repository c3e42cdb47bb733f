"""Slot planner: how many GPU hot slots each layer gets under one memory budget.

Minimizes the decode time summed over layers, sum_l t_l(n_l), subject to sum_l n_l * bytes_per_expert <= budget, with
an optional upload-cost term lambda * sum_l n_l (a plan that fills more slots costs more to (re)load). The objective
is separable, so an exact dynamic program over (layer, slots used) solves it; slot counts are searched in steps of
`granularity` to bound the table. `best()` sweeps lambda and `guard()` keeps a uniform layout unless the plan gains at
least `min_gain`.

Reference parity: xtier/planner/auto.py:29-63 (DP), :74 (lambda sweep), :113 (guard), :124 (from_env).
"""
from __future__ import annotations

import json

import numpy as np

from .. import config
from .cost import Coeffs, layer_time_curve


def solve(curves: list[np.ndarray], budget_slots: int, granularity: int = 1, lam: float = 0.0) -> list[int]:
    """curves[l][n]: time of layer l with n hot slots. Returns n_l minimizing sum t_l(n_l) + lam * n_l with
    sum n_l <= budget_slots."""
    L = len(curves)
    g = max(1, granularity)
    B = budget_slots // g
    INF = float('inf')
    best = np.full(B + 1, INF)
    best[0] = 0.0
    choice = np.zeros((L, B + 1), dtype=np.int32)
    for li, cur in enumerate(curves):
        E = len(cur) - 1
        opts = list(range(0, E // g + 1))
        if E % g:
            opts.append(-1)   # every expert (E not a multiple of g)
        nxt = np.full(B + 1, INF)
        for used in range(B + 1):
            if best[used] == INF:
                continue
            for o in opts:
                n = E if o < 0 else o * g
                w = (n + g - 1) // g
                if used + w > B:
                    continue
                v = best[used] + cur[n] + lam * n
                if v < nxt[used + w]:
                    nxt[used + w] = v
                    choice[li, used + w] = n
        best = nxt
        # carry back-pointers: remember which `used` we came from via the chosen n
        choice[li, :] = np.where(nxt < INF, choice[li, :], -1)
    end = int(np.argmin(best))
    plan = [0] * L
    used = end
    for li in range(L - 1, -1, -1):
        n = int(choice[li, used])
        plan[li] = n
        used -= (n + g - 1) // g
    return plan


def plan_time(curves, plan) -> float:
    return float(sum(c[n] for c, n in zip(curves, plan)))


def uniform(curves, budget_slots: int) -> list[int]:
    L = len(curves)
    per = budget_slots // max(1, L)
    return [min(per, len(c) - 1) for c in curves]


def best(curves, budget_slots: int, granularity: int = 1, lams=(0.0, 0.05, 0.2, 1.0)):
    """Sweeps the upload weight; returns the plan with the lowest decode time (ties: fewer slots)."""
    out = None
    for lam in lams:
        p = solve(curves, budget_slots, granularity, lam)
        key = (plan_time(curves, p), sum(p))
        if out is None or key < out[0]:
            out = (key, p, lam)
    return out[1], out[2]


def guard(curves, plan, budget_slots: int, min_gain: float = 0.01):
    """Keeps the uniform layout unless `plan` is at least min_gain faster."""
    uni = uniform(curves, budget_slots)
    t_plan, t_uni = plan_time(curves, plan), plan_time(curves, uni)
    return (plan, t_plan, t_uni) if t_plan <= (1 - min_gain) * t_uni else (uni, t_uni, t_uni)


def curves_from_profile(profile: dict, coeffs: Coeffs, m: int = 1,
                        peer_held: dict | None = None) -> list[np.ndarray]:
    """profile: {"layers": {layer: [per-token route probability of each expert]}} (plan_trace output). peer_held:
    {layer: bool [E]} experts other GPUs' pools hold (peer mode), costed at the probe's NVLink term."""
    layers = sorted(int(k) for k in profile['layers'])
    return [layer_time_curve(np.asarray(profile['layers'][str(l)] if str(l) in profile['layers']
                                        else profile['layers'][l]), coeffs, m,
                             None if peer_held is None else peer_held.get(l)) for l in layers]


def make_plan(profile: dict, probe: dict | None, budget_slots: int, granularity: int = 1,
              peer_held: dict | None = None) -> dict:
    coeffs = Coeffs(**(probe or {}).get('coeffs', {}))
    layers = sorted(int(k) for k in profile['layers'])
    curves = curves_from_profile(profile, coeffs, peer_held=peer_held)
    plan, lam = best(curves, budget_slots, granularity)
    plan, t_plan, t_uni = guard(curves, plan, budget_slots)
    return {'slots': {str(l): int(n) for l, n in zip(layers, plan)}, 'predicted_us': t_plan, 'uniform_us': t_uni,
            'lambda': lam, 'budget_slots': budget_slots, 'coeffs': coeffs.to_dict()}


def from_env(layers: int, experts: int, bytes_per_expert: int) -> dict[int, int] | None:
    """XTIER_CACHE_PLAN=auto: plan from XTIER_PLANNER_TRACE (profile) and XTIER_PLANNER_PROBE (coefficients) under
    XTIER_CACHE_BUDGET_GIB; None when the inputs are missing."""
    prof_path, probe_path = config.get('XTIER_PLANNER_TRACE'), config.get('XTIER_PLANNER_PROBE')
    budget = config.get('XTIER_CACHE_BUDGET_GIB')
    if not prof_path or budget <= 0:
        return None
    with open(prof_path) as f:
        profile = json.load(f)
    probe = None
    if probe_path:
        with open(probe_path) as f:
            probe = json.load(f)
    slots = int(budget * (1 << 30) // bytes_per_expert)
    plan = make_plan(profile, probe, slots)
    return {int(k): v for k, v in plan['slots'].items()}
