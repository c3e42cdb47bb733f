"""Per-layer hot-slot planning: which layers get how many GPU slots (reference parity: xtier/planner/__init__.py).

`layer_slots(layer, experts)` answers for one layer from, in order: XTIER_LAYERS (untouched layers keep every expert on
the GPU), XTIER_CACHE_FULL, the plan file of XTIER_CACHE_PLAN (or a plan computed from the profile and probe when it is
"auto"), XTIER_CACHE_FRACTION, XTIER_CACHE_SLOTS.
"""
from __future__ import annotations

import json

from .. import config

_plan_cache: dict = {}


def cache_plan(layers: int = 0, experts: int = 0, bytes_per_expert: int = 0) -> dict[int, int]:
    spec = config.get('XTIER_CACHE_PLAN')
    if not spec:
        return {}
    if spec in _plan_cache:
        return _plan_cache[spec]
    if spec == 'auto':
        from .auto import from_env
        plan = from_env(layers, experts, bytes_per_expert) or {}
    else:
        with open(spec) as f:
            plan = {int(k): int(v) for k, v in json.load(f)['slots'].items()}
    _plan_cache[spec] = plan
    return plan


def layer_slots(layer: int, experts: int, layers: int = 0, bytes_per_expert: int = 0) -> int:
    if not config.get('XTIER') or not config.layer_selected(layer):
        return experts
    if layer in config.get('XTIER_CACHE_FULL'):
        return experts
    plan = cache_plan(layers, experts, bytes_per_expert)
    if layer in plan:
        return min(experts, plan[layer])
    frac = config.get('XTIER_CACHE_FRACTION')
    if frac > 0:
        return max(1, min(experts, int(round(frac * experts))))
    slots = config.get('XTIER_CACHE_SLOTS')
    return experts if slots < 0 else min(experts, slots)


def configured() -> bool:
    """Whether any of the per-layer slot switches is set (then they, not a model's single hot fraction, decide)."""
    return bool(config.get('XTIER_CACHE_PLAN') or config.get('XTIER_CACHE_FRACTION') > 0
                or config.get('XTIER_CACHE_SLOTS') >= 0 or config.get('XTIER_CACHE_FULL')
                or str(config.get('XTIER_LAYERS')).strip() not in ('', 'all'))


def profile_popularity(path, layers: int, experts: int):
    """[layers, experts] route probabilities of a route profile ({"layers": {layer: [p_e]}}, tools/plan_trace.py);
    layers it does not cover are zero (id order decides there)."""
    import torch
    with open(path) as f:
        prof = json.load(f)
    out = torch.zeros(layers, experts)
    for k, v in prof.get('layers', {}).items():
        if int(k) < layers:
            row = torch.tensor(v[:experts], dtype=torch.float32)
            out[int(k), :row.numel()] = row
    return out

