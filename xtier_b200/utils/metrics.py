"""Serving metrics: one snapshot of the tiered model's counters, as a dict or in the Prometheus text format.

Counters: requests and generated tokens (the server's), mailbox calls / mean CPU time per call / error counts, and per
MoE layer the routes served by the GPU slots and by the CPU tier (the hit rate), the CPU microseconds per call, the
adaptive policy's swap total, the cold store's bytes read and the elastic cache's extra slots.
(Reference parity: the periodic `XTier cache:` lines of csrc/mailbox/mailbox.cpp:597-621 -- hit rate, CPU us per layer
call, swaps -- and the cold-store reporter of xtier/cache/cold.py:600.)
"""
from __future__ import annotations


def snapshot(model=None, mailbox=None, state: dict | None = None) -> dict:
    out: dict = {}
    if state:
        out['requests_total'] = state.get('requests', 0)
        out['tokens_total'] = state.get('tokens', 0)
    if mailbox is not None:
        st = mailbox.stats()
        out['mailbox_calls_total'] = st['calls']
        out['mailbox_cpu_us_mean'] = st['mean_us']
        out['mailbox_errors_total'] = st['cpu_error'] + st['gpu_error']
        layers = []
        for L in getattr(model, 'layers', []) or []:
            moe = L.get('moe') if isinstance(L, dict) else None
            if moe is None or getattr(moe, 'mailbox', None) is None:
                continue
            E = getattr(moe, 'E', None) or moe.comm.E     # TieredMoE, or EPMoE (experts of the exchange)
            try:
                _, ls = mailbox.layer_stats(moe.layer, E)
            except KeyError:
                continue
            routes = ls['cpu_routes'] + ls['gpu_routes']
            layers.append(dict(layer=moe.layer, gpu_routes=ls['gpu_routes'], cpu_routes=ls['cpu_routes'],
                               hit_rate=(ls['gpu_routes'] / routes) if routes else None,
                               cpu_us_per_call=(ls['cpu_us'] / ls['calls']) if ls['calls'] else None))
        out['layers'] = layers
    pol = getattr(model, 'policy', None)
    if pol is not None:
        out['swaps_total'] = pol.total_swaps
    cold = getattr(model, 'cold', None)
    if cold is not None:
        out['cold_bytes_read_total'] = cold.stats()['bytes_read']
    gov = getattr(model, 'governor', None)
    if gov is not None:
        out['elastic_extra_slots'] = gov.extra
    return out


def prometheus_text(snap: dict, prefix: str = 'xtier') -> str:
    """The snapshot in the Prometheus exposition format (counters and gauges; per-layer series labelled)."""
    lines = []
    kinds = dict(requests_total='counter', tokens_total='counter', mailbox_calls_total='counter',
                 mailbox_errors_total='counter', swaps_total='counter', cold_bytes_read_total='counter',
                 mailbox_cpu_us_mean='gauge', elastic_extra_slots='gauge')
    for k, kind in kinds.items():
        if k in snap and snap[k] is not None:
            lines.append(f'# TYPE {prefix}_{k} {kind}')
            lines.append(f'{prefix}_{k} {float(snap[k]):g}')
    per = snap.get('layers') or []
    for name, kind in (('gpu_routes', 'counter'), ('cpu_routes', 'counter'), ('hit_rate', 'gauge'),
                       ('cpu_us_per_call', 'gauge')):
        rows = [(r['layer'], r[name]) for r in per if r.get(name) is not None]
        if rows:
            lines.append(f'# TYPE {prefix}_layer_{name} {kind}')
            lines += [f'{prefix}_layer_{name}{{layer="{l}"}} {float(v):g}' for l, v in rows]
    return '\n'.join(lines) + '\n'
