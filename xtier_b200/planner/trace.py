"""Route traces and route profiles.

A route trace (XTIER_ROUTE_TRACE=file, written by the mailbox dispatcher) is a sequence of records: a 32-byte head
{double t_us, double wall_us, int32 layer, int32 m, int32 k, int32 groups} followed by m * k int32 expert ids as routed
(GPU-served routes included, -1 for shared experts). A route profile is the planner's input:
{"tokens": {layer: n}, "layers": {layer: [p_e]}} with p_e the probability that a token routes to expert e.

Reference parity: csrc/mailbox/mailbox.cpp:33-50 (TraceHead), tools/plan_trace.py (profile).
"""
from __future__ import annotations

import json
import struct

import numpy as np

HEAD = struct.Struct('<ddiiii')


def read_trace(path):
    """Yields (t_us, wall_us, layer, m, k, groups, ids[m, k])."""
    with open(path, 'rb') as f:
        data = f.read()
    off = 0
    while off + HEAD.size <= len(data):
        t, wall, layer, m, k, groups = HEAD.unpack_from(data, off)
        off += HEAD.size
        n = m * k
        ids = np.frombuffer(data, dtype=np.int32, count=n, offset=off).reshape(m, k)
        off += 4 * n
        yield t, wall, layer, m, k, groups, ids


def write_trace(path, records):
    """records: iterable of (t_us, wall_us, layer, groups, ids[m, k]) (tests, synthetic traces)."""
    with open(path, 'wb') as f:
        for t, wall, layer, groups, ids in records:
            ids = np.ascontiguousarray(ids, dtype=np.int32)
            f.write(HEAD.pack(t, wall, layer, ids.shape[0], ids.shape[1], groups))
            f.write(ids.tobytes())


def profile_from_counts(counts: dict[int, np.ndarray], tokens: dict[int, float]) -> dict:
    return {'tokens': {str(l): float(tokens[l]) for l in counts},
            'layers': {str(l): (np.asarray(c, dtype=np.float64) / max(tokens[l], 1.0)).tolist()
                       for l, c in counts.items()}}


def profile_from_trace(path, experts: int) -> dict:
    counts: dict[int, np.ndarray] = {}
    tokens: dict[int, float] = {}
    for _, _, layer, m, _, _, ids in read_trace(path):
        c = counts.setdefault(layer, np.zeros(experts))
        v = ids[ids >= 0]
        np.add.at(c, v[v < experts], 1.0)
        tokens[layer] = tokens.get(layer, 0.0) + m
    return profile_from_counts(counts, tokens)


def save(obj, path):
    with open(path, 'w') as f:
        json.dump(obj, f)
