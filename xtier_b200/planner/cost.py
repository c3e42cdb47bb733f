"""Decode cost model of one tiered MoE layer, used by the slot planner.

For a layer whose experts have per-token route probabilities p_e (from a route profile), keeping the n most routed
experts on the GPU gives, per decode call of m tokens:

  GPU part  t_gpu(n) = g0 + g1 * E[# distinct hot experts touched]           (weight streaming of the hot routes)
  CPU part  t_cpu(n) = P(any cold route) * (c0 + c1 * E[# distinct cold experts touched])   (mailbox round trip +
                                                                                  engine time per cold expert)
  layer     t(n)     = max(t_gpu(n), t_cpu(n)) + a                            (both halves run at the same time)

With a node-wide slot pool (peer mode), a cold expert that another GPU's pool holds is read over NVLink by the GPU
kernels instead of going to the CPU: it adds p1 per expert touched to the GPU part and leaves the CPU part.

With PCIe staging (`stage` slots), up to `stage` of the touched cold experts are copied from the engine's host memory
by the GPU instead of computed by the engine: h1 per staged expert moves to the GPU part (the copy runs before the
expert kernels), the CPU part keeps the rest. The staging share that balances both is c1 / (c1 + h1) of the touched
cold experts (`staging_share`).

The expected distinct-expert counts treat the m * k routes of a call as independent draws (an expert is touched with
probability 1 - (1 - p_e)^m, p_e the per-token probability of being among the token's k routes). The max of two
random times is approximated by the max of their means plus a spread term (Clark's formula for the expected maximum
of two normals, C. E. Clark, "The greatest of a finite set of random variables", Operations Research 9(2), 1961),
which matters when both halves are close.

Reference parity: xtier/planner/cost.py:1-22 (model), :43-74 (fit), :85 (expected max); the formulation here (route
probabilities, distinct-expert expectations) is this project's own.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np


@dataclasses.dataclass
class Coeffs:
    g0: float = 8.0       # us: GPU fixed cost of a call (route + two expert kernels)
    g1: float = 0.45      # us per hot expert touched (weight streaming)
    c0: float = 12.0      # us: mailbox round trip when the CPU has work
    c1: float = 25.0      # us per cold expert touched (CPU engine)
    p1: float = 0.0       # us per expert touched that another GPU's pool holds (NVLink read)
    h1: float = 0.0       # us per cold expert the GPU copies from host memory (PCIe staging)
    stage: int = 0        # PCIe staging slots per call (0: off)
    a: float = 0.0        # us: per-layer work outside the MoE (attention), added to every option
    sd_frac: float = 0.15  # relative spread of both halves (for the expected max)

    def to_dict(self):
        return dataclasses.asdict(self)


def expected_max(m1: float, s1: float, m2: float, s2: float) -> float:
    """E[max(X1, X2)] of independent normals (Clark 1961)."""
    th = math.sqrt(s1 * s1 + s2 * s2)
    if th < 1e-12:
        return max(m1, m2)
    al = (m1 - m2) / th
    phi = math.exp(-0.5 * al * al) / math.sqrt(2 * math.pi)
    Phi = 0.5 * (1 + math.erf(al / math.sqrt(2)))
    return m1 * Phi + m2 * (1 - Phi) + th * phi


def touch_probabilities(p: np.ndarray, m: int) -> np.ndarray:
    """Probability that each expert is touched by a call of m tokens, given per-token route probabilities p."""
    p = np.clip(np.asarray(p, dtype=np.float64), 0.0, 1.0)
    return 1.0 - np.power(1.0 - p, m)


def layer_time_curve(p: np.ndarray, c: Coeffs, m: int = 1, peer_held: np.ndarray | None = None) -> np.ndarray:
    """t(n) for n = 0..E hot slots (the n most routed experts on the GPU), microseconds per call. peer_held: bool [E]
    (expert order of p), experts another GPU's pool holds: when not hot here they cost p1 on the GPU side."""
    order = np.argsort(-np.asarray(p))
    q = touch_probabilities(np.asarray(p)[order], m)
    E = len(q)
    peer = (np.zeros(E, dtype=bool) if peer_held is None else np.asarray(peer_held, dtype=bool)[order])
    out = np.empty(E + 1)
    cum_hot = np.concatenate([[0.0], np.cumsum(q)])
    # touched experts past the n hottest: the peer-held ones (NVLink) and the rest (CPU)
    cum_peer_tail = np.concatenate([np.cumsum((q * peer)[::-1])[::-1], [0.0]])
    cum_cpu_tail = np.concatenate([np.cumsum((q * ~peer)[::-1])[::-1], [0.0]])
    log_none = np.concatenate([np.cumsum(np.log1p(-np.minimum(q * ~peer, 1 - 1e-12))[::-1])[::-1], [0.0]])
    for n in range(E + 1):
        hot = cum_hot[n]
        on_peer = cum_peer_tail[n]
        cold = cum_cpu_tail[n]
        p_any_cold = 1.0 - math.exp(log_none[n])
        staged = min(float(c.stage), cold) if c.h1 > 0 else 0.0
        tg = c.g0 + c.g1 * (hot + staged) + c.p1 * on_peer + c.h1 * staged
        tc = p_any_cold * c.c0 + c.c1 * (cold - staged)
        out[n] = expected_max(tg, c.sd_frac * tg, tc, c.sd_frac * tc) + c.a
    return out


def staging_share(c: Coeffs) -> float:
    """Share of the touched cold experts to stage over PCIe so that the engine and the copy finish together."""
    return c.c1 / (c.c1 + c.h1) if c.h1 > 0 else 0.0


def fit(samples: list[tuple[float, float]]) -> tuple[float, float]:
    """Least-squares line y = b0 + b1 x through (x, y) samples (probe timings)."""
    x = np.array([s[0] for s in samples], dtype=np.float64)
    y = np.array([s[1] for s in samples], dtype=np.float64)
    A = np.stack([np.ones_like(x), x], 1)
    b, *_ = np.linalg.lstsq(A, y, rcond=None)
    return float(b[0]), float(b[1])
