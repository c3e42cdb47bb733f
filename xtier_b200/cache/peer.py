"""Hot-expert slots spread over the GPUs of a node: every rank's slot pool lives in symmetric peer memory, and a route
to an expert that another GPU holds is computed from that GPU's slot over NVLink (plain 16-byte loads from the mapped
peer pool inside the decode expert kernels), instead of going to the CPU tier.

Placement (`plan_sets`, the same on every rank): experts in popularity order; the most popular X are replicated on
every GPU (local reads for the bulk of the routes), the next (budget - X) * W are dealt round robin, one share per GPU.
X is the largest count that still covers every expert when the node's slots can (budget * W >= E), and at least half
the budget. With W = 1 this is the plain hot set.

Slot names in peer mode: global slot = rank * spr + local slot (spr: slots per rank, the same on every rank); the
decode kernels split it with the per-layer table of every rank's pool base addresses. Prefill keeps local names
(`TieredMoE.table_local`): the grouped GEMM reads only this GPU's pool, other experts come from the host staging copy.

(Reference parity: xtier/cache/second.py:1-16 and XTIER_GPU2_SLOTS -- a second GPU's expert pool reached through host
memory; here every GPU's pool is reached directly over NVLink.)
"""
from __future__ import annotations

import numpy as np
import torch

FIELDS = ('w13', 's13', 'g13', 'w2', 's2', 'g2')   # order of the kernels' peer table entries


def plan_sets(E: int, budget: int, world: int, popularity) -> list[list[int]]:
    """Hot set of every rank (each `budget` experts, most popular first)."""
    order = [int(e) for e in np.argsort(-np.asarray(popularity, dtype=np.float64), kind='stable')]
    budget = min(budget, E)
    if world <= 1:
        return [order[:budget]]
    X = (budget * world - E) // (world - 1) if budget * world >= E else 0
    X = max(min(budget, X), budget // 2)
    rep, rest = order[:X], order[X:]
    per = budget - X
    dealt = rest[:per * world]
    sets = [rep + dealt[r::world][:per] for r in range(world)]
    for hot in sets:   # a short deal (fewer experts than slots): fill with the most popular ones this GPU lacks
        have = set(hot)
        for e in order:
            if len(hot) >= budget:
                break
            if e not in have:
                hot.append(e)
                have.add(e)
    return sets


def owners(sets: list[list[int]], rank: int) -> dict[int, tuple[int, int]]:
    """expert -> (rank, local slot) of the copy this rank reads: its own when it has one, else the first peer's."""
    out = {e: (rank, s) for s, e in enumerate(sets[rank])}
    for r, hot in enumerate(sets):
        for s, e in enumerate(hot):
            out.setdefault(e, (r, s))
    return out


class PeerPools:
    """One symmetric device buffer with every layer's slot pool (the same layout on every rank)."""

    def __init__(self, shapes: list[tuple[int, int, int, int]], device):
        """shapes: per layer (slots, hidden, inter, block size)."""
        from ..parallel.symm import SymmetricBuffer
        self.layouts = []
        off = 0
        for S, H, I, bs in shapes:
            sizes = dict(w13=S * 2 * I * H // 2, s13=S * 2 * I * H // bs, g13=S * 2 * 4, w2=S * H * I // 2,
                         s2=S * H * I // bs, g2=S * 4)
            lay = {}
            for f in FIELDS:
                lay[f] = off
                off += (sizes[f] + 255) // 256 * 256
            self.layouts.append((S, H, I, bs, lay))
        self.buf = SymmetricBuffer(max(off, 256), device)
        self.device = self.buf.device
        from .elastic import _CudaArray
        self.all = torch.as_tensor(_CudaArray(self.buf.base, self.buf.nbytes, self.buf), device=self.device)

    def storage(self, layer: int) -> dict:
        """Views of this rank's pool of `layer`: w13 [S, 2I, H/2], s13 [S, 2I, H/bs], g13 [S, 2] fp32, w2 [S, H, I/2],
        s2 [S, H, I/bs], g2 [S] fp32."""
        S, H, I, bs, lay = self.layouts[layer]
        shp = dict(w13=(S, 2 * I, H // 2), s13=(S, 2 * I, H // bs), g13=(S, 2), w2=(S, H, I // 2), s2=(S, H, I // bs),
                   g2=(S,))
        out = {}
        for f in FIELDS:
            n = int(np.prod(shp[f])) * (4 if f in ('g13', 'g2') else 1)
            t = self.all[lay[f]:lay[f] + n]
            out[f] = (t.view(torch.float32) if f in ('g13', 'g2') else t).view(*shp[f])
        return out

    def table(self, layer: int) -> torch.Tensor:
        """int64 [W * 6]: rank r's base address of each field (FIELDS order) for the decode kernels."""
        lay = self.layouts[layer][4]
        vals = [p + lay[f] for p in self.buf.ptrs for f in FIELDS]
        return torch.tensor(vals, dtype=torch.int64, device=self.device)

    def close(self):
        self.buf.close()
