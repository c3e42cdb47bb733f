"""Adaptive hot-slot residency: move the most routed experts of each layer onto the GPU while decoding.

The mailbox dispatcher keeps, per layer, exponentially decayed route counts of every call (GPU-served routes
included). Every `every` decode steps `AdaptivePolicy.step()` reads them and, per layer, swaps in the non-resident
experts whose count beats the coldest resident expert's by a factor `min_gain`, most valuable first, at most `swaps`
per round. A swap (TieredMoE.swap) unpublishes the victim in the residency table, copies the incoming expert's bytes
into the freed slot and publishes it, all on the compute stream between graph replays, so no replay ever reads a slot
whose copy is in flight. The route counts of a layer with no CPU routes stay empty, so such layers never swap.

Reference parity: csrc/mailbox/mailbox.cpp:144-360 (PoolManager: decayed counts, gain-ordered swap rounds, command
ring), xtier/cache/pool.py:603 (policy start). Settings: XTIER_CACHE_ADAPT, _EVERY, _SWAPS, _MIN_GAIN, _LOG.
"""
from __future__ import annotations

import logging

import numpy as np

from .. import config

logger = logging.getLogger('xtier_b200')


class AdaptivePolicy:
    def __init__(self, layers, mailbox, every: int | None = None, swaps: int | None = None,
                 min_gain: float | None = None, log_every: int | None = None):
        """layers: TieredMoE layers sharing `mailbox` (those with a CPU part)."""
        self.layers = [l for l in layers if l.mailbox is not None and l.can_refill]
        self.mailbox = mailbox
        self.every = every or config.get('XTIER_CACHE_EVERY')
        self.swaps = swaps or config.get('XTIER_CACHE_SWAPS')
        self.min_gain = min_gain or config.get('XTIER_CACHE_MIN_GAIN')
        self.log_every = log_every if log_every is not None else config.get('XTIER_CACHE_LOG')
        self.enabled = bool(config.get('XTIER_CACHE_ADAPT'))
        self.steps = 0
        self.rounds = 0
        self.total_swaps = 0

    def plan_layer(self, layer, counts: np.ndarray, budget: int) -> list[tuple[int, int | None]]:
        """(incoming, victim) pairs for one layer, best gain first; victim None: an empty elastic slot takes it."""
        resident = list(layer.resident())
        res_set = set(resident)
        cold = [e for e in np.argsort(-counts) if e not in res_set and counts[e] > 0]
        out = []
        el = getattr(layer, 'elastic', None)
        free = 0 if el is None else el.mapped - len(el.occupants())
        while cold and free > 0 and len(out) < budget:
            out.append((int(cold.pop(0)), None))
            free -= 1
        victims = sorted(resident, key=lambda e: counts[e])
        for inc, vic in zip(cold, victims):
            if len(out) >= budget:
                break
            if counts[inc] <= self.min_gain * max(counts[vic], 1e-9):
                break
            out.append((int(inc), int(vic)))
        return out

    def step(self) -> int:
        """Call between decode steps (outside graph capture). Returns the number of swaps applied."""
        if not self.enabled or not self.layers:
            return 0
        self.steps += 1
        if self.steps % self.every:
            return 0
        self.rounds += 1
        budget = self.swaps
        done = 0
        for layer in self.layers:
            if budget <= 0:
                break
            if getattr(layer, 'peer', None) is not None:   # peer mode: other GPUs read this pool, no swaps
                continue
            counts, _ = self.mailbox.layer_stats(layer.layer, layer.E)
            for inc, vic in self.plan_layer(layer, counts, budget):
                if vic is None:
                    layer.fill(inc)
                else:
                    layer.swap(inc, vic)
                done += 1
                budget -= 1
        self.total_swaps += done
        if self.log_every and self.rounds % self.log_every == 0:
            st = self.mailbox.stats()
            logger.info('xtier_b200 cache: round %d, %d swaps (total %d), mailbox calls %d, mean CPU %.1f us',
                        self.rounds, done, self.total_swaps, st['calls'], st['mean_us'])
        return done
