"""Elastic cache sizing on the host: need prediction (bound, extrapolation), release before an allocating forward,
growth after idle decode steps, the critical-memory release with its cool-down, the out-of-memory retry, and the
adaptive policy filling empty elastic slots before it swaps."""
import numpy as np
import pytest
import torch

from xtier_b200.cache.elastic import GIB, Governor
from xtier_b200.cache.policy import AdaptivePolicy


class FakeSlots:
    def __init__(self, cap, row):
        self.cap, self.row, self.mapped = cap, row, 0
        self.log = []

    def slot_bytes(self):
        return self.row

    def grow(self, n):
        self.mapped = max(self.mapped, min(n, self.cap))
        self.log.append(('grow', n))

    def release(self, n):
        self.mapped = min(self.mapped, n)
        self.log.append(('release', n))


class Mem:
    def __init__(self, free):
        self.free = free

    def __call__(self):
        return self.free, 180 * GIB


class Clock:
    t = 0.0

    def __call__(self):
        return self.t


def _gov(free_gib, cap=8, **kw):
    layers = [FakeSlots(cap, GIB // 4) for _ in range(4)]        # one level = 4 x 0.25 GiB = 1 GiB
    mem, clk = Mem(free_gib * GIB), Clock()
    g = Governor(layers, mem_info=mem, reserve_gib=2.0, critical_gib=1.0, margin=1.25, idle=3, every=2,
                 cooldown_s=100.0, extrapolate=2.0, step=4, clock=clk, **kw)
    return g, layers, mem, clk


def test_predict_bounds_and_extrapolation():
    g, *_ = _gov(50)
    assert g.predict(1000, 1000) is None
    g.learn(2048, 2048, 4 * GIB)
    g.learn(512, 512, 1 * GIB)
    assert g.predict(2048, 2048) == 4 * GIB
    assert g.predict(500, 500) == 1 * GIB               # the tightest bound wins
    assert g.predict(1024, 512) == 2 * GIB              # 512-token need scaled 2x
    assert g.predict(4096, 2048) == 8 * GIB             # 2x the 2048 one
    assert g.predict(8192, 8192) is None                # beyond every extrapolation


def test_release_before_alloc_and_regrow_after_idle():
    g, layers, mem, _ = _gov(20)
    for _ in range(3):
        g.after_decode()
    assert g.extra == 4 and all(l.mapped == 4 for l in layers)      # grew one step (4 levels)
    mem.free = 12 * GIB
    assert g.before_alloc(100, 100) == 4                 # nothing learnt: release every level
    g.learn(100, 100, 8 * GIB)
    g._set(6, 'test')
    mem.free = 9 * GIB        # need 8 * 1.25 + 2 reserve = 12 GiB: 3 GiB short -> 3 levels
    assert g.before_alloc(100, 100) == 3 and g.extra == 3
    assert layers[0].log[-1] == ('release', 3)
    mem.free = 30 * GIB
    assert g.after_decode() == 0 and g.after_decode() == 0          # idle count restarted by the allocating forward
    assert g.after_decode() == 4 and g.extra == 7
    assert g.after_decode() == 1 and g.extra == 8                    # capped


def test_growth_leaves_room_for_the_usual_small_prefill():
    g, _, mem, _ = _gov(10)
    g.learn(1000, 1000, 5 * GIB)       # a small prefill needs 5 GiB: keep 2 + 6.25 GiB free
    for _ in range(3):
        g.after_decode()
    assert g.extra == 1                # floor((10 - 8.25) / 1)


def test_critical_release_and_cooldown():
    g, _, mem, clk = _gov(40)
    for _ in range(3):
        g.after_decode()
    assert g.extra == 4
    mem.free = GIB // 2
    assert g.after_decode() == -4 and g.extra == 0
    mem.free = 40 * GIB
    for _ in range(6):
        assert g.after_decode() == 0   # cooling down
    clk.t = 101.0
    assert g.after_decode() == 4


def test_oom_retry_releases_and_disables():
    g, _, _, _ = _gov(40)
    g._set(5, 'test')
    calls = []

    def fwd(x):
        calls.append(x)
        if len(calls) == 1:
            raise torch.cuda.OutOfMemoryError('injected')
        return x + 1

    assert g.guarded(fwd, 1) == 2 and g.extra == 0 and not g.enabled
    for _ in range(10):
        assert g.after_decode() == 0
    g2, *_ = _gov(40)
    with pytest.raises(torch.cuda.OutOfMemoryError):    # nothing held: the error is the caller's
        g2.guarded(lambda: (_ for _ in ()).throw(torch.cuda.OutOfMemoryError('x')))


def test_policy_fills_free_elastic_slots_first():
    class El:
        mapped, first = 3, 10
        occupant = [7, -1, -1]

        def occupants(self):
            return [e for e in self.occupant[:self.mapped] if e >= 0]

    class Layer:
        E, layer, mailbox, host = 16, 0, object(), object()
        elastic = El()

        def resident(self):
            return [0, 1, 2] + self.elastic.occupants()

    pol = AdaptivePolicy([], None, every=1, swaps=8, min_gain=1.5)
    counts = np.zeros(16)
    counts[[0, 1, 2, 7]] = 1.0
    counts[[9, 11, 12]] = [50.0, 40.0, 30.0]
    plan = pol.plan_layer(Layer(), counts, 8)
    assert plan[:2] == [(9, None), (11, None)]           # two empty slots: no victims
    assert plan[2][0] == 12 and plan[2][1] in (0, 1, 2, 7)
