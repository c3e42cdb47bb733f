"""Planner on the CPU: Clark's expected max vs Monte Carlo, the DP stays within budget and beats or matches the
uniform layout, route traces round-trip into profiles, and the CLI tools chain (trace -> profile -> plan)."""
import json
import subprocess
import sys
from pathlib import Path

import numpy as np

from xtier_b200.planner import auto, cost, trace

ROOT = Path(__file__).resolve().parent.parent


def test_expected_max_vs_monte_carlo():
    rng = np.random.default_rng(0)
    for m1, s1, m2, s2 in [(10, 1, 10, 1), (10, 2, 12, 1), (5, 0.5, 20, 3)]:
        mc = np.maximum(rng.normal(m1, s1, 400000), rng.normal(m2, s2, 400000)).mean()
        assert abs(cost.expected_max(m1, s1, m2, s2) - mc) < 0.02 * mc


def _profile(L=6, E=32, seed=0):
    rng = np.random.default_rng(seed)
    layers = {}
    for l in range(L):
        z = (np.arange(1, E + 1) ** -(0.6 + 0.15 * l))
        z = rng.permutation(z / z.sum() * 8)   # 8 routes per token
        layers[str(l)] = np.minimum(z, 1.0).tolist()
    return {'layers': layers, 'tokens': {str(l): 1000 for l in range(L)}}


def test_dp_within_budget_and_not_worse_than_uniform():
    prof = _profile()
    curves = auto.curves_from_profile(prof, cost.Coeffs())
    for budget in (0, 10, 40, 96, 300):
        for g in (1, 4):
            plan = auto.solve(curves, budget, g)
            assert sum(plan) <= budget
            assert all(0 <= n <= 32 for n in plan)
            assert auto.plan_time(curves, plan) <= auto.plan_time(curves, auto.uniform(curves, budget)) + 1e-9
    # exhaustive check on a tiny case
    small = [c[:5] for c in curves[:3]]
    import itertools
    best = min((sum(c[n] for c, n in zip(small, ns)), ns) for ns in itertools.product(range(5), repeat=3)
               if sum(ns) <= 6)
    plan = auto.solve(small, 6)
    assert abs(auto.plan_time(small, plan) - best[0]) < 1e-9


def test_curve_monotone_in_slots():
    c = cost.layer_time_curve(np.array(_profile()['layers']['0']), cost.Coeffs(g1=0.0))
    assert np.all(np.diff(c) <= 1e-9)   # more hot slots never costs more when GPU experts are free


def test_trace_roundtrip_and_tools(tmp_path):
    rng = np.random.default_rng(1)
    recs = [(float(i), 10.0, i % 3, 0, rng.integers(0, 16, size=(2, 4))) for i in range(60)]
    p = tmp_path / 'trace.bin'
    trace.write_trace(p, recs)
    got = list(trace.read_trace(p))
    assert len(got) == 60 and np.array_equal(got[5][6], recs[5][4])
    prof = trace.profile_from_trace(p, 16)
    assert abs(sum(prof['layers']['0']) - 4.0) < 1e-9   # 4 routes per token
    env = dict(PYTHONPATH=str(ROOT))
    subprocess.run([sys.executable, '-m', 'xtier_b200.tools.plan_trace', str(p), '--experts', '16', '--out',
                    str(tmp_path / 'prof.json')], check=True, env=env, capture_output=True)
    subprocess.run([sys.executable, '-m', 'xtier_b200.tools.plan_auto', '--profile', str(tmp_path / 'prof.json'),
                    '--budget-slots', '20', '--write', str(tmp_path / 'plan.json')], check=True, env=env,
                   capture_output=True)
    plan = json.loads((tmp_path / 'plan.json').read_text())
    assert sum(plan['slots'].values()) <= 20 and set(plan['slots']) == {'0', '1', '2'}


def test_layer_slots_from_env(monkeypatch, tmp_path):
    from xtier_b200 import planner
    planner._plan_cache.clear()
    monkeypatch.setenv('XTIER_CACHE_SLOTS', '10')
    assert planner.layer_slots(3, 64) == 10
    monkeypatch.setenv('XTIER_CACHE_FRACTION', '0.25')
    assert planner.layer_slots(3, 64) == 16
    (tmp_path / 'p.json').write_text(json.dumps({'slots': {'3': 7}}))
    monkeypatch.setenv('XTIER_CACHE_PLAN', str(tmp_path / 'p.json'))
    assert planner.layer_slots(3, 64) == 7 and planner.layer_slots(4, 64) == 16
    monkeypatch.setenv('XTIER_CACHE_FULL', '4')
    assert planner.layer_slots(4, 64) == 64
    planner._plan_cache.clear()


def test_model_takes_per_layer_slots_and_the_route_profile(tmp_path, monkeypatch):
    """A slot plan gives each layer its own hot count; a route profile picks which experts are hot."""
    import json
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    plan = tmp_path / 'plan.json'
    plan.write_text(json.dumps({'slots': {'0': 3, '1': 8}}))
    prof = tmp_path / 'profile.json'
    p0 = [0.01, 0.3, 0.02, 0.25, 0.05, 0.2, 0.1, 0.07]
    prof.write_text(json.dumps({'tokens': {'0': 100}, 'layers': {'0': p0}}))
    monkeypatch.setenv('XTIER_CACHE_PLAN', str(plan))
    monkeypatch.setenv('XTIER_CACHE_PROFILE', str(prof))
    monkeypatch.setenv('XTIER_GPU2_SLOTS', 'off')
    from xtier_b200 import planner
    planner._plan_cache.clear()
    cfg = Qwen3MoeConfig.tiny(layers=2, experts=8)
    model = Qwen3MoeModel(cfg, device='cpu', seed=0, hot_fraction=0.5, engine_threads=2, synthetic_experts=False)
    l0, l1 = model.layers[0]['moe'], model.layers[1]['moe']
    assert l0.hot == [1, 3, 5] and l1.all_hot                 # the profile's three most routed experts
    assert len(model.engines) == 1
    for e in model.engines:
        e.close()


def test_cost_curve_peer_term():
    """Experts another GPU holds cost p1 on the GPU side instead of the CPU round trip: with a cheap NVLink term the
    curve drops where those experts would otherwise be cold, and is unchanged when every expert is hot here."""
    import numpy as np
    from xtier_b200.planner.cost import Coeffs, layer_time_curve
    p = np.linspace(0.3, 0.01, 16)
    c = Coeffs(g0=8.0, g1=0.5, c0=12.0, c1=25.0, p1=1.5)
    base = layer_time_curve(p, c, m=4)
    held = np.zeros(16, dtype=bool)
    held[8:] = True                                    # the 8 least routed experts live in a peer's pool
    peer = layer_time_curve(p, c, m=4, peer_held=held)
    assert peer[16] == base[16]
    assert np.all(peer[:8] < base[:8])
    assert abs(peer[8] - (c.g0 + c.g1 * (1 - (1 - p[:8]) ** 4).sum() + c.p1 * (1 - (1 - p[8:]) ** 4).sum())) < 1e-6


def test_cost_curve_pcie_staging_term():
    """PCIe staging moves up to `stage` touched cold experts from the engine (c1 each) to the GPU (h1 + g1 each): the
    curve drops while the engine is the slower half, not at all when every expert is hot, and the balancing share is
    c1 / (c1 + h1)."""
    import numpy as np
    from xtier_b200.planner.cost import Coeffs, layer_time_curve, staging_share, touch_probabilities
    p = np.full(64, 8 / 64)
    c = Coeffs(g0=20.0, g1=5.0, c0=30.0, c1=300.0, h1=500.0, stage=0, sd_frac=0.0)
    base = layer_time_curve(p, c, m=32)
    c.stage = 12
    staged = layer_time_curve(p, c, m=32)
    assert staged[64] == base[64] and np.all(staged[:40] < base[:40])
    q = touch_probabilities(p, 32)
    n = 10                                             # 10 hot experts, the other 54 cold
    cold = q[n:].sum()
    tg = c.g0 + c.g1 * (q[:n].sum() + 12) + c.h1 * 12
    tc = (1 - np.prod(1 - q[n:])) * c.c0 + c.c1 * (cold - 12)
    assert abs(staged[n] - max(tg, tc)) < 1e-6
    assert abs(staging_share(c) - 300 / 800) < 1e-12 and staging_share(Coeffs()) == 0.0
