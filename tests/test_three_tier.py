"""Three-tier runner pieces on the CPU: route profiles of DeepSeek-style routers, the planner's GPU slot layout,
popularity-ranked expert placement over EP ranks, and the streamed synthetic bigram table."""
import os

import numpy as np
import pytest
import torch

from xtier_b200.models.deepseek_v3 import DeepSeekV3Config, ep_layout_ranked, ranked_pool_width
from xtier_b200.tools.three_tier import route_profile, tier_plan


def _routers(cfg, layers, skew=None):
    g = torch.Generator().manual_seed(0)
    out = {}
    for li in layers:
        w = torch.randn(cfg.experts, cfg.hidden, generator=g) * 0.02
        corr = torch.zeros(cfg.experts)
        if skew is not None and li in skew:
            corr[:skew[li]] = 1.0   # a few experts win most selections
        out[li] = (w.bfloat16(), corr)
    return out


def test_route_profile_sums_to_top_k():
    cfg = DeepSeekV3Config.tiny()
    prof = route_profile(_routers(cfg, [1, 2]), cfg, tokens=512)
    assert sorted(prof['layers']) == ['1', '2']
    for p in prof['layers'].values():
        assert len(p) == cfg.experts
        assert abs(sum(p) - cfg.top_k) < 1e-9
        assert max(p) <= 1.0


def test_tier_plan_respects_the_budget_and_follows_the_routes():
    cfg = DeepSeekV3Config.tiny(experts=64, n_group=8, topk_group=4, top_k=8)
    prof = route_profile(_routers(cfg, [1, 2, 3], skew={2: 6}), cfg, tokens=2048)
    budget = 3 * 13
    slots, summary = tier_plan(prof, None, budget, cfg.experts)
    assert sum(slots.values()) <= budget
    assert all(0 <= n <= cfg.experts for n in slots.values())
    assert summary['predicted_us'] <= summary['uniform_us'] + 1e-9
    # the concentrated layer needs fewer slots for the same share of its routes
    assert slots[2] <= max(slots[1], slots[3])


def test_ep_layout_ranked_places_the_most_routed():
    E, W = 16, 4
    pop = np.arange(E, dtype=np.float64)[::-1].copy()   # expert 0 most routed
    table, pools, cpu = ep_layout_ranked(E, W, 6, pop, stride=5, width=4)
    gpu = sorted(e for p in pools for e in p)
    assert gpu == [0, 1, 2, 3, 4, 5]
    assert cpu == list(range(6, 16))                     # most routed first
    assert pools[0] == [0, 1, 2, 3] and pools[1] == [4, 5] and pools[2] == [] and pools[3] == []
    for r, p in enumerate(pools):
        for s, e in enumerate(p):
            assert int(table[e]) == r * 5 + s
    assert all(int(table[e]) == -1 for e in cpu)
    with pytest.raises(ValueError):
        ep_layout_ranked(E, W, 6, pop, stride=5, width=3)
    assert ranked_pool_width(E, W, {1: 6, 2: 3}, {1: pop, 2: pop[::-1].copy()}) == 4


def test_synthetic_table_streams_and_reuses(tmp_path):
    from xtier_b200.tables import RowStore
    from xtier_b200.tables.engram import synthetic_table
    path = str(tmp_path / 'bigram')
    segs = synthetic_table(path, 3000, 64, std=0.02, seed=3, segments=2, chunk_rows=256, device='cpu')
    assert [s.count for s in segs] == [1500, 1500]
    st = RowStore(segs, 128, io_threads=1, cache_rows=64)
    rows = torch.from_numpy(st.lookup(np.arange(0, 3000, 7))).view(torch.bfloat16).float()
    assert 0.015 < float(rows.std()) < 0.025
    # the bytes depend on (shape, seed) only: a second call reuses the files, another path gets the same bytes
    m0 = os.path.getmtime(segs[0].path)
    assert synthetic_table(path, 3000, 64, std=0.02, seed=3, segments=2, chunk_rows=256, device='cpu') == segs
    assert os.path.getmtime(segs[0].path) == m0
    first = torch.from_numpy(st.lookup(np.array([0, 1500]))).clone()
    st.close()
    segs2 = synthetic_table(str(tmp_path / 'other'), 3000, 64, std=0.02, seed=3, segments=2, chunk_rows=256,
                            device='cpu')
    st2 = RowStore(segs2, 128, io_threads=1, cache_rows=64)
    assert torch.equal(torch.from_numpy(st2.lookup(np.array([0, 1500]))), first)
    st2.close()
