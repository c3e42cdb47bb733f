"""Three tiers on the GPU: a DeepSeek-style EP layer whose experts sit in a planned GPU pool, the CPU engine's RAM and
cold records on disk matches the fp32 reference over all experts; the config-5 runner decodes end to end (planner
layout, cold reads, the bigram table inside the graph)."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_three_tier_layer_matches_reference(cuda_ops, tmp_path):
    from xtier_b200 import formats
    from xtier_b200.cache.cold import ColdPool
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.deepseek_v3 import (DeepSeekV3Config, DeepSeekV3Model, empty_experts,
                                               synthetic_experts_by_id)
    for v in ('RANK', 'WORLD_SIZE', 'LOCAL_RANK'):
        os.environ.pop(v, None)
    cfg = DeepSeekV3Config.tiny(layers=2, dense_layers=1, shared=0)
    E, T, seed = cfg.experts, 4, 3
    pop = {1: np.arange(E, dtype=np.float64)[::-1].copy()}   # expert 0 most routed
    seen = {}

    def plan_fn(routers):
        seen.update(routers)
        return {1: 4}, pop

    pool = ColdPool(str(tmp_path / 'cold'))
    mb = Mailbox(cfg.hidden, timeout_s=10.0)
    model = DeepSeekV3Model(cfg, device='cuda', seed=seed, ep=True, mailbox=mb, engine_threads=2, decode_tokens=T,
                            plan_fn=plan_fn, cold=pool, ram_experts=6)
    mb.start()
    try:
        assert sorted(seen) == [1]
        moe = model.layers[1]['moe']
        table = moe.table.cpu()
        assert [e for e in range(E) if int(table[e]) >= 0] == [0, 1, 2, 3]   # the planned GPU tier
        x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(9)).bfloat16()
        for _ in range(3):   # repeated calls: cold experts read into RAM slots, others evicted
            out = moe.forward(x.cuda())
            torch.cuda.synchronize()
            model.check()
            ids, w = moe.router.ids[:T, :cfg.top_k].cpu(), moe.router.wt[:T, :cfg.top_k].cpu()
            full = empty_experts(E, cfg.hidden, cfg.inter, cfg.fmt, 'cuda')
            synthetic_experts_by_id(full, list(range(E)), seed * 1000 + 1, cfg.std)
            ref = formats.reference_moe(x, ids, w, full.to('cpu'))
            rel = float((out.cpu().float() - ref).norm() / ref.norm())
            assert rel < 2e-2, rel
        # GPU tier 0-3, RAM 4-9 (the next most routed), cold 10-15: a route to a cold expert read its record
        if any(e >= 10 for e in ids.view(-1).tolist()):
            assert pool.stats()['bytes_read'] > 0
    finally:
        mb.stop()
        model.close()
        pool.close()


def test_three_tier_runner_small(cuda_ops, tmp_path):
    env = dict(os.environ, PYTHONPATH=ROOT)
    for v in ('RANK', 'WORLD_SIZE', 'LOCAL_RANK'):
        env.pop(v, None)
    cmd = [sys.executable, '-m', 'xtier_b200.tools.three_tier', '--layers', '2', '--dense-layers', '1',
           '--context', '2048', '--steps', '4', '--warmup', '2', '--cold-dir', str(tmp_path / 'cold'),
           '--table-rows', '65536', '--threads', '4']
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-3000:]
    line = json.loads([ln for ln in r.stdout.splitlines() if ln.startswith('{')][-1])
    assert line['tool'] == 'three_tier' and line['tok_s_per_request'] > 0
    assert line['planner']['mode'] == 'auto'
    assert sum(line['gpu_experts_per_layer'].values()) <= line['planner']['budget_slots']
    assert line['mailbox_calls_per_token'] > 0          # the CPU tier served routes
    assert line['table']['lookup']['lookups'] > 0       # the bigram rows were read inside the graph
