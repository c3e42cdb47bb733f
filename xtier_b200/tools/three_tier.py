"""benchmark config 5: three-tier decode of the DeepSeek-V3-shaped model at batch 1 over a 32K random-id context.

Tiers of every MoE layer: GPU hot slots (by default 20 % of the experts node-wide, spread over the process group's
GPUs by expert parallelism: a token's routes to another GPU's experts reach that GPU over NVLink inside the fused
dispatch / combine kernel), the CPU engine's RAM (50 %) and cold records on NVMe read on demand (the rest, with the
engine's decayed-use RAM slot replacement). A hashed-bigram BF16 table (4M rows x 4096, 32 GiB) on NVMe is looked up
inside the decode graph with a row cache and projected to the hidden size.

Planner auto-layout: the route probability of every expert of every layer (the layer's own router over random
hidden states, DeepSeek's grouped sigmoid top-8 with the correction bias), the probe coefficients (a `plan_probe`
JSON, or the cost model's defaults) and the GPU slot budget go through `planner.auto.make_plan`; a layer's most routed
experts take its GPU slots (in their owners' pools), the next ones its RAM slots, the rest stay cold.

Each rank decodes its own batch-1 request (random prompt ids whose 32K-token KV cache is filled with random latent
rows; the prefill is not part of this measurement). Device time by CUDA events over the timed steps, max over ranks.

    python -m xtier_b200.tools.three_tier --cold-dir DIR --table-dir DIR [--layers 61] [--context 32768]
    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m xtier_b200.tools.three_tier --cold-dir DIR ...

Full size needs about 0.8 x 256 experts x 58 layers of cold records (~260 GB) and the CPU tier's RAM (~165 GB per
rank); `--layers` scales the model (and every tier) down to what a machine holds.

Reference parity: benchmark config 5 (the reference's three-tier run: xtier/cache/ with remote slots, the CPU engine,
xtier/cache/cold.py, xtier/tables/lookup.py, xtier/planner/auto.py).
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch


def route_profile(routers: dict, cfg, tokens: int = 4096, seed: int = 0) -> dict:
    """Per-token route probability of every expert of every MoE layer: `tokens` random unit-RMS hidden states through
    the layer's router with DeepSeek's selection (sigmoid scores plus the correction bias, the top `topk_group` of
    `n_group` groups by their two best scores, top-k inside them). routers: {layer: (router_w [E, H], corr [E])}."""
    out = {}
    for li, (w, corr) in sorted(routers.items()):
        g = torch.Generator(device=w.device).manual_seed(seed * 7919 + li)
        x = torch.randn(tokens, w.shape[1], device=w.device, generator=g)
        s = torch.sigmoid(x @ w.float().t()) + corr.to(w.device).float()
        E = s.shape[1]
        grp = s.view(tokens, cfg.n_group, E // cfg.n_group).topk(2, -1).values.sum(-1)
        keep = grp.topk(cfg.topk_group, -1).indices
        mask = torch.zeros(tokens, cfg.n_group, dtype=torch.bool, device=w.device)
        mask.scatter_(1, keep, True)
        s = s.masked_fill(~mask.repeat_interleave(E // cfg.n_group, 1), float('-inf'))
        ids = s.topk(cfg.top_k, -1).indices
        counts = torch.bincount(ids.reshape(-1), minlength=E).double().cpu().numpy()
        out[str(li)] = (counts / tokens).tolist()
    return {'layers': out}


def tier_plan(profile: dict, probe: dict | None, budget_slots: int, E: int) -> tuple[dict, dict]:
    """({layer: node-wide GPU experts}, planner summary) for `budget_slots` GPU experts over the layers."""
    from ..planner.auto import make_plan
    plan = make_plan(profile, probe, budget_slots)
    slots = {int(k): max(0, min(E, int(v))) for k, v in plan['slots'].items()}
    summary = {k: plan[k] for k in ('predicted_us', 'uniform_us', 'lambda', 'budget_slots')}
    return slots, summary


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device='cuda')
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--layers', type=int, default=61)
    ap.add_argument('--dense-layers', type=int, default=3, help='leading dense layers (the rest are MoE)')
    ap.add_argument('--context', type=int, default=32768, help='tokens of context each request decodes after')
    ap.add_argument('--steps', type=int, default=32)
    ap.add_argument('--warmup', type=int, default=4)
    ap.add_argument('--gpu-frac', type=float, default=0.2, help='node-wide GPU slots, as a share of the experts')
    ap.add_argument('--cpu-frac', type=float, default=0.5, help='CPU engine RAM slots, as a share of the experts')
    ap.add_argument('--cold-dir', required=True, help='directories (comma separated, one per drive) of the cold store')
    ap.add_argument('--table-dir', default=None, help='directory of the bigram table (default: the first cold dir)')
    ap.add_argument('--table-rows', type=int, default=1 << 22)
    ap.add_argument('--table-dim', type=int, default=4096)
    ap.add_argument('--no-table', action='store_true')
    ap.add_argument('--probe', default=None, help='plan_probe JSON with the cost coefficients (default: built-in)')
    ap.add_argument('--no-plan', action='store_true', help='the same GPU share in every layer (no planner)')
    ap.add_argument('--threads', type=int, default=0, help='CPU engine workers per rank (0: this rank\'s share)')
    ap.add_argument('--seed', type=int, default=1234)
    a = ap.parse_args(argv)
    from ..cache.cold import ColdPool
    from ..engine.mailbox import Mailbox
    from ..models.deepseek_v3 import DeepSeekV3Config, DeepSeekV3Model
    from ..parallel import dist as xdist
    from ..runtime.decode import Generator
    env = xdist.init()
    world, rank = env.world, env.rank
    torch.cuda.set_device(env.local_rank)
    cfg = DeepSeekV3Config(layers=a.layers, dense_layers=a.dense_layers, attn='mla')
    E, moe_layers = cfg.experts, cfg.moe_layers()
    n_ram = max(1, int(round(a.cpu_frac * E)))
    budget = int(round(a.gpu_frac * E * moe_layers))
    threads = a.threads or max(1, (os.cpu_count() or 2) // world - 2)
    probe = None
    if a.probe:
        with open(a.probe) as f:
            probe = json.load(f)
    info = {}

    def plan_fn(routers):
        profile = route_profile(routers, cfg, seed=a.seed)
        popularity = {int(k): np.asarray(v) for k, v in profile['layers'].items()}
        if a.no_plan:
            per = max(1, budget // max(1, moe_layers))
            slots = {li: per for li in popularity}
            info['planner'] = {'mode': 'uniform', 'budget_slots': budget}
        else:
            slots, summary = tier_plan(profile, probe, budget, E)
            info['planner'] = dict(mode='auto', **summary)
        info['gpu_experts_per_layer'] = {str(k): v for k, v in sorted(slots.items())}
        return slots, popularity

    t0 = time.time()
    pool = ColdPool(a.cold_dir, key=f'xtier-three-tier-{a.layers}L-s{a.seed}')
    mailbox = Mailbox(cfg.hidden)
    model = DeepSeekV3Model(cfg, device='cuda', seed=a.seed, ep=True, mailbox=mailbox, engine_threads=threads,
                            decode_tokens=1, plan_fn=plan_fn, cold=pool, ram_experts=n_ram)
    build_s = time.time() - t0
    table = None
    if not a.no_table:
        from ..tables import RowStore
        from ..tables.engram import BigramTable, synthetic_table
        tdir = a.table_dir or a.cold_dir.split(',')[0]
        os.makedirs(tdir, exist_ok=True)
        path = os.path.join(tdir, f'bigram-{a.table_rows}x{a.table_dim}')
        if rank == 0:
            segs = synthetic_table(path, a.table_rows, a.table_dim, std=cfg.std, seed=a.seed)
        _barrier(world)
        if rank != 0:
            segs = synthetic_table(path, a.table_rows, a.table_dim, std=cfg.std, seed=a.seed)   # reuses rank 0's
        store = RowStore(segs, a.table_dim * 2)
        gp = torch.Generator(device='cuda').manual_seed(a.seed + 77)
        proj = (torch.randn(cfg.hidden, a.table_dim, device='cuda', generator=gp) * cfg.std).bfloat16()
        table = BigramTable(store, a.table_rows, a.table_dim, cfg.hidden, batch=1, device='cuda', seed=a.seed,
                            proj=proj)
        model.attach_bigram(table)
    setup_s = time.time() - t0
    mailbox.start()
    max_len = (a.context + a.warmup + a.steps + 8 + 127) // 128 * 128
    try:
        gen = Generator(model, batch=1, max_len=max_len)
        model.fill_synthetic_cache(gen.state, a.context, seed=11, first_request=rank)
        tok = torch.randint(0, cfg.vocab, (world,), generator=torch.Generator().manual_seed(100))[rank:rank + 1]
        gen.buf['tokens'].copy_(tok)
        gen.host_tokens.copy_(tok)
        gen.buf['prev'].copy_(torch.randint(0, cfg.vocab, (1,), generator=torch.Generator().manual_seed(101)))
        gen.buf['pos'].fill_(a.context)
        gen.capture()
        for _ in range(a.warmup):
            gen.step()
        torch.cuda.synchronize()
        model.check(gen.state)
        calls0 = mailbox.stats()['calls']
        cold0 = pool.stats()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        _barrier(world)
        e0.record()
        for _ in range(a.steps):
            gen.step()
        e1.record()
        _barrier(world)
        model.check(gen.state)
        ms = _max_over_ranks(e0.elapsed_time(e1), world)
        mb = mailbox.stats()
        cold1 = pool.stats()
        line = {
            'tool': 'three_tier', 'config': 'benchmark config 5', 'n_gpus': world, 'layers': cfg.layers,
            'moe_layers': moe_layers, 'context': a.context, 'batch_per_rank': 1, 'steps': a.steps,
            'warmup': a.warmup, 'ms_per_token': round(ms / a.steps, 3),
            'tok_s_per_request': round(a.steps / ms * 1e3, 2),
            'tok_s_all_ranks': round(world * a.steps / ms * 1e3, 2),
            'tiers': {'gpu_frac': a.gpu_frac, 'ram_experts_per_layer': n_ram,
                      'cold_share': round(1 - a.gpu_frac - a.cpu_frac, 3),
                      'gpu_pool_slots_per_rank': model.gpu_per_rank},
            'mailbox_calls_per_token': round((mb['calls'] - calls0) / a.steps, 2),
            'cpu_call_mean_us': round(mb.get('mean_us', 0) or 0, 1),
            'cold_store': {k: cold1.get(k, 0) - cold0.get(k, 0) for k in cold1} if isinstance(cold1, dict) else None,
            'table': (None if table is None else dict(table_rows=a.table_rows, dim=a.table_dim,
                                                      gib=round(a.table_rows * a.table_dim * 2 / 2 ** 30, 2),
                                                      lookup=table.store.stats())),
            'engine_threads': threads, 'cpus': os.cpu_count(),
            'setup_s': {'model': round(build_s, 1), 'total': round(setup_s, 1)},
            'timing': 'device events over the timed steps, max over ranks; KV of the context: random latent rows',
            **info,
        }
        if rank == 0:
            print(json.dumps(line), flush=True)
        gen.graph = None
    finally:
        mailbox.stop()
        model.close()
        pool.close()
        if world > 1:
            _barrier(world)
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == '__main__':
    main()
