"""Headline benchmark of BASELINE.json: 32-way decode tokens/s of the DeepSeek-V3-shaped model (config 3) at N GPUs of
one node, device-timed, max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 3|2]

Config 3 (default): the 61-layer DeepSeek-V3 shape (MLA 128 heads, 256 MXFP4 experts top-8 with grouped sigmoid
routing, one shared expert, first 3 layers dense, vocab 129280), random-init weights, 32 concurrent requests of a
4096-token random prompt and 256 decode tokens. The requests are split over the N ranks (attention data parallel,
32 / N requests per rank); the routed experts are split over the ranks (expert parallelism: rank r owns experts
[r * 256 / N, (r + 1) * 256 / N), tokens reach their experts' owners and come back through in-kernel NVLink peer
stores). When the N GPUs cannot hold all 347 GB of experts (N = 1, 2), every owner keeps as many of its experts in HBM
as fit and the rest form a CPU tier on the C++ engine, reached through the mailbox inside the captured step -- the
tiered product. The KV cache of the prompts is filled with random latent rows (the prompt ids are random; prefill is
measured on its own) up to the middle of the 256 decode positions, so the timed steps see the average context. W
untimed and K timed decode steps (one token for every request) are replayed from one captured CUDA graph, bracketed by
a barrier and a device synchronize, timed with CUDA events; the job time is the max over ranks. Each step streams
tens of GB of weights (far more than the 126 MB L2), so no L2 flush is needed. `e2e` repeats the K steps through the
public API (`Generator.decode_one`: pinned H2D of the step's input tokens, replay, D2H of the next tokens).

Config 2 (--config 2): the Qwen3-style 48-layer model of round one's flagship (one request per GPU, 40 % of the
experts in HBM, the rest on the CPU tier).

The reference arm (--impl reference) would run the unmodified reference from baseline/_ref; it is an SGLang plugin
and SGLang is not installed in this image, so that arm reports itself unavailable.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = 'decode tok/s (bs=1, 32-way) & 64K-prefill TTFT at 1/2/4/8 B200, max over ranks'
QWEN_BASELINE_TOKS = 139.5   # the reference's published Qwen3.8 decode, packs off (tok/s, bs=1, RTX PRO 5000)
GB = 1e9


class ClockSampler:
    """nvidia-smi samples of this rank's GPU (every 50 ms) while the timed work runs."""

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', '-i', str(self.gpu), '--query-gpu=clocks.sm,clocks.max.sm,power.draw,'
                 'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
                 'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap',
                 '--format=csv,noheader,nounits', '-lms', '50'],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)   # the first sample is in before the timed work starts
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(',')]
            if len(parts) >= 7:
                self.samples.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if not self.samples:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['not sampled']}
        sm = [float(s[0]) for s in self.samples if s[0].replace('.', '').isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace('.', '').isdigit()]
        names = ['hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap']
        reasons = sorted({n for s in self.samples for n, v in zip(names, s[3:7]) if v.lower() == 'active'})
        return {'sm_mhz': statistics.median(sm) if sm else None, 'sm_max_mhz': max(mx) if mx else None,
                'reasons': reasons, 'samples': len(self.samples)}


def cpu_model() -> str:
    try:
        for line in open('/proc/cpuinfo'):
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


def reference_arm(args):
    line = {'impl': 'reference',
            'unavailable': 'the reference is an SGLang plugin (entry point xtier.plugin:load) and SGLang is not '
                           'installed in this image (no network); its pip install into baseline/_ref succeeds but '
                           'nothing can run it'}
    if int(os.environ.get('RANK', '0')) == 0:
        print(json.dumps(line), flush=True)


class Ctx:
    """Per-rank plumbing shared by the configs: process group, CPU placement, timing helpers."""

    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get('WORLD_SIZE', '1'))
        self.rank = int(os.environ.get('RANK', '0'))
        self.local = int(os.environ.get('LOCAL_RANK', '0'))
        if self.world != args.gpus:
            raise SystemExit(f'bench: --gpus {args.gpus} but WORLD_SIZE={self.world}')
        torch.cuda.set_device(self.local)
        if self.world > 1:
            from datetime import timedelta
            dist.init_process_group('nccl', timeout=timedelta(seconds=300),
                                    device_id=torch.device('cuda', self.local))
        # CPU partition of this rank (NUMA node of its GPU when the node has enough of them): engine workers, the
        # main thread, the mailbox dispatcher (xtier_b200/engine/placement.py)
        from xtier_b200.engine import placement
        self.place = placement.for_rank(self.local, self.world, spare_siblings=False)
        mine = sorted(set(self.place.workers) | {self.place.main, self.place.dispatcher})
        os.sched_setaffinity(0, mine)
        self.threads = args.threads or len(self.place.workers)
        os.environ["XTIER_DISPATCH_CPU"] = str(self.place.dispatcher)
        os.environ["XTIER_WORKER_CPUS"] = ','.join(map(str, self.place.workers))
        os.environ.setdefault("XTIER_SPIN_US", "5000")   # decode calls come every few hundred microseconds
        torch.set_num_threads(1)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device='cuda')
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device='cuda')
        self.dist.all_reduce(t)
        return float(t.item())

    def timed_decode(self, gen, args):
        """W warm-up replays, then K replays between barriers timed by CUDA events (max over ranks), then K steps
        through the public API (wall clock, max over ranks). Clocks are sampled over both timed loops."""
        torch = self.torch
        for _ in range(args.warmup):
            gen.step()
        torch.cuda.synchronize()
        gen.check()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(self.local) as clocks:
            self.barrier()
            start.record()
            for _ in range(args.steps):
                gen.step()
            end.record()
            self.barrier()
            gen.check()
            ms = self.max_over_ranks(start.elapsed_time(end))
            e2e_s = None
            if not args.no_e2e:
                self.barrier()
                t2 = time.perf_counter()
                for _ in range(args.steps):
                    gen.decode_one()
                e2e_s = self.max_over_ranks(time.perf_counter() - t2)
                gen.check()
        return ms, e2e_s, clocks.summary()

    def gather_tokens(self, t) -> list[int]:
        torch = self.torch
        if self.world == 1:
            return t.cpu().tolist()
        out = [torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t.contiguous())
        return torch.cat(out).cpu().tolist()

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def graph_launches(gen) -> dict:
    from xtier_b200.runtime.decode import graph_kernels, own_kernel_launches
    try:
        counts = graph_kernels(gen.graph)
    except Exception as e:   # the count is a claim only when it was read from the graph
        return {'error': f'{type(e).__name__}: {e}'}
    return {'own_per_step': own_kernel_launches(counts), 'all_per_step': sum(counts.values()),
            'own_kernels': len([k for k in counts if k.startswith('_ZN2xt')])}


def plan_config3(cfg, world: int, B: int, max_len: int, torch, reserve_gb: float, stage_slots: int = 0):
    """HBM pool slots per rank and MoE layer: what fits beside the dense weights, the KV cache, the workspaces and the
    PCIe staging slots (shared by the layers)."""
    free, _ = torch.cuda.mem_get_info()
    nsel = (max_len + 127) // 128 * 128
    kv = B * max_len * 416 * cfg.layers
    ws = B * nsel * 1088 * 2 + B * (nsel // 128) * 128 * 514 * 4
    spare = free - cfg.dense_bytes() - kv - ws - int(reserve_gb * GB) - stage_slots * cfg.expert_bytes()
    El = cfg.experts // world
    n = max(0, spare // (cfg.expert_bytes() * cfg.moe_layers()))
    return int(min(El, n)), free


def run_config3(args, ctx: Ctx) -> dict:
    torch = ctx.torch
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Config, DeepSeekV3Model
    from xtier_b200.runtime.decode import Generator
    world, rank = ctx.world, ctx.rank
    cfg = DeepSeekV3Config(layers=args.layers, attn='mla')
    if args.requests % world:
        raise SystemExit(f'bench: {args.requests} requests do not split over {world} ranks')
    B = args.requests // world
    # the timed steps straddle the middle of the 256 decode positions (the average context of the decode)
    fill = max(args.prompt, args.prompt + args.gen // 2 - args.warmup - args.steps // 2)
    max_len = (fill + args.warmup + 2 * args.steps + 8 + 127) // 128 * 128
    El = cfg.experts // world
    gpu_per_rank, free = plan_config3(cfg, world, B, max_len, torch, args.reserve_gb)
    S = 0   # PCIe staging slots (with a CPU tier): explicit, or the share of the touched CPU-tier experts
    if gpu_per_rank < El:
        from xtier_b200 import config as xconfig
        S = xconfig.get('XTIER_EP_PCIE_SLOTS') if args.pcie_slots == -2 else args.pcie_slots
        if S < 0:
            touched = (cfg.experts - world * gpu_per_rank) * (1.0 - (1.0 - cfg.top_k / cfg.experts) ** B)
            S = math.ceil(xconfig.get('XTIER_EP_PCIE_SHARE') * touched)
        if S:
            gpu_per_rank, free = plan_config3(cfg, world, B, max_len, torch, args.reserve_gb, S)
    if gpu_per_rank < 1:
        raise SystemExit('bench: the dense weights and the KV cache leave no HBM for routed experts')
    cpu_per_layer = world * (El - gpu_per_rank)
    cpu_bytes = cpu_per_layer * cfg.moe_layers() * cfg.expert_bytes()
    if cpu_per_layer:
        import psutil
        avail = psutil.virtual_memory().available / max(1, world)
        need = cpu_bytes + 6 * GB   # + the process itself, the pinned bounce buffer and slack
        if need > avail:
            raise SystemExit(f'bench: the CPU tier needs {need / GB:.1f} GB of host memory per rank, '
                             f'{avail / GB:.1f} GB is available')
    mailbox = Mailbox(cfg.hidden) if cpu_per_layer else None
    with_ttft = args.ttft and not cpu_per_layer   # the sparse prefill needs every expert in some GPU's HBM
    if rank == 0:
        print(f'bench: config 3 at {world} GPU(s): {B} requests per rank, {gpu_per_rank} of {El} experts per rank and '
              f'layer in HBM ({free / GB:.1f} GB free), CPU tier {cpu_per_layer} experts per layer '
              f'({cpu_bytes / GB:.1f} GB per rank)', file=sys.stderr, flush=True)
    t0 = time.time()
    model = DeepSeekV3Model(cfg, device='cuda', seed=1234, ep=True, gpu_experts=gpu_per_rank, mailbox=mailbox,
                            engine_threads=ctx.threads, decode_tokens=B, indexer=with_ttft, pcie_slots=S)
    if mailbox is not None:
        mailbox.start(cpu=ctx.place.dispatcher)
    os.sched_setaffinity(0, [ctx.place.main])   # main thread off the workers' CPUs
    build_s = time.time() - t0
    if rank == 0:
        print(f'bench: model built in {build_s:.1f} s', file=sys.stderr, flush=True)
    gen = Generator(model, batch=B, max_len=max_len)
    # the 32 requests (input tokens and caches) do not depend on N: rank r serves requests r * B .. r * B + B - 1
    model.fill_synthetic_cache(gen.state, fill, seed=11, first_request=rank * B)
    toks = torch.randint(0, cfg.vocab, (args.requests,), generator=torch.Generator().manual_seed(100))
    toks = toks[rank * B:(rank + 1) * B].contiguous()
    gen.buf['tokens'].copy_(toks)
    gen.host_tokens.copy_(toks)
    gen.buf['pos'].fill_(fill)
    gen.capture(keep_graph=True)
    launches = graph_launches(gen)
    if args.profile:
        return profile_steps(gen, args, ctx)
    # the first step's next token of every request, gathered (the same requests, caches and weights at every N). The
    # tokens agree across N only in part: the projections' split-K depends on the rows per rank and the EP combine
    # order on the rank count, and the FP32 summation-order differences flip near-tied top-8 routes and argmaxes of a
    # random-init model (1 vs 2 GPUs, 8 layers: 18 of 32 equal)
    gen.step()
    first_tokens = ctx.gather_tokens(gen.buf['next'])
    ms, e2e_s, clocks = ctx.timed_decode(gen, args)
    ms_per_step = ms / args.steps
    value = args.requests * args.steps / (ms / 1000.0)
    e2e = None
    if e2e_s is not None:
        e2e = {'value': round(args.requests * args.steps / e2e_s, 2), 'unit': 'tok/s',
               'h2d_bytes_per_step': gen.h2d_bytes_per_step * world, 'd2h_bytes_per_step': gen.d2h_bytes_per_step * world,
               'api': 'Generator.decode_one (each rank: pinned H2D of its requests\' tokens, replay, D2H of the next)'}
    mb = mailbox.stats() if mailbox is not None else {}
    gpu_experts_bytes = gpu_per_rank * cfg.moe_layers() * cfg.expert_bytes()
    gen.graph = None
    if with_ttft:
        del gen
        torch.cuda.empty_cache()
        ttft = time_ttft(args, ctx, model)
    elif args.ttft:
        ttft = {'tokens': args.ttft_tokens,
                'unavailable': f'the prefill computes every expert on a GPU; at {world} GPU(s) '
                               f'{cpu_per_layer} experts per layer live in host RAM (the decode CPU tier)'}
    else:
        ttft = None
    line = {
        'metric': METRIC, 'value': round(value, 2), 'unit': 'tok/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(ms_per_step, 4), 'higher_is_better': True, 'scaling': 'strong',
        'vs_baseline': None, 'dtype': 'bf16', 'data': 'synthetic',
        'config': {
            'model': 'DeepSeek-V3-shaped 61L H7168 MLA-128h 256 MXFP4 experts top-8 (grouped sigmoid) + 1 shared, '
                     'I2048, 3 dense layers I18432, vocab 129280 (benchmark config 3)',
            'global_batch': args.requests, 'seq_len': args.prompt + args.gen, 'prompt': args.prompt,
            'decode_tokens': args.gen, 'context_at_timed_steps': fill,
            'parallelism': f'ep{world} (experts) + dp{world} (attention, {B} requests per rank)',
            'layers': cfg.layers,
            'experts_in_hbm_per_rank_and_layer': gpu_per_rank, 'experts_per_rank_and_layer': El,
            'cpu_tier_experts_per_layer': cpu_per_layer, 'cpu_tier_gb_per_rank': round(cpu_bytes / GB, 1),
            'hbm_expert_gb_per_rank': round(gpu_experts_bytes / GB, 1),
            'cpu_engine_threads': ctx.threads if cpu_per_layer else 0, 'cpu': cpu_model(), 'cpus': os.cpu_count(),
            'pcie_staging_slots': model.pcie_slots,
            'kv': 'NVFP4 latent cache filled with random latent rows for the random prompts (prefill measured '
                  'separately)',
            'l2': 'inputs larger than L2: each step streams tens of GB of weights',
            'weights': 'random-init; experts as random MXFP4 codes with block scales',
            'baseline': 'no published number of the reference for this model and machine (vs_baseline null)'},
        'clocks': clocks, 'e2e': e2e,
        'gpu_launches': (launches['own_per_step'] * args.steps) if 'own_per_step' in launches else None,
        'graph_kernels': launches,
        'mailbox': {'calls': mb.get('calls'), 'mean_us': round(mb.get('mean_us', 0) or 0, 2)},
        'setup_s': {'build': round(build_s, 1)},
        'first_step_tokens': first_tokens,
        'ttft_64k': ttft,
    }
    if mailbox is not None:
        mailbox.stop()
    model.close()
    return line


def time_ttft(args, ctx: Ctx, model) -> dict:
    """benchmark config 4: time to first token of one random-id prompt of --ttft-tokens tokens with DSA sparse
    attention (index top-2048) over the group (models/deepseek_prefill.py). One untimed run (allocations), then one
    timed by CUDA events between barriers, max over ranks."""
    torch = ctx.torch
    from xtier_b200.models.deepseek_prefill import SparsePrefill
    T = args.ttft_tokens
    try:
        sp = SparsePrefill(model, T, q_chunk=args.ttft_q_chunk, moe_chunk=16384)
        ids = torch.randint(0, model.cfg.vocab, (T,), generator=torch.Generator().manual_seed(77))
        mine = ids[ctx.rank * sp.Tl:(ctx.rank + 1) * sp.Tl].cuda()
        t0 = time.time()
        first = sp.run(mine)
        ctx.barrier()
        warm_s = time.time() - t0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ctx.barrier()
        e0.record()
        first = sp.run(mine)
        e1.record()
        ctx.barrier()
        sp.check()
        ms = ctx.max_over_ranks(e0.elapsed_time(e1))
        tok = int(ctx.max_over_ranks(float(first[0])))
    except Exception as e:   # reported in the line; the decode measurement above stands
        return {'tokens': T, 'error': f'{type(e).__name__}: {e}'[:300]}
    return {'tokens': T, 'ttft_ms': round(ms, 1), 'tok_s': round(T / ms * 1e3, 1), 'first_token': tok,
            'untimed_first_run_s': round(warm_s, 1),
            'parallelism': f'sequence-parallel attention over {ctx.world} rank(s) (latent + index caches all-gathered), '
                           f'expert-parallel MoE (all-to-all, grouped FP4 tcgen05 GEMM)',
            'attention': f'DSA: FP8 lightning indexer (64 heads x 128), top-{sp.topk} keys per query, tcgen05 MLA '
                         f'over the NVFP4 latent cache',
            'timing': 'warm (second run), device events, max over ranks'}


def profile_steps(gen, args, ctx):
    from torch.profiler import ProfilerActivity, profile
    torch = ctx.torch
    for _ in range(args.warmup):
        gen.step()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(args.profile):
            gen.step()
        torch.cuda.synchronize()
    if ctx.rank == 0:
        print(prof.key_averages().table(sort_by='cuda_time_total', row_limit=30, max_name_column_width=70))
    gen.graph = None
    return None


def run_config2(args, ctx: Ctx) -> dict:
    torch = ctx.torch
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    world, rank = ctx.world, ctx.rank
    cfg = Qwen3MoeConfig(layers=args.layers)
    mailbox = Mailbox(cfg.hidden) if args.hot < 1.0 else None
    t0 = time.time()
    peer = world > 1 and not args.no_peer
    # data parallel replicas of one model (same weights on every GPU); with peer slots each GPU keeps its 40 % budget
    # of hot slots and reads the experts held by the other GPUs' slots over NVLink
    model = Qwen3MoeModel(cfg, device='cuda', seed=1234, hot_fraction=args.hot, engine_threads=ctx.threads,
                          mailbox=mailbox, peer=peer)
    if mailbox is not None:
        mailbox.start(cpu=ctx.place.dispatcher)
    os.sched_setaffinity(0, [ctx.place.main])
    build_s = time.time() - t0
    max_len = args.prompt + args.warmup + 2 * args.steps + 16
    gen = Generator(model, batch=1, max_len=max_len)
    prompt = torch.randint(0, cfg.vocab, (1, args.prompt), generator=torch.Generator().manual_seed(rank))
    gen.prefill(prompt)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    gen.prefill(prompt)
    e1.record()
    torch.cuda.synchronize()
    ttft_ms = e0.elapsed_time(e1)
    gen.capture(keep_graph=True)
    launches = graph_launches(gen)
    if args.profile:
        return profile_steps(gen, args, ctx)
    ms, e2e_s, clocks = ctx.timed_decode(gen, args)
    value = world * args.steps / (ms / 1000.0)
    e2e = None
    if e2e_s is not None:
        e2e = {'value': round(world * args.steps / e2e_s, 2), 'unit': 'tok/s',
               'h2d_bytes_per_step': gen.h2d_bytes_per_step * world, 'd2h_bytes_per_step': gen.d2h_bytes_per_step * world,
               'api': 'Generator.decode_one'}
    mb = mailbox.stats() if mailbox is not None else {}
    line = {
        'metric': 'decode tok/s (bs=1 per GPU)', 'value': round(value, 2), 'unit': 'tok/s', 'n_gpus': world,
        'steps': args.steps, 'warmup': args.warmup, 'ms_per_step': round(ms / args.steps, 4),
        'higher_is_better': True, 'scaling': 'weak', 'vs_baseline': round(value / QWEN_BASELINE_TOKS, 3),
        'dtype': 'bf16', 'data': 'synthetic',
        'config': {'model': 'qwen3-style MoE 48L H2048 GQA32/4 128E top-8 I768 NVFP4 (benchmark config 2)',
                   'global_batch': world, 'seq_len': args.prompt + args.warmup + args.steps,
                   'prompt': args.prompt, 'parallelism': f'dp{world}', 'hot_fraction': args.hot,
                   'hot_slots': ('each GPU holds hot_fraction of the experts; the GPUs\' slots form one pool read '
                                 'over NVLink peer memory' if peer else 'per GPU'),
                   'cpu_engine_threads': ctx.threads, 'cpu': cpu_model(), 'layers': cfg.layers,
                   'l2': 'inputs larger than L2: each step streams > 1.8 GB of weights',
                   'weights': 'random-init, experts as random NVFP4 codes and block scales',
                   'baseline': 'vs_baseline divides by 139.5 tok/s, the reference\'s Qwen3.8 bs=1 decode '
                               '(published, RTX PRO 5000; a different model and machine)'},
        'clocks': clocks, 'e2e': e2e,
        'gpu_launches': (launches['own_per_step'] * args.steps) if 'own_per_step' in launches else None,
        'graph_kernels': launches,
        'mailbox': {'calls': mb.get('calls'), 'mean_us': round(mb.get('mean_us', 0) or 0, 2)},
        'setup_s': {'build': round(build_s, 1)},
        'prefill': {'tokens': args.prompt, 'ttft_ms': round(ttft_ms, 1), 'timing': 'warm, device events'},
    }
    gen.graph = None
    if mailbox is not None:
        mailbox.stop()
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=4)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--config', type=int, default=3, choices=[2, 3])
    ap.add_argument('--requests', type=int, default=32, help='config 3: concurrent requests of the whole job')
    ap.add_argument('--prompt', type=int, default=None, help='prompt tokens (config 3: 4096, config 2: 2048)')
    ap.add_argument('--gen', type=int, default=256, help='config 3: decode tokens per request')
    ap.add_argument('--layers', type=int, default=None, help='layers (config 3: 61, config 2: 48)')
    ap.add_argument('--reserve-gb', type=float, default=3.0,
                    help='config 3: HBM kept free beside the dense weights, KV and workspaces')
    ap.add_argument('--hot', type=float, default=0.4, help='config 2: fraction of each layer\'s experts in HBM')
    ap.add_argument('--threads', type=int, default=0, help='CPU engine workers per rank (0: auto)')
    ap.add_argument('--pcie-slots', type=int, default=-2,
                    help='config 3 with a CPU tier: GPU staging slots for CPU-tier experts read over PCIe (-2: '
                         'XTIER_EP_PCIE_SLOTS, -1: XTIER_EP_PCIE_SHARE of the touched CPU-tier experts, 0: off)')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-peer', action='store_true', help='config 2, N > 1: no node-wide slot pool')
    ap.add_argument('--profile', type=int, default=0, help='print per-kernel device time of N graph replays and exit')
    ap.add_argument('--no-ttft', dest='ttft', action='store_false',
                    help='config 3: skip the 64K-prefill time to first token (config 4, same model)')
    ap.add_argument('--ttft-tokens', type=int, default=65536)
    ap.add_argument('--ttft-q-chunk', type=int, default=1024, help='queries per indexer / attention chunk')
    args = ap.parse_args()
    if args.impl == 'reference':
        return reference_arm(args)
    if args.warmup < 3:
        raise SystemExit('bench: at least 3 warm-up steps')
    if args.prompt is None:
        args.prompt = 4096 if args.config == 3 else 2048
    if args.layers is None:
        args.layers = 61 if args.config == 3 else 48
    ctx = Ctx(args)
    line = run_config3(args, ctx) if args.config == 3 else run_config2(args, ctx)
    if line is not None and ctx.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


if __name__ == '__main__':
    main()
