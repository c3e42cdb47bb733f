"""Headline benchmark: decode tokens/s of the tiered MoE model (the Qwen3-style 48-layer config at one request per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Per GPU: the Qwen3-style 48-layer MoE (hidden 2048, GQA 32/4 x 128, 128 NVFP4 experts top-8 of I 768, vocab 151936,
random-init weights, Zipf(1.1) router bias) with only 40% of each layer's experts in GPU hot slots; the other 60% run
on the C++ CPU engine through the mailbox inside the CUDA graph. A 2048-token random prompt is prefilled, then W
untimed and K timed greedy decode steps (batch 1) are replayed from the captured graph; the K steps are bracketed by a
barrier and a device synchronize on both sides and timed with CUDA events; the job time is the max over ranks. With
N > 1 every rank runs its own request (data parallel, weak scaling: per-GPU work fixed) and `value` is the total
tokens/s of the job. Each step streams > 1.8 GB of weights (more than the 126 MB L2), so no L2 flush is needed.
`e2e` repeats the measurement through the public API (`Generator.decode_one`: pinned H2D of the input token, graph
replay, D2H read of the next token, every step), wall-clock, max over ranks.

The reference arm (--impl reference) would run the unmodified reference from baseline/_ref; it is an SGLang plugin
and SGLang is not installed in this image, so that arm reports itself unavailable.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

BASELINE_TOKS = 139.5   # the reference's published Qwen3.8 decode, packs off (tok/s, bs=1, RTX PRO 5000)
METRIC = 'decode tok/s (bs=1 per GPU)'


class ClockSampler:
    """nvidia-smi samples of this rank's GPU during the timed region."""

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
                 '--format=csv,noheader,nounits', '-lms', '200'],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
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


def reference_arm(args):
    line = {'impl': 'reference',
            'unavailable': 'the reference is an SGLang plugin (entry point xtier.plugin:load) and SGLang is not '
                           'installed in this image (no network); its pip install into baseline/_ref succeeds but '
                           'nothing can run it'}
    if int(os.environ.get('RANK', '0')) == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=256)
    ap.add_argument('--warmup', type=int, default=4)
    ap.add_argument('--impl', default='ours', choices=['ours', 'reference'])
    ap.add_argument('--prompt', type=int, default=2048)
    ap.add_argument('--hot', type=float, default=0.4, help='fraction of each layer\'s experts in GPU hot slots')
    ap.add_argument('--layers', type=int, default=48)
    ap.add_argument('--threads', type=int, default=0, help='CPU engine workers per rank (0: auto)')
    ap.add_argument('--no-e2e', action='store_true')
    ap.add_argument('--no-peer', action='store_true',
                    help='N > 1: keep every GPU\'s hot slots to itself (default: the hot slots of all GPUs form one pool '
                         'read over NVLink)')
    ap.add_argument('--long-prefill', type=int, default=65536,
                    help='also time a warm prefill of this many random tokens (0: skip)')
    ap.add_argument('--profile', type=int, default=0, help='print per-kernel device time of N graph replays and exit')
    args = ap.parse_args()
    if args.impl == 'reference':
        return reference_arm(args)
    if args.warmup < 3:
        raise SystemExit('bench: at least 3 warm-up steps')

    import torch
    import torch.distributed as dist

    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local = int(os.environ.get('LOCAL_RANK', '0'))
    if world != args.gpus:
        raise SystemExit(f'bench: --gpus {args.gpus} but WORLD_SIZE={world}')
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group('nccl', timeout=timedelta(seconds=600), device_id=torch.device('cuda', local))

    # CPU partition of this rank (NUMA node of its GPU when the node has enough of them): engine workers, the main
    # thread, the mailbox dispatcher (xtier_b200/engine/placement.py)
    from xtier_b200.engine import placement
    place = placement.for_rank(local, world, spare_siblings=False)
    mine = sorted(set(place.workers) | {place.main, place.dispatcher})
    os.sched_setaffinity(0, mine)
    threads = args.threads or len(place.workers)
    os.environ["XTIER_DISPATCH_CPU"] = str(place.dispatcher)
    os.environ["XTIER_WORKER_CPUS"] = ','.join(map(str, place.workers))
    os.environ.setdefault("XTIER_SPIN_US", "5000")   # decode calls come every few hundred microseconds: keep workers hot
    torch.set_num_threads(1)

    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator

    cfg = Qwen3MoeConfig(layers=args.layers)
    mailbox = Mailbox(cfg.hidden) if args.hot < 1.0 else None
    t0 = time.time()
    peer = world > 1 and not args.no_peer
    # data parallel replicas of one model (same weights on every GPU); with peer slots each GPU keeps its 40 % budget
    # of hot slots and reads the experts held by the other GPUs' slots over NVLink
    model = Qwen3MoeModel(cfg, device='cuda', seed=1234, hot_fraction=args.hot, engine_threads=threads,
                          mailbox=mailbox, peer=peer)
    if mailbox is not None:
        mailbox.start(cpu=place.dispatcher)
    os.sched_setaffinity(0, [place.main])   # main thread off the workers' CPUs
    build_s = time.time() - t0
    max_len = args.prompt + args.warmup + 2 * args.steps + 16
    gen = Generator(model, batch=1, max_len=max_len)
    prompt = torch.randint(0, cfg.vocab, (1, args.prompt), generator=torch.Generator().manual_seed(rank))
    t1 = time.time()
    gen.prefill(prompt)
    prefill_s = time.time() - t1
    # time to first token of a warm prefill of the same prompt (device time; rewrites the same KV entries)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    gen.prefill(prompt)
    e1.record()
    torch.cuda.synchronize()
    ttft_ms = e0.elapsed_time(e1)
    gen.capture()
    for _ in range(args.warmup):
        gen.step()
    torch.cuda.synchronize()
    gen.check()

    if args.profile:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(args.profile):
                gen.step()
            torch.cuda.synchronize()
        if rank == 0:
            print(prof.key_averages().table(sort_by='cuda_time_total', row_limit=25, max_name_column_width=70))
        gen.graph = None
        if mailbox is not None:
            mailbox.stop()
        return

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device='cuda')
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        for _ in range(args.steps):
            gen.step()
        end.record()
        barrier()
    gen.check()
    ms = max_over_ranks(start.elapsed_time(end))
    ms_per_step = ms / args.steps
    value = world * 1 * args.steps / (ms / 1000.0)

    e2e = None
    if not args.no_e2e:
        barrier()
        t2 = time.perf_counter()
        for _ in range(args.steps):
            gen.decode_one()
        e2e_s = max_over_ranks(time.perf_counter() - t2)
        gen.check()
        e2e = {'value': world * args.steps / e2e_s, 'unit': 'tok/s', 'h2d_bytes_per_step': gen.h2d_bytes_per_step,
               'd2h_bytes_per_step': gen.d2h_bytes_per_step, 'api': 'Generator.decode_one'}

    long_prefill = None
    if args.long_prefill:
        # time to first token of a long prompt: a fresh KV state, one untimed run (allocations, upload buffers,
        # kernel selection), then one timed by device events between barriers, max over ranks
        st2 = model.alloc_state(1, args.long_prefill + 8)
        ids = torch.randint(0, cfg.vocab, (args.long_prefill,), generator=torch.Generator().manual_seed(7 + rank))
        ids = ids.cuda()
        model.prefill(st2, ids)
        barrier()
        e0.record()
        model.prefill(st2, ids)
        e1.record()
        barrier()
        t_long = max_over_ranks(e0.elapsed_time(e1))
        long_prefill = {'tokens': args.long_prefill, 'ttft_ms': round(t_long, 1),
                        'tok_s': round(world * args.long_prefill / t_long * 1e3, 1),
                        'timing': 'warm, device events, max over ranks', 'scaling': 'weak (one prompt per GPU)'}
        del st2
        torch.cuda.empty_cache()

    mb_stats = mailbox.stats() if mailbox is not None else {}
    launches_per_step = 7 * cfg.layers + 1   # norms x2, rope+kv, attention, route, gate/up, down per layer; final norm
    line = {
        'metric': METRIC, 'value': round(value, 2), 'unit': 'tok/s', 'n_gpus': world, 'steps': args.steps,
        'warmup': args.warmup, 'ms_per_step': round(ms_per_step, 4), 'higher_is_better': True, 'scaling': 'weak',
        'vs_baseline': round(value / BASELINE_TOKS, 3), 'dtype': 'bf16', 'data': 'synthetic',
        'config': {'model': 'qwen3-style MoE 48L H2048 GQA32/4 128E top-8 I768 NVFP4 (BASELINE config 2)',
                   'global_batch': world, 'seq_len': args.prompt + args.warmup + args.steps,
                   'prompt': args.prompt, 'parallelism': f'dp{world}', 'hot_fraction': args.hot,
                   'hot_slots': ('each GPU holds hot_fraction of the experts; the GPUs\' slots form one pool read '
                                 'over NVLink peer memory' if peer else 'per GPU'),
                   'cpu_engine_threads': threads, 'layers': cfg.layers,
                   'l2': 'inputs larger than L2: each step streams > 1.8 GB of weights',
                   'weights': 'random-init, experts as random NVFP4 codes and block scales',
                   'baseline': 'vs_baseline divides by 139.5 tok/s, the reference\'s Qwen3.8 bs=1 decode '
                               '(published, RTX PRO 5000; a different model and machine)'},
        'clocks': clocks.summary(), 'e2e': e2e, 'gpu_launches': launches_per_step * args.steps,
        'mailbox': {'calls': mb_stats.get('calls'), 'mean_us': round(mb_stats.get('mean_us', 0) or 0, 2)},
        'setup_s': {'build': round(build_s, 1), 'prefill': round(prefill_s, 2)},
        'prefill': {'tokens': args.prompt, 'ttft_ms': round(ttft_ms, 1),
                    'tok_s': round(args.prompt / ttft_ms * 1e3, 1), 'timing': 'warm, device events'},
        'prefill_long': long_prefill,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    gen.graph = None
    if mailbox is not None:
        mailbox.stop()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
