"""Time to first token of a long prompt on the flagship model (Qwen3-style, 48 layers, 128 NVFP4 experts), and where it goes.

    python -m xtier_b200.tools.prefill_profile [--tokens 65536] [--layers 48] [--hot 0.4] [--threads 12]

Builds the Qwen3-style model (random-init, NVFP4 experts, `--hot` of each layer's experts in GPU slots, the rest
uploaded from pinned host memory per layer for the grouped GEMM), runs one untimed prefill of `--tokens` random ids,
one timed by CUDA events, then one under the PyTorch profiler, and prints the TTFT and the per-kernel device-time
table (sorted by total CUDA time).
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--tokens', type=int, default=65536)
    ap.add_argument('--layers', type=int, default=48)
    ap.add_argument('--hot', type=float, default=0.4)
    ap.add_argument('--threads', type=int, default=12)
    ap.add_argument('--rows', type=int, default=30)
    a = ap.parse_args(argv)
    from ..engine.mailbox import Mailbox
    from ..models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    cfg = Qwen3MoeConfig(layers=a.layers)
    mb = Mailbox(cfg.hidden) if a.hot < 1.0 else None
    model = Qwen3MoeModel(cfg, device='cuda', seed=1, hot_fraction=a.hot, engine_threads=a.threads, mailbox=mb)
    if mb is not None:
        mb.start()
    try:
        st = model.alloc_state(1, a.tokens + 8)
        ids = torch.randint(0, cfg.vocab, (a.tokens,), generator=torch.Generator().manual_seed(0)).cuda()
        model.prefill(st, ids)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        model.prefill(st, ids)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        print(json.dumps({'tool': 'prefill_profile', 'tokens': a.tokens, 'layers': a.layers, 'hot': a.hot,
                          'ttft_ms': round(ms, 1), 'tok_s': round(a.tokens / ms * 1e3, 1)}), flush=True)
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            model.prefill(st, ids)
            torch.cuda.synchronize()
        print(prof.key_averages().table(sort_by='cuda_time_total', row_limit=a.rows, max_name_column_width=60))
    finally:
        if mb is not None:
            mb.stop()


if __name__ == '__main__':
    main()
