"""Grouped FP4 expert GEMM (prefill) benchmark: one MoE layer's routed experts for `--tokens` tokens on the tensor
cores (xtier_b200.cache.prefill.grouped_experts), every expert resident on the GPU.

    python -m xtier_b200.tools.prefill_bench [--tokens 2048] [--hidden 2048] [--inter 768] [--experts 128] [--top-k 8]

Prints one JSON line: device time per call (CUDA events over --iters calls after warm-up, host planning included),
the FLOPs of the expert GEMMs (3 * 2 * H * I per route) and the achieved TFLOP/s.
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--tokens', type=int, default=2048)
    ap.add_argument('--hidden', type=int, default=2048)
    ap.add_argument('--inter', type=int, default=768)
    ap.add_argument('--experts', type=int, default=128)
    ap.add_argument('--top-k', type=int, default=8)
    ap.add_argument('--fmt', default='nvfp4')
    ap.add_argument('--iters', type=int, default=10)
    a = ap.parse_args(argv)
    from .. import formats, ops
    from ..cache.prefill import grouped_experts
    ops.load()
    dev = 'cuda'
    g = torch.Generator(device=dev).manual_seed(0)
    ew = formats.synthetic_experts(a.experts, a.hidden, a.inter, a.fmt, dev)
    ew.g13 = ew.g13.float()
    ew.g2 = ew.g2.float()
    x = torch.randn(a.tokens, a.hidden, device=dev, generator=g).bfloat16()
    scores = torch.rand(a.tokens, a.experts, device=dev, generator=g)
    slots = scores.topk(a.top_k, -1).indices.int()
    w = torch.rand(a.tokens, a.top_k, device=dev, generator=g)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    for _ in range(2):
        grouped_experts(x, slots, w, ew, err)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.iters):
        grouped_experts(x, slots, w, ew, err)
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) / a.iters * 1e3
    flops = 2.0 * 3 * a.hidden * a.inter * a.tokens * a.top_k
    print(json.dumps(dict(tool='prefill_bench', tokens=a.tokens, hidden=a.hidden, inter=a.inter, experts=a.experts,
                          top_k=a.top_k, fmt=a.fmt, us=round(us, 1), tflops=round(flops / us / 1e6, 1),
                          error_word=int(err))), flush=True)


if __name__ == '__main__':
    main()
