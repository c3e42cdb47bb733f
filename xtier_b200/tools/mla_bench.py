"""MLA decode attention benchmark on the DeepSeek-V3 shape (128 heads, latent 512 + rotary 64, NVFP4 latent cache):
one layer's attention step -- indexer scores + top-k (sparse mode) + the attention -- timed with CUDA events over
--iters calls captured in a CUDA graph (device time, no host launch cost). The attention is timed twice: the one-pass
tcgen05 kernel (mla_flash: gather into shared memory, online softmax, O in TMEM) and the three-kernel form
(mla_decode: gather to global BF16 tiles, attend per 128-key block, merge). --prefill Q times Q queries of one
sequence each attending its own top-k (the shape of one 64K prefill chunk).

    python -m xtier_b200.tools.mla_bench [--batch 1] [--context 32768] [--topk 2048]   # sparse (DSA)
    python -m xtier_b200.tools.mla_bench --batch 32 --context 4096 --topk 0             # dense over the context

Prints one JSON line: microseconds per step for the indexer, the top-k and the attention, the attention's achieved
TFLOP/s (2 * 128 * selected * (576 + 512) per query) and the KV bytes read.
"""
from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters):
    """Device time of one call: `iters` calls captured in a CUDA graph (no host launch cost), replayed after warm-up."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--batch', type=int, default=1)
    ap.add_argument('--context', type=int, default=32768)
    ap.add_argument('--topk', type=int, default=2048, help='0: dense attention over the whole context')
    ap.add_argument('--iters', type=int, default=20)
    ap.add_argument('--prefill', type=int, default=0, help='Q queries over one sequence of --context keys (flash only)')
    a = ap.parse_args(argv)
    from .. import ops
    from ..attention import dsa
    from ..attention.mla import (FlashWorkspace, LatentCache, MlaWorkspace, default_scale, flash_splits, mla_decode,
                                 mla_flash)
    ops.load()
    if a.prefill:
        return _prefill(a)
    B, n = a.batch, a.context
    dev = 'cuda'
    g = torch.Generator(device=dev).manual_seed(0)
    lcache = LatentCache(B, n)
    lcache.write(torch.randn(B * n, 576, device=dev, generator=g).bfloat16(), torch.arange(B * n, device=dev))
    rows = torch.arange(B, device=dev)
    lens = torch.full((B,), n, dtype=torch.int32, device=dev)
    q = (torch.randn(B, 128, 576, device=dev, generator=g) * 0.5).bfloat16()
    res = dict(tool='mla_bench', batch=B, context=n, topk=a.topk)
    if a.topk:
        icache = dsa.IndexCache(B, n)
        icache.write(torch.randn(B * n, 128, device=dev, generator=g).bfloat16(), torch.arange(B * n, device=dev))
        qi = torch.randn(B, 64, 128, device=dev, generator=g).bfloat16()
        w = torch.rand(B, 64, device=dev, generator=g)
        scores = torch.empty(B, n, device=dev)
        res['indexer_us'] = round(_time(lambda: dsa.index_scores(qi, w, icache, rows, lens, out=scores), a.iters), 1)
        res['indexer_cuda_core_us'] = round(_time(lambda: dsa.index_scores(qi, w, icache, rows, lens, out=scores,
                                                                           tensor_cores=False), a.iters), 1)
        dsa.index_scores(qi, w, icache, rows, lens, out=scores)
        sel = torch.empty(B, a.topk, dtype=torch.int32, device=dev)
        res['topk_us'] = round(_time(lambda: dsa.topk(scores, a.topk, out=sel), a.iters), 1)
        slots = dsa.select_slots(scores, rows, a.topk, n)
        nsel = a.topk
    else:
        nsel = (n + 127) // 128 * 128
        pos = torch.arange(nsel, device=dev)
        slots = torch.where(pos < n, pos, torch.full_like(pos, -1))[None].repeat(B, 1)
        slots = torch.where(slots >= 0, slots + rows[:, None] * n, slots).int()
    ws = MlaWorkspace(B, nsel)
    out = torch.empty(B, 128, 512, dtype=torch.bfloat16, device=dev)
    us = _time(lambda: mla_decode(q, slots, lcache, ws, default_scale(), out=out), a.iters)
    flops = 2.0 * B * 128 * min(nsel, n) * (576 + 512)
    sp = flash_splits(B, nsel)
    fws = FlashWorkspace(B, sp)
    fus = _time(lambda: mla_flash(q, slots, lcache, default_scale(), sp, fws, out=out), a.iters)
    res.update(attention_us=round(us, 1), attention_tflops=round(flops / us / 1e6, 1),
               flash_us=round(fus, 1), flash_tflops=round(flops / fus / 1e6, 1), flash_splits=sp,
               kv_bytes=int(B * min(nsel, n) * 416), error_word=int(ws.err), flash_error_word=int(fws.err))
    print(json.dumps(res), flush=True)


def _prefill(a):
    from ..attention.mla import FlashWorkspace, LatentCache, default_scale, mla_flash
    dev = 'cuda'
    Q, n, k = a.prefill, a.context, a.topk or 2048
    g = torch.Generator(device=dev).manual_seed(0)
    lcache = LatentCache(1, n)
    lcache.write(torch.randn(n, 576, device=dev, generator=g).bfloat16(), torch.arange(n, device=dev))
    q = (torch.randn(Q, 128, 576, device=dev, generator=g) * 0.5).bfloat16()
    slots = torch.stack([torch.randperm(n, device=dev, generator=g)[:k] for _ in range(Q)]).int()
    ws = FlashWorkspace(Q, 1)
    out = torch.empty(Q, 128, 512, dtype=torch.bfloat16, device=dev)
    us = _time(lambda: mla_flash(q, slots, lcache, default_scale(), 1, ws, out=out), a.iters)
    flops = 2.0 * Q * 128 * k * (576 + 512)
    print(json.dumps(dict(tool='mla_bench', prefill_queries=Q, context=n, topk=k, flash_us=round(us, 1),
                          flash_tflops=round(flops / us / 1e6, 1), error_word=int(ws.err))), flush=True)


if __name__ == '__main__':
    main()
