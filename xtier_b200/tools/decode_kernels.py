"""Device time of the decode-step kernels of the flagship shape in isolation (hidden 2048, GQA 32/4
with head dim 128, 128 experts top-8): GQA decode attention at several context lengths and split counts, and the
router (8-CTA cluster per token), and the hot-expert gate/up and down kernels of one token's 8 routes.

    python -m xtier_b200.tools.decode_kernels [--contexts 2084,8000,32768] [--iters 48]

Each measurement captures `--iters` calls in a CUDA graph and divides one replay's CUDA-event time by `--iters`
(back-to-back calls, device time, no host launch cost). Prints one JSON line. `--once` runs each kernel a few times
without timing (the small case for an ncu capture).
"""
from __future__ import annotations

import argparse
import json

import torch


def _graph_us(fn, iters: int) -> float:
    for _ in range(3):
        fn()
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
    del g
    return a.elapsed_time(b) / iters * 1e3


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--contexts', default='2084,8000,32768')
    ap.add_argument('--iters', type=int, default=48)
    ap.add_argument('--once', action='store_true')
    a = ap.parse_args(argv)
    from .. import formats, ops
    from ..cache.pool import TieredMoE
    ops.load()
    res = {'tool': 'decode_kernels'}
    B, Hq, Hkv, D = 1, 32, 4, 128
    G = Hq // Hkv
    g = torch.Generator(device='cuda').manual_seed(0)
    for n in [int(x) for x in a.contexts.split(',')]:
        L = n + 128
        k = torch.randn(B, Hkv, L, D, device='cuda', generator=g).bfloat16()
        v = torch.randn(B, Hkv, L, D, device='cuda', generator=g).bfloat16()
        q = torch.randn(B, Hq, D, device='cuda', generator=g).bfloat16()
        splits = ops.attn_decode_splits(B, Hkv, L)
        ws_o = torch.empty(B * Hkv * splits * G * D, device='cuda')
        ws_ml = torch.empty(B * Hkv * splits * G * 2, device='cuda')
        cnt = torch.zeros(B * Hkv, dtype=torch.int32, device='cuda')
        sl = torch.full((B,), n, dtype=torch.int32, device='cuda')
        out = torch.empty(B, Hq, D, device='cuda').bfloat16()
        f = lambda: ops.attn_decode(q, k, v, sl, out, ws_o, ws_ml, cnt, splits, D ** -0.5)
        if a.once:
            for _ in range(3):
                f()
            continue
        us = _graph_us(f, a.iters)
        kv_bytes = 2 * B * Hkv * n * D * 2
        res[f'attn_ctx{n}'] = dict(splits=splits, us=round(us, 2), kv_gbs=round(kv_bytes / us / 1e3, 1))
    E, H, I, k_ = 128, 2048, 768, 8
    ex = formats.synthetic_experts(E, H, I, 'nvfp4', 'cuda', seed=1)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(1)) * 0.02).bfloat16()
    layer = TieredMoE(0, router, ex, k_, router_bias=torch.linspace(2, -2, E), device='cuda')
    x = torch.randn(1, H, generator=torch.Generator().manual_seed(2)).bfloat16().cuda()
    fr = lambda: layer.route(x, False)
    if a.once:
        for _ in range(3):
            fr()
        torch.cuda.synchronize()
        print('ok')
        return
    res['route_m1_us'] = round(_graph_us(fr, a.iters), 2)
    # the hot experts of one token (8 routes, all on this GPU): gate/up and down on the routes above
    layer.route(x, False)
    out = torch.empty_like(x)
    fg = lambda: ops.moe_gate_up(x, layer.slots[:1], layer.pool.w13, layer.pool.s13, layer.pool.g13,
                                 layer.mid[:k_], 0)
    fd = lambda: ops.moe_down(layer.mid[:k_], layer.slots[:1], layer.w[:1], layer.pool.w2, layer.pool.s2,
                              layer.pool.g2, None, out, None, 0)
    gu_us, dn_us = _graph_us(fg, a.iters), _graph_us(fd, a.iters)
    res['gate_up_us'] = round(gu_us, 2)
    res['down_us'] = round(dn_us, 2)
    res['gate_up_gbs'] = round(k_ * 2 * I * H * (0.5 + 1 / 16) / gu_us / 1e3, 1)
    res['down_gbs'] = round(k_ * H * I * (0.5 + 1 / 16) / dn_us / 1e3, 1)
    res['moe_layer_us'] = round(_graph_us(lambda: layer.forward(x, out=out), a.iters), 2)
    print(json.dumps(res), flush=True)


if __name__ == '__main__':
    main()
