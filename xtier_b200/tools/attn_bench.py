"""Causal GQA prefill attention: this framework's tcgen05 kernel (ops.attn_prefill) against PyTorch's fused
scaled_dot_product_attention (cuDNN / flash backends) on the same B200, Qwen3-30B-A3B heads (32 query heads, 4 KV heads,
head dim 128). Device time by CUDA events over `reps` calls after warm-up; TFLOP/s counts the causal half
(2 products x 2 flops x T (T + 1) / 2 x 128 x heads).

    python -m xtier_b200.tools.attn_bench [--tokens 4096,16384,65536] [--heads 32] [--kv-heads 4]
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def _time_ms(fn, reps: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--tokens', default='4096,16384,65536')
    ap.add_argument('--heads', type=int, default=32)
    ap.add_argument('--kv-heads', type=int, default=4)
    ap.add_argument('--reps', type=int, default=5)
    ap.add_argument('--no-sdpa', action='store_true')
    a = ap.parse_args(argv)
    from .. import ops
    ops.load()
    Hq, Hkv, D = a.heads, a.kv_heads, 128
    scale = 1.0 / math.sqrt(D)
    F = torch.nn.functional
    for T in [int(t) for t in a.tokens.split(',')]:
        k = torch.randn(1, Hkv, T, D, device='cuda').bfloat16()
        v = torch.randn(1, Hkv, T, D, device='cuda').bfloat16()
        q = torch.randn(T, Hq, D, device='cuda').bfloat16()
        out = torch.empty_like(q)
        flops = 4.0 * T * (T + 1) / 2 * D * Hq
        err = ops.gemm_error_word(q.device)
        err.zero_()
        ours = _time_ms(lambda: ops.attn_prefill(q, k, v, 0, 0, scale, out=out), a.reps)
        r = dict(tool='attn_bench', tokens=T, heads=Hq, kv_heads=Hkv, ours_ms=round(ours, 3),
                 ours_tflops=round(flops / ours / 1e9, 1), err=int(err.item()))
        if not a.no_sdpa:
            qq = q.transpose(0, 1).unsqueeze(0)
            sd = _time_ms(lambda: F.scaled_dot_product_attention(qq, k, v, is_causal=True, enable_gqa=True), a.reps)
            ref = F.scaled_dot_product_attention(qq, k, v, is_causal=True, enable_gqa=True)[0].transpose(0, 1)
            r.update(sdpa_ms=round(sd, 3), sdpa_tflops=round(flops / sd / 1e9, 1),
                     rel_diff=float('%.3g' % float((out.float() - ref.float()).norm() / ref.float().norm())))
        print(json.dumps(r), flush=True)
        del k, v, q, out


if __name__ == '__main__':
    main()
