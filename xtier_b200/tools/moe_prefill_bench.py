"""Prefill MoE layer timings on one GPU: the exact W4A16 grouped path, the block-scaled MXFP4 x MXFP8 path (both
this framework's tcgen05 kernels, the whole call: routing plan, gather, both GEMMs, route-ordered combine) and,
with --flashinfer, FlashInfer's CUTLASS fused MoE in its MXFP4 x MXFP8 mode (the library the reference's prefill
calls) on the same experts and routes. Device time per call from CUDA events after warm-up; one JSON line per
(shape, tokens, arm) with TFLOP/s over the routed work (tokens x top-k x 3 GEMMs of H x I).

    python -m xtier_b200.tools.moe_prefill_bench [--shapes deepseek,qwen3] [--tokens 2048,16384,65536] [--flashinfer]
                                                [--arms w4a16,mx] [--experts E]
"""
from __future__ import annotations

import argparse
import json
import os

import torch

SHAPES = {'deepseek': dict(H=7168, I=2048, E=256, k=8), 'qwen3': dict(H=2048, I=768, E=128, k=8)}


def _time(fn, iters=3):
    for _ in range(2):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3


def _flashinfer_arm(x, ids, w, pool):
    """FlashInfer cutlass_fused_moe, MXFP8 activations x MXFP4 weights (scales interleaved by the library's own
    helper): returns a closure running one call, or raises with the reason it cannot run."""
    from flashinfer import block_scale_interleave, mxfp8_quantize
    from flashinfer.fused_moe import cutlass_fused_moe
    E = pool.experts
    w13 = pool.w13.contiguous().view(torch.int64)
    w2 = pool.w2.contiguous().view(torch.int64)
    s13 = block_scale_interleave(pool.s13.contiguous()).reshape_as(pool.s13).view(torch.int32)
    s2 = block_scale_interleave(pool.s2.contiguous()).reshape_as(pool.s2).view(torch.int32)
    ones = torch.ones(E, dtype=torch.float32, device=x.device)
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)

    def run():
        xq, xsf = mxfp8_quantize(x, is_sf_swizzled_layout=True, alignment=32)
        cutlass_fused_moe(input=xq, token_selected_experts=ids, token_final_scales=w, fc1_expert_weights=w13,
                          fc2_expert_weights=w2, output_dtype=torch.bfloat16, quant_scales=[s13, ones, s2, ones],
                          input_sf=xsf, use_mxfp8_act_scaling=True, output=out,
                          tune_max_num_tokens=max(8192, x.shape[0]))
        return out

    return run


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--shapes', default='deepseek,qwen3')
    ap.add_argument('--tokens', default='2048,16384,65536')
    ap.add_argument('--flashinfer', action='store_true')
    ap.add_argument('--arms', default='w4a16,mx')
    ap.add_argument('--experts', type=int, default=0, help='override the shape\'s expert count (small profiles)')
    a = ap.parse_args(argv)
    from .. import formats, ops
    from ..cache.prefill import grouped_experts
    ops.load()
    dev = torch.device('cuda')
    for name in a.shapes.split(','):
        sh = SHAPES[name]
        H, I, E, k = sh['H'], sh['I'], a.experts or sh['E'], sh['k']
        pool = formats.synthetic_experts(E, H, I, formats.MXFP4, dev, seed=1)
        for T in [int(t) for t in a.tokens.split(',')]:
            g = torch.Generator(device=dev).manual_seed(T)
            x = torch.randn(T, H, device=dev, generator=g).bfloat16()
            ids = torch.argsort(torch.rand(T, E, device=dev, generator=g), 1)[:, :k].int().contiguous()
            w = torch.rand(T, k, device=dev, generator=g)
            flops = 2.0 * T * k * 3 * H * I
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            for arm in a.arms.split(','):
                os.environ['XTIER_PREFILL_MX'] = '1' if arm == 'mx' else '0'
                us = _time(lambda: grouped_experts(x, ids, w, pool, err))
                print(json.dumps(dict(tool='moe_prefill_bench', shape=name, tokens=T, arm=arm, us=round(us, 1),
                                      tflops=round(flops / us / 1e6, 1), error_word=int(err))), flush=True)
                torch.cuda.empty_cache()
            os.environ.pop('XTIER_PREFILL_MX', None)
            if a.flashinfer:
                try:
                    run = _flashinfer_arm(x, ids, w, pool)
                    us = _time(run)
                    res = dict(us=round(us, 1), tflops=round(flops / us / 1e6, 1))
                except Exception as e:   # the library's API or build differs: report, do not stop
                    res = dict(unavailable=f'{type(e).__name__}: {str(e)[:160]}')
                print(json.dumps(dict(tool='moe_prefill_bench', shape=name, tokens=T, arm='flashinfer_cutlass_mxfp8',
                                      **res)), flush=True)
                torch.cuda.empty_cache()
            del x, ids, w


if __name__ == '__main__':
    main()
