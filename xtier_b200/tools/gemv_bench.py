"""Decode projection GEMMs (M tokens x weight [N, K] BF16): the CUDA-core weight-streaming GEMV against the tcgen05
skinny GEMM, device time per call from CUDA-graph replays and the weight bandwidth each reaches.

    python -m xtier_b200.tools.gemv_bench [--rows 1,4,8,32]
"""
from __future__ import annotations

import argparse
import json

import torch

SHAPES = {'qkv_a': (2112, 7168), 'q_b': (24576, 1536), 'o_proj': (7168, 16384), 'idx_q': (8192, 1536),
          'dense_gate_up': (36864, 7168), 'dense_down': (7168, 18432), 'lm_head': (129280, 7168)}


def _time(fn, iters=20):
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
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
    ap.add_argument('--rows', default='1,4,8,32')
    a = ap.parse_args(argv)
    from .. import ops
    ops.load()
    for name, (N, K) in SHAPES.items():
        w = torch.randn(N, K, device='cuda').bfloat16()
        for M in [int(v) for v in a.rows.split(',')]:
            x = torch.randn(M, K, device='cuda').bfloat16()
            y = torch.empty(M, N, dtype=torch.bfloat16, device='cuda')
            res = dict(tool='gemv_bench', shape=name, M=M, N=N, K=K)
            if M <= 16 and M * K * 2 <= 200 * 1024:
                res['gemv_us'] = round(_time(lambda: ops.gemv(x, w, y)), 1)
            res['skinny_us'] = round(_time(lambda: ops.skinny_gemm(x, w, y)), 1)
            res['skinny_weight_tbs'] = round(N * K * 2 / res['skinny_us'] / 1e6, 2)
            print(json.dumps(res), flush=True)
        del w


if __name__ == '__main__':
    main()
