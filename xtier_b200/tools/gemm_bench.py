"""BF16 GEMM microbenchmark: the tcgen05 kernel (`torch.ops.xtier.gemm_tc`) against torch.matmul (cuBLAS) on the same
operands, D[M, N] = A[M, K] . B[N, K]^T.

    python -m xtier_b200.tools.gemm_bench [--shapes 8192x8192x8192,4096x7168x2304] [--iters 20]

Times are CUDA-event device times of --iters back-to-back calls after 3 warm-up calls (operands of these shapes are
larger than L2 or reused as a GEMM reuses them); prints one JSON line per shape with TFLOP/s, the ratio to cuBLAS and
the relative error against an fp32 matmul. XTIER_GEMM_PAIR=1 selects the CTA-pair kernel. --mx8 adds the
block-scaled FP8 GEMM (`ops.linear_mx8`: the GEMM alone on pre-quantized activations, and with the per-call
activation quantization) on the same shapes.
"""
from __future__ import annotations

import argparse
import json

import torch


def _time(fn, iters):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters * 1e3


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--shapes', default='8192x8192x8192,4096x4096x4096,2048x5120x2048,16384x7168x2048')
    ap.add_argument('--iters', type=int, default=20)
    ap.add_argument('--no-cublas', action='store_true')
    ap.add_argument('--mx8', action='store_true', help='also the MXFP8 GEMM (tcgen05 kind::mxf8f6f4)')
    a = ap.parse_args(argv)
    from .. import ops
    ops.load()
    for shp in a.shapes.split(','):
        M, N, K = (int(v) for v in shp.lower().split('x'))
        A = torch.randn(M, K, device='cuda').bfloat16()
        B = (torch.randn(N, K, device='cuda') * K ** -0.5).bfloat16()
        out = torch.empty(M, N, device='cuda', dtype=torch.bfloat16)
        err = ops.gemm_error_word(A.device)
        us = _time(lambda: torch.ops.xtier.gemm_tc(A, B, None, out, err), a.iters)
        ref = A.float() @ B.float().t()
        rel = float((out.float() - ref).norm() / ref.norm())
        del ref
        fl = 2.0 * M * N * K
        res = dict(tool='gemm_bench', M=M, N=N, K=K, us=round(us, 1), tflops=round(fl / us / 1e6, 1),
                   rel_err=round(rel, 5), error_word=int(err))
        if not a.no_cublas:
            ub = _time(lambda: torch.matmul(A, B.t(), out=out), a.iters)
            res.update(cublas_us=round(ub, 1), cublas_tflops=round(fl / ub / 1e6, 1), vs_cublas=round(ub / us, 3))
        if a.mx8:
            wq = ops.MX8Weight(B)
            x8 = torch.empty(M, K, dtype=torch.uint8, device='cuda')
            sfx = torch.empty(M * K // 32, dtype=torch.uint8, device='cuda')
            torch.ops.xtier.mx_quant_rows(A, None, x8, sfx)
            um = _time(lambda: torch.ops.xtier.gemm_mx8(x8, sfx, M, wq.w8, wq.sf, None, out, err), a.iters)
            uq = _time(lambda: ops.linear_mx8(A, wq, out=out), a.iters)
            ref = A.float() @ B.float().t()
            relm = float((out.float() - ref).norm() / ref.norm())
            del ref
            res.update(mx8_us=round(um, 1), mx8_tflops=round(fl / um / 1e6, 1), mx8_with_quant_us=round(uq, 1),
                       mx8_rel_err=round(relm, 4))
        print(json.dumps(res), flush=True)


if __name__ == '__main__':
    main()
