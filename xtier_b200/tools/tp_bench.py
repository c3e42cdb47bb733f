"""Fused tensor-parallel GEMMs against their NCCL baselines: GEMM -> reduce-scatter (row-parallel linear) and
all-gather -> GEMM (column-parallel linear), on a sequence-parallel MLP's shapes.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m xtier_b200.tools.tp_bench [--tokens 8192] [--hidden 8192] [--inter 28672]

gemm_rs: a [M, I/W] x w2 [H, I/W] -> rows M/W of [M, H]. ag_gemm: x [M/W, H] gathered -> x w13 [2I/W, H]^T.
Times are CUDA-event device times over `--iters` calls after warm-up, between a barrier and a synchronize, max over
ranks. Also prints the roofline target per op: the slower of FLOPs / --peak-tflops and NVLink bytes / --link-gbs.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--tokens', type=int, default=8192)
    ap.add_argument('--hidden', type=int, default=8192)
    ap.add_argument('--inter', type=int, default=28672)
    ap.add_argument('--iters', type=int, default=20)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--peak-tflops', type=float, default=1590.0)
    ap.add_argument('--link-gbs', type=float, default=770.0)
    ap.add_argument('--iters-only', action='store_true', help='fused ops only (no NCCL baseline): a single GPU')
    a = ap.parse_args(argv)
    from .. import ops
    from ..parallel import dist as xdist
    from ..parallel.tp import TPComm, nccl_ag_gemm, nccl_gemm_rs
    env = xdist.init(timeout_s=120)
    ops.load()
    W, r, dev = env.world, env.rank, env.device
    M, H, I = a.tokens, a.hidden, a.inter
    Il = I // W
    g = torch.Generator(device=dev).manual_seed(r)
    act = torch.randn(M, Il, device=dev, generator=g).bfloat16()
    w2 = (torch.randn(H, Il, device=dev, generator=g) * 0.02).bfloat16()
    x = torch.randn(M // W, H, device=dev, generator=g).bfloat16()
    w13 = (torch.randn(2 * Il, H, device=dev, generator=g) * 0.02).bfloat16()
    comm = TPComm(M * max(H, 2 * Il), M, dev, timeout_s=10.0)
    o_rs = torch.empty(M // W, H, dtype=torch.bfloat16, device=dev)
    o_ag = torch.empty(M, 2 * Il, dtype=torch.bfloat16, device=dev)

    def timed(fn):
        for _ in range(a.warmup):
            fn()
        xdist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        xdist.barrier()
        t = torch.tensor([s.elapsed_time(e) / a.iters * 1e3], dtype=torch.float64, device=dev)
        if W > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    res = dict(tool='tp_bench', world=W, tokens=M, hidden=H, inter=I)
    fl_rs = 2.0 * M * H * Il
    link_rs = (W - 1) / W * M * H * 2
    fl_ag = 2.0 * M * 2 * Il * H
    link_ag = (W - 1) / W * M * H * 2
    for name, fused, base, fl, link in (
            ('gemm_rs', lambda: comm.gemm_rs(act, w2, out=o_rs), lambda: nccl_gemm_rs(act, w2), fl_rs, link_rs),
            ('ag_gemm', lambda: comm.ag_gemm(x, w13, out=o_ag), lambda: nccl_ag_gemm(x, w13), fl_ag, link_ag)):
        tf = timed(fused)
        tb = timed(base) if (W > 1 and not a.iters_only) else float('nan')
        target = max(fl / (a.peak_tflops * 1e12), link / (a.link_gbs * 1e9)) * 1e6
        res[name] = dict(fused_us=round(tf, 1), nccl_us=round(tb, 1) if tb == tb else None, speedup=round(tb / tf, 3) if tb == tb else None,
                         roofline_us=round(target, 1), of_roofline=round(target / tf, 3),
                         tflops=round(fl / tf / 1e6, 1))
    # the same GEMMs alone (this rank's shard, no collective), for the overhead of the fused exchange
    res['gemm_rs']['gemm_only_us'] = round(timed(lambda: ops.gemm(act, w2)), 1)
    xfull = torch.cat([x] * W)
    res['ag_gemm']['gemm_only_us'] = round(timed(lambda: ops.gemm(xfull, w13)), 1)
    comm.check()
    if r == 0:
        print(json.dumps(res), flush=True)
    xdist.barrier()
    comm.close()
    if W > 1:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
