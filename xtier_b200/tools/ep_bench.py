"""Expert-parallel MoE layer benchmark: the fused NVLink path (one graph-captured call: peer-store dispatch, expert
kernels, peer-store return, ordered combine) against the NCCL baseline (all_to_all_single of the routed rows, the same
expert kernels, all_to_all_single back), one MoE layer of the DeepSeek-V3 shape by default.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m xtier_b200.tools.ep_bench [--tokens 4] [--hidden 7168] [--inter 2048] [--experts 256] [--top-k 8]

--tokens is per rank (32 concurrent requests over 8 ranks: 4). Times are CUDA-event device times of `--iters` calls
after warm-up, between a barrier and a synchronize, max over ranks; prints one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--tokens', type=int, default=4)
    ap.add_argument('--hidden', type=int, default=7168)
    ap.add_argument('--inter', type=int, default=2048)
    ap.add_argument('--experts', type=int, default=256)
    ap.add_argument('--top-k', type=int, default=8)
    ap.add_argument('--fmt', default='mxfp4')
    ap.add_argument('--iters', type=int, default=50)
    ap.add_argument('--warmup', type=int, default=5)
    a = ap.parse_args(argv)
    from .. import formats, ops
    from ..parallel import dist as xdist
    from ..parallel.ep import EPComm, EPMoE, nccl_ep_moe
    env = xdist.init(timeout_s=120)
    ops.load()
    W, r = env.world, env.rank
    El = a.experts // W
    local = formats.synthetic_experts(El, a.hidden, a.inter, a.fmt, env.device, seed=r)
    router = (torch.randn(a.experts, a.hidden, generator=torch.Generator().manual_seed(5)) * 0.02).bfloat16()
    comm = EPComm(a.hidden, a.inter, a.experts, a.top_k, a.tokens, env.device, timeout_s=10.0)
    layer = EPMoE(0, comm, router, local, a.top_k, mode=1, n_group=8 if a.experts % 8 == 0 else 1,
                  topk_group=4 if a.experts % 8 == 0 else 1, scale=2.5)
    x = torch.randn(a.tokens, a.hidden, device=env.device).bfloat16()
    out = torch.empty_like(x)

    def timed(fn, iters):
        xdist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        xdist.barrier()
        t = torch.tensor([s.elapsed_time(e) / iters * 1e3], dtype=torch.float64, device=env.device)
        if W > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    # fused: graph-captured
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        for _ in range(a.warmup):
            layer.forward(x, out=out)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        layer.forward(x, out=out)
    for _ in range(a.warmup):
        g.replay()
    fused_us = timed(g.replay, a.iters)
    comm.check()
    # NCCL baseline (eager; routing included as in the fused call)
    def base():
        ids, w = layer.router(x)
        nccl_ep_moe(x, ids, w, layer.local, a.experts)
    for _ in range(a.warmup):
        base()
    nccl_us = timed(base, a.iters)
    res = dict(tool='ep_bench', world=W, tokens_per_rank=a.tokens, hidden=a.hidden, inter=a.inter,
               experts=a.experts, top_k=a.top_k, fmt=a.fmt, fused_us=round(fused_us, 2), nccl_us=round(nccl_us, 2),
               speedup=round(nccl_us / fused_us, 2))
    if r == 0:
        print(json.dumps(res), flush=True)
    del g
    xdist.barrier()
    comm.close()
    if W > 1:
        dist.destroy_process_group()


if __name__ == '__main__':
    main()
