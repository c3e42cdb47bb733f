"""Tensor parallelism with the collective fused into the tcgen05 GEMM, on 2 GPUs (one process per GPU): GEMM ->
reduce-scatter and all-gather -> GEMM against the fp32 reference and the NCCL baselines, ragged N tiles, residual,
back-to-back calls (parity double buffering) and CUDA-graph replays."""
import os
import socket
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rel(a, b):
    return float((a.float().cpu() - b.float().cpu()).norm() / b.float().cpu().norm())


def _worker(rank, world, port, q, M, N, K):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR='127.0.0.1',
                          MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
        from xtier_b200.parallel import dist as xdist
        from xtier_b200.parallel.tp import TPComm, TPMLP, nccl_ag_gemm, nccl_gemm_rs
        env = xdist.init(timeout_s=60)
        dev = env.device
        g = torch.Generator().manual_seed(7)
        # full problem, identical on every rank; each rank takes its shards
        A = torch.randn(M, K, generator=g).bfloat16()
        B = (torch.randn(N, K, generator=g) * 0.05).bfloat16()
        R = torch.randn(M, N, generator=g).bfloat16()
        Kr, Mo = K // world, M // world
        H, I = K, 2 * N
        Il = I // world
        comm = TPComm(M * max(N, K, 2 * Il), M, dev, timeout_s=5.0)
        res = {}
        # GEMM -> RS: K split
        a = A[:, rank * Kr:(rank + 1) * Kr].contiguous().to(dev)
        b = B[:, rank * Kr:(rank + 1) * Kr].contiguous().to(dev)
        resid = R[rank * Mo:(rank + 1) * Mo].contiguous().to(dev)
        ref_rs = (A.float() @ B.float().t())[rank * Mo:(rank + 1) * Mo] + R[rank * Mo:(rank + 1) * Mo].float()
        outs = [comm.gemm_rs(a, b, residual=resid) for _ in range(3)]   # back-to-back: both parities, twice
        torch.cuda.synchronize()
        comm.check()
        res['rs'] = max(_rel(o, ref_rs) for o in outs)
        res['rs_nccl'] = _rel(nccl_gemm_rs(a, b, residual=resid), ref_rs)
        # AG -> GEMM: rows split
        a_sh = A[rank * Mo:(rank + 1) * Mo].contiguous().to(dev)
        bf = B.to(dev)
        ref_ag = A.float() @ B.float().t()
        outs = [comm.ag_gemm(a_sh, bf) for _ in range(3)]
        torch.cuda.synchronize()
        comm.check()
        res['ag'] = max(_rel(o, ref_ag) for o in outs)
        res['ag_nccl'] = _rel(nccl_ag_gemm(a_sh, bf), ref_ag)
        # interleaved RS / AG calls replayed from one CUDA graph
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        o_rs = torch.empty(Mo, N, dtype=torch.bfloat16, device=dev)
        o_ag = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        with torch.cuda.stream(s):
            comm.gemm_rs(a, b, residual=resid, out=o_rs)
            comm.ag_gemm(a_sh, bf, out=o_ag)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            comm.gemm_rs(a, b, residual=resid, out=o_rs)
            comm.ag_gemm(a_sh, bf, out=o_ag)
        worst = 0.0
        for _ in range(3):
            o_rs.zero_()
            o_ag.zero_()
            graph.replay()
            torch.cuda.synchronize()
            worst = max(worst, _rel(o_rs, ref_rs), _rel(o_ag, ref_ag))
        comm.check()
        res['graph'] = worst
        # sequence-parallel MLP against its fp32 reference
        w1 = (torch.randn(I, H, generator=g) * 0.05).bfloat16()
        w3 = (torch.randn(I, H, generator=g) * 0.05).bfloat16()
        w2 = (torch.randn(H, I, generator=g) * 0.05).bfloat16()
        w13 = torch.cat([w1[rank * Il:(rank + 1) * Il], w3[rank * Il:(rank + 1) * Il]]).to(dev)
        mlp = TPMLP(comm, w13, w2[:, rank * Il:(rank + 1) * Il].contiguous().to(dev))
        y = mlp(a_sh)
        torch.cuda.synchronize()
        comm.check()
        Af = A.float()
        hf = torch.nn.functional.silu(Af @ w1.float().t()) * (Af @ w3.float().t())
        ref_mlp = (hf.bfloat16().float() @ w2.float().t())[rank * Mo:(rank + 1) * Mo]
        res['mlp'] = _rel(y, ref_mlp)
        del graph
        xdist.barrier()
        comm.close()
        q.put((rank, res, None))
        torch.distributed.destroy_process_group()
    except Exception:   # reported to the parent
        import traceback
        q.put((rank, None, traceback.format_exc()))


@pytest.mark.parametrize('M,N,K', [(256, 384, 512), (512, 2048 + 128, 1024)])
def test_tp_fused_two_gpus(M, N, K):
    if torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, M, N, K)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, res, err in results:
        assert err is None, err
        for key, v in res.items():
            assert v < 1e-2, (rank, key, v)
