"""Expert parallelism over NVLink peer memory on 2+ GPUs (one process per GPU): the fused EP MoE against the fp32
reference of the same routes and against the NCCL all-to-all baseline, eager and replayed from a CUDA graph."""
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


def _worker(rank, world, port, q, fmt_name, H, I, E, k, T):
    try:
        sys.path.insert(0, ROOT)
        os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR='127.0.0.1',
                          MASTER_PORT=str(port), NCCL_NVLS_ENABLE='0')
        from xtier_b200 import formats, ops
        from xtier_b200.parallel import dist as xdist
        from xtier_b200.parallel.ep import EPComm, EPMoE, nccl_ep_moe
        env = xdist.init(timeout_s=60)
        ops.load()
        ex = formats.random_experts(E, H, I, fmt_name, seed=11, std=0.05)
        El = E // world
        local = ex.select(torch.arange(rank * El, (rank + 1) * El))
        router = (torch.randn(E, H, generator=torch.Generator().manual_seed(12)) * 0.02).bfloat16()
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(100 + rank)).bfloat16()
        comm = EPComm(H, I, E, k, T, env.device, timeout_s=5.0)
        layer = EPMoE(0, comm, router, local, k)
        xd = x.to(env.device)
        out = layer.forward(xd)
        torch.cuda.synchronize()
        comm.check()
        ids, w = layer.router.ids[:T].cpu(), layer.router.wt[:T].cpu()
        ref = formats.reference_moe(x, ids, w, ex)
        rel = float((out.cpu().float() - ref).norm() / ref.norm())
        base = nccl_ep_moe(xd, layer.router.ids[:T], layer.router.wt[:T], layer.local, E)
        rel_nccl = float((base.cpu().float() - ref).norm() / ref.norm())
        # graph replays of the fused exchange
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        out_g = torch.empty_like(out)
        with torch.cuda.stream(s):
            layer.forward(xd, out=out_g)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer.forward(xd, out=out_g)
        same = True
        for _ in range(3):
            out_g.zero_()
            xdist.barrier()
            g.replay()
            torch.cuda.synchronize()
            same = same and torch.equal(out_g, out)
        comm.check()
        del g
        xdist.barrier()
        comm.close()
        q.put((rank, rel, rel_nccl, same, None))
        torch.distributed.destroy_process_group()
    except Exception as e:   # reported to the parent
        import traceback
        q.put((rank, None, None, None, traceback.format_exc()))


@pytest.mark.parametrize('fmt_name,H,I,E,k,T', [('nvfp4', 512, 256, 8, 2, 5), ('mxfp4', 1024, 512, 16, 4, 12)])
def test_ep_moe_two_gpus(fmt_name, H, I, E, k, T):
    if torch.cuda.device_count() < 2:
        pytest.skip('needs 2 GPUs')
    import torch.multiprocessing as mp
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, fmt_name, H, I, E, k, T)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, rel, rel_nccl, same, err in results:
        assert err is None, err
        assert rel < 1e-2, (rank, rel)
        assert rel_nccl < 1e-2, (rank, rel_nccl)
        assert same, rank


@pytest.mark.parametrize('fmt_name,H,I,E,k,T', [('mxfp4', 7168, 2048, 16, 8, 4), ('nvfp4', 2048, 768, 32, 8, 3),
                                                ('nvfp4', 4096, 1536, 8, 4, 2)])
def test_ep_moe_one_gpu_shapes(fmt_name, H, I, E, k, T):
    """The fused EP op at world size 1 (no process group; the peer table holds this GPU's own buffer) on
    DeepSeek-V3 / Qwen3 expert shapes: exercises every K split of the streaming expert kernels."""
    from xtier_b200 import formats, ops
    from xtier_b200.parallel import dist as xdist
    from xtier_b200.parallel.ep import EPComm, EPMoE
    for v in ('RANK', 'WORLD_SIZE', 'LOCAL_RANK'):
        os.environ.pop(v, None)
    env = xdist.init(timeout_s=60)
    ops.load()
    ex = formats.random_experts(E, H, I, fmt_name, seed=3, std=0.05)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(4)) * 0.02).bfloat16()
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(5)).bfloat16()
    comm = EPComm(H, I, E, k, T, env.device, timeout_s=5.0)
    layer = EPMoE(0, comm, router, ex, k)
    out = layer.forward(x.to(env.device))
    torch.cuda.synchronize()
    comm.check()
    ref = formats.reference_moe(x, layer.router.ids[:T].cpu(), layer.router.wt[:T].cpu(), ex)
    rel = float((out.cpu().float() - ref).norm() / ref.norm())
    comm.close()
    assert rel < 1e-2, rel
