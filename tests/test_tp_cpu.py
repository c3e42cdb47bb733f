"""Tensor parallelism of the CPU tier without GPUs: each rank's engine holds its slice of every expert's intermediate
units, in its own process; the ranks' outputs summed with a gloo all-reduce equal the whole engine's (and each slice
dequantizes to the matching rows / columns of the whole expert)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from xtier_b200 import formats

H, I, E = 256, 256, 8


def _experts(fmt):
    return formats.random_experts(E, H, I, fmt, seed=3)


@pytest.mark.parametrize('fmt', [formats.NVFP4, formats.MXFP4])
def test_slices_dequantize_to_the_whole(fmt):
    ew = _experts(fmt)
    w1, w3, w2 = ew.dequant(5)
    for r in range(2):
        s = ew.tp_slice(r, 2)
        a1, a3, a2 = s.dequant(5)
        n = I // 2
        assert torch.equal(a1, w1[r * n:(r + 1) * n]) and torch.equal(a3, w3[r * n:(r + 1) * n])
        assert torch.equal(a2, w2[:, r * n:(r + 1) * n])
    with pytest.raises(ValueError):
        ew.tp_slice(0, 3)


def _worker(rank, world, port, fmt, q):
    import torch.distributed as dist
    from xtier_b200.engine import CpuEngine
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    ew = _experts(fmt)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, H, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, generator=g)[:3] for _ in range(5)]).int()
    w = torch.rand(5, 3, generator=g)
    eng = CpuEngine(ew.tp_slice(rank, world), threads=2)
    part = eng.forward(x, ids, w).float()
    eng.close()
    dist.all_reduce(part)
    q.put((rank, part))
    dist.destroy_process_group()


@pytest.mark.parametrize('fmt', [formats.NVFP4, formats.MXFP4])
def test_two_rank_cpu_tier_sums_to_the_whole_engine(fmt):
    from xtier_b200.engine import CpuEngine
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, fmt, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted([q.get(timeout=120) for _ in ps], key=lambda t: t[0])
    for p in ps:
        p.join(timeout=30)
    ew = _experts(fmt)
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, H, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, generator=g)[:3] for _ in range(5)]).int()
    w = torch.rand(5, 3, generator=g)
    full = CpuEngine(ew, threads=2)
    want = full.forward(x, ids, w).float()
    full.close()
    assert torch.equal(res[0][1], res[1][1])
    assert torch.allclose(res[0][1], want, rtol=1e-4, atol=1e-6)
