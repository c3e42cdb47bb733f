"""Miss share (XTIER_DECODE_MISS_GPU): a token's first CPU-tier route is computed on the GPU from the pinned host
copy of the expert (PCIe loads inside the decode expert kernels) and skipped by the CPU engine; the layer output
matches the fp32 reference, eager and replayed from a CUDA graph."""
import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def test_miss_share_matches_reference(cuda_ops, monkeypatch):
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    monkeypatch.setenv('XTIER_DECODE_MISS_GPU', '0.5')      # one shared route per token with any CPU route
    E, H, I, k = 16, 1024, 512, 4
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=8, std=0.05)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(9)) * 0.02).bfloat16()
    bias = torch.zeros(E)
    bias[[10, 11, 12, 13]] = 4.0                              # most routes go to CPU-tier experts
    mb = Mailbox(H, timeout_s=10.0)
    eng = CpuEngine(ex, threads=2)
    layer = TieredMoE(0, router, ex, k, hot=[0, 1, 2, 3], router_bias=bias, mailbox=mb, engine=eng, device='cuda',
                      host_experts=ex)
    layer.prepare_prefill()
    assert layer.host_table is not None and layer.share_min == 1
    mb.start()
    try:
        x = torch.randn(3, H, generator=torch.Generator().manual_seed(1)).bfloat16().cuda()
        out = layer.forward(x)
        torch.cuda.synchronize()
        mb.check()
        slots = layer.slots[:3, :k].cpu()
        assert int((slots >= layer.HOST_BASE).sum()) == 3     # one shared route per token
        ids, w = layer.ids[:3, :k].cpu(), layer.w[:3, :k].cpu()
        ref = formats.reference_moe(x.cpu(), ids, w, ex)
        rel = float((out.cpu().float() - ref).norm() / ref.norm())
        assert rel < 1e-2, rel
        # graph replays
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        out_g = torch.empty_like(out)
        with torch.cuda.stream(s):
            layer.forward(x, out=out_g)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer.forward(x, out=out_g)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        mb.check()
        rel_g = float((out_g.cpu().float() - ref).norm() / ref.norm())
        assert rel_g < 1e-2, rel_g
        del g
    finally:
        mb.stop()
        mb.close()
