"""Adaptive residency on the GPU: a layer that starts with its least routed experts hot moves the most routed ones in
after a few decode calls, and its output still matches the fp32 reference afterwards."""
import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def test_policy_swaps_toward_routed_experts(cuda_ops):
    from xtier_b200.cache.policy import AdaptivePolicy
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    E, H, I, k = 16, 512, 256, 2
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=21, std=0.05)
    router = (torch.randn(E, H) * 0.02).bfloat16()
    bias = torch.zeros(E)
    bias[:4] = 6.0   # experts 0..3 take almost every route
    mb = Mailbox(H, timeout_s=10.0)
    eng = CpuEngine(ex, threads=2)
    layer = TieredMoE(0, router, ex, k, hot=[12, 13, 14, 15], router_bias=bias, mailbox=mb, engine=eng,
                      device='cuda', host_experts=ex)
    mb.start(decay=0.9)
    try:
        pol = AdaptivePolicy([layer], mb, every=1, swaps=8, min_gain=1.5)
        x = torch.randn(2, H).bfloat16().cuda()
        for _ in range(4):
            layer.forward(x)
        torch.cuda.synchronize()
        mb.check()
        n = pol.step()
        assert n >= 2
        assert {0, 1, 2, 3} & set(layer.resident())
        out = layer.forward(x)
        torch.cuda.synchronize()
        mb.check()
        ids, w = layer.ids[:2].cpu(), layer.w[:2].cpu()
        ref = formats.reference_moe(x.cpu(), ids, w, ex)
        assert float((out.cpu().float() - ref).norm() / ref.norm()) < 1e-2
        # the table and the resident list agree
        tab = layer.table.cpu()
        for s, e in enumerate(layer.resident()):
            assert int(tab[e]) == s
    finally:
        mb.stop()
        mb.close()
