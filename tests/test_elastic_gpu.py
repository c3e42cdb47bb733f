"""Elastic slots on the GPU: a VMM arena keeps its address while granules are mapped and unmapped, and a tiered layer
whose extra slots are grown, filled, released and grown again matches the fp32 reference at every stage (routes of a
released slot's expert fall back to the CPU engine)."""
import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def test_vmm_arena_map_unmap(cuda_ops):
    from xtier_b200.cache.elastic import VmmArena
    probe = VmmArena(1, 'cuda')
    g = probe.granule
    probe.close()
    a = VmmArena(3 * g, 'cuda')
    a.ensure(1)
    assert a.granules == 1
    t = a.tensor()
    base = t.data_ptr()
    t[:g].fill_(7)
    a.ensure(3 * g)
    t[g:3 * g].fill_(9)
    torch.cuda.synchronize()
    assert bool((t[:g] == 7).all()) and bool((t[g:3 * g] == 9).all())
    torch.cuda.synchronize()
    a.shrink(g)
    assert a.granules == 1 and a.mapped_bytes == g
    assert bool((t[:g] == 7).all())        # the kept prefix is untouched
    a.ensure(2 * g)
    t[g:2 * g].fill_(3)
    torch.cuda.synchronize()
    assert bool((t[g:2 * g] == 3).all()) and a.tensor().data_ptr() == base
    del t
    a.close()


def _check(layer, x, ex, mb):
    out = layer.forward(x)
    torch.cuda.synchronize()
    mb.check()
    m = x.shape[0]
    ids, w = layer.ids[:m].cpu(), layer.w[:m].cpu()
    ref = formats.reference_moe(x.cpu(), ids, w, ex)
    rel = float((out.cpu().float() - ref).norm() / ref.norm())
    assert rel < 1e-2, rel
    return ids


def test_elastic_layer_grow_fill_release(cuda_ops):
    from xtier_b200.cache.elastic import ElasticSlots
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    E, H, I, k = 16, 1024, 1024, 2
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=5, std=0.05)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(1)) * 0.02).bfloat16()
    bias = torch.zeros(E)
    bias[[8, 9, 10]] = 6.0                 # the routes go to 8, 9, 10: none of them in a base slot
    mb = Mailbox(H, timeout_s=10.0)
    eng = CpuEngine(ex, threads=2)
    layer = TieredMoE(0, router, ex, k, hot=[0, 1, 2, 3], router_bias=bias, mailbox=mb, engine=eng, device='cuda',
                      host_experts=ex)
    el = ElasticSlots(layer, 4)
    mb.start()
    try:
        x = torch.randn(2, H, generator=torch.Generator().manual_seed(2)).bfloat16().cuda()
        _check(layer, x, ex, mb)                            # no extra slots: CPU routes
        el.grow(4)
        for e in (8, 9, 10):
            layer.fill(e)
        torch.cuda.synchronize()
        assert set(layer.resident()) == {0, 1, 2, 3, 8, 9, 10}
        ids = _check(layer, x, ex, mb)
        slots = layer.slots[:2, :k].cpu()
        assert bool((slots >= 4).all()), (ids, slots)      # served from the extra slots
        mapped = el.mapped_bytes()
        el.release(0)
        assert el.mapped_bytes() < mapped and set(layer.resident()) == {0, 1, 2, 3}
        _check(layer, x, ex, mb)                            # back on the CPU
        el.grow(2)
        layer.fill(9)
        torch.cuda.synchronize()
        _check(layer, x, ex, mb)
    finally:
        mb.stop()
        mb.close()
        el.close()
