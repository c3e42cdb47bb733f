"""Swap ring of the hot-slot pool (cache/ring.py, csrc/cuda/pool_ring.cu) on the GPU: the commit kernel applies
UNMAPs at once and MAPs only after their copy has landed, in sequence order; swaps made between replays of a captured
decode call take effect inside the graph, and every output on the way matches the fp32 reference."""
import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def _commit(h, tables, err):
    torch.ops.xtier.pool_ring_commit(h, tables, err)
    torch.cuda.synchronize()


def test_commit_order_and_landing(cuda_ops):
    E = 8
    t0 = torch.full((E,), -1, dtype=torch.int32, device='cuda')
    t1 = torch.full((E,), -1, dtype=torch.int32, device='cuda')
    t0[3] = 0
    tables = torch.tensor([t0.data_ptr(), t1.data_ptr()], dtype=torch.int64, device='cuda')
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    h = torch.ops.xtier.pool_ring_create(16)
    try:
        post = lambda seq, l, e, s: torch.ops.xtier.pool_ring_post(h, seq, l, e, s)
        assert post(1, 0, 3, -1) == 0          # UNMAP expert 3 of layer 0
        assert post(2, 0, 5, 0) == 0           # MAP expert 5 into slot 0: its copy has not landed
        assert post(3, 1, 2, 1) == 0           # MAP on layer 1, behind it
        assert post(4, 1, 6, -1) == 0          # an UNMAP behind the blocked MAPs still applies
        t1[6] = 4
        _commit(h, tables, err)
        assert int(t0[3]) == -1 and int(t0[5]) == -1 and int(t1[2]) == -1 and int(t1[6]) == -1
        assert int(torch.ops.xtier.pool_ring_applied(h)) == 1
        torch.ops.xtier.pool_ring_landed(h, 2, err)   # seq 2's copy landed, seq 3's not yet
        _commit(h, tables, err)
        assert int(t0[5]) == 0 and int(t1[2]) == -1
        assert int(torch.ops.xtier.pool_ring_applied(h)) == 2
        torch.ops.xtier.pool_ring_landed(h, 3, err)
        _commit(h, tables, err)
        assert int(t1[2]) == 1 and int(t1[6]) == -1
        assert int(torch.ops.xtier.pool_ring_applied(h)) == 4
        assert int(err.item()) == 0
        # a command naming a layer outside the tables sets the error word and is skipped
        assert post(5, 7, 0, -1) == 0
        _commit(h, tables, err)
        assert int(err.item()) == 3
        assert int(torch.ops.xtier.pool_ring_applied(h)) == 5
        # the host never posts more than capacity - 1 unapplied commands
        for seq in range(6, 21):
            assert post(seq, 0, 1, -1) == 0
        assert post(21, 0, 1, -1) == -3
    finally:
        torch.cuda.synchronize()
        torch.ops.xtier.pool_ring_destroy(h)


def test_ring_swaps_between_graph_replays(cuda_ops):
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.cache.ring import SwapRing
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    E, H, I, k = 16, 512, 256, 2
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=31, std=0.05)
    router = (torch.randn(E, H) * 0.02).bfloat16()
    bias = torch.zeros(E)
    bias[:4] = 6.0   # experts 0..3 take almost every route
    mb = Mailbox(H, timeout_s=10.0)
    eng = CpuEngine(ex, threads=2)
    layer = TieredMoE(0, router, ex, k, hot=[12, 13, 14, 15], router_bias=bias, mailbox=mb, engine=eng,
                      device='cuda', host_experts=ex)
    ring = SwapRing([layer], 'cuda', capacity=64)
    mb.start()
    try:
        x = torch.randn(2, H).bfloat16().cuda()
        out = torch.empty_like(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ring.commit()
            layer.forward(x, out=out)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            ring.commit()
            layer.forward(x, out=out)

        def replay_and_check():
            g.replay()
            torch.cuda.synchronize()
            mb.check()
            ids, w = layer.ids[:2].cpu(), layer.w[:2].cpu()
            ref = formats.reference_moe(x.cpu(), ids, w, ex)
            assert float((out.cpu().float() - ref).norm() / ref.norm()) < 1e-2

        replay_and_check()
        for inc, vic in ((0, 12), (1, 13), (2, 14)):
            layer.swap(inc, vic)
            assert int(layer.table[vic].item()) == -1      # unmapped before the swap call returned to the host
            replay_and_check()                              # the incoming expert may still route to the CPU tier
        ring.stream.synchronize()
        replay_and_check()                                  # every copy landed: this replay's commit mapped them
        assert ring.applied() == ring.seq == 6
        tab = layer.table.cpu()
        for slot, e in enumerate(layer.resident()):
            assert int(tab[e]) == slot
        assert sorted(layer.resident()) == [0, 1, 2, 15]
        ring.check()
        del g
    finally:
        mb.stop()
        mb.close()
        ring.close()


def test_ring_prefill_sees_the_swaps(cuda_ops):
    """A prefill right after swaps whose copies are in flight waits for them (sync) and matches the reference."""
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.cache.ring import SwapRing
    E, H, I, k = 16, 512, 256, 2
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=32, std=0.05)
    router = (torch.randn(E, H) * 0.02).bfloat16()
    layer = TieredMoE(0, router, ex, k, hot=list(range(8)), device='cuda', host_experts=ex)
    layer.prepare_prefill()
    ring = SwapRing([layer], 'cuda')
    try:
        for inc, vic in ((9, 0), (11, 3), (15, 7)):
            layer.swap(inc, vic)
        x = (torch.randn(1100, H) * 0.5).bfloat16().cuda()   # grouped prefill: every expert on the GPU
        out = torch.empty_like(x)
        layer.prefill(x, out)
        # the same residency built directly, without swaps: the same kernels, the same routes
        fresh = TieredMoE(0, router, ex, k, hot=list(layer.hot), device='cuda', host_experts=ex)
        fresh.prepare_prefill()
        want = torch.empty_like(x)
        fresh.prefill(x, want)
        torch.cuda.synchronize()
        assert sorted(layer.hot) == [1, 2, 4, 5, 6, 9, 11, 15]
        assert float((out.float() - want.float()).norm() / want.float().norm()) < 1e-3
        assert ring.applied() == ring.seq
    finally:
        ring.close()
