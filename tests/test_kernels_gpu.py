"""sm_100a kernels vs plain fp32 PyTorch references (B200 only)."""
import math

import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_add_rmsnorm(cuda_ops):
    torch.manual_seed(0)
    x = torch.randn(7, 2048, device='cuda').bfloat16()
    r = torch.randn(7, 2048, device='cuda').bfloat16()
    w = (torch.rand(2048, device='cuda') + 0.5).bfloat16()
    out = torch.empty_like(x)
    r_ref = (x.float() + r.float()).bfloat16()
    cuda_ops.add_rmsnorm(x, r, w, out, 1e-6)
    assert torch.equal(r, r_ref)
    ref = r_ref.float() * torch.rsqrt(r_ref.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert _rel(out, ref) < 1e-2
    out2 = cuda_ops.rmsnorm(x, w, 1e-6)
    ref2 = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert _rel(out2, ref2) < 1e-2


@pytest.mark.parametrize('m,N,K', [(1, 5120, 2048), (3, 2048, 4096), (16, 512, 2048), (2, 1000, 7168)])
def test_gemv_bf16(cuda_ops, m, N, K):
    torch.manual_seed(m)
    x = torch.randn(m, K, device='cuda').bfloat16()
    w = (torch.randn(N, K, device='cuda') * 0.02).bfloat16()
    add = torch.randn(m, N, device='cuda').bfloat16()
    out = torch.empty(m, N, dtype=torch.bfloat16, device='cuda')
    cuda_ops.gemv(x, w, out)
    assert _rel(out, x.float() @ w.float().T) < 1e-2
    cuda_ops.gemv(x, w, out, add=add)
    assert _rel(out, x.float() @ w.float().T + add.float()) < 1e-2


def _rope_ref(x, pos, theta):
    D = x.shape[-1]
    inv = theta ** (-torch.arange(0, D // 2, dtype=torch.float64, device=x.device) * 2 / D)
    ang = pos.double()[:, None] * inv[None]
    cos, sin = ang.cos().float(), ang.sin().float()
    x1, x2 = x[..., :D // 2], x[..., D // 2:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


def test_qk_norm_rope_kv(cuda_ops):
    torch.manual_seed(1)
    T, Hq, Hkv, D, L = 5, 8, 2, 128, 64
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device='cuda').bfloat16()
    qn = (torch.rand(D, device='cuda') + .5).bfloat16()
    kn = (torch.rand(D, device='cuda') + .5).bfloat16()
    pos = torch.tensor([0, 3, 17, 40, 63], dtype=torch.int32, device='cuda')
    rows = torch.tensor([0, 0, 1, 1, 0], dtype=torch.int32, device='cuda')
    q = torch.empty(T, Hq, D, dtype=torch.bfloat16, device='cuda')
    kc = torch.zeros(2, Hkv, L, D, dtype=torch.bfloat16, device='cuda')
    vc = torch.zeros_like(kc)
    cuda_ops.qk_norm_rope_kv(qkv, qn, kn, pos, rows, q, kc, vc, Hq, Hkv, 1e6, 1e-6)
    x = qkv.float().view(T, Hq + 2 * Hkv, D)

    def norm(t, w):
        return (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).bfloat16().float()
    q_ref = _rope_ref(norm(x[:, :Hq], qn), pos, 1e6)
    k_ref = _rope_ref(norm(x[:, Hq:Hq + Hkv], kn), pos, 1e6)
    assert _rel(q, q_ref) < 1e-2
    for t in range(T):
        assert _rel(kc[rows[t], :, pos[t]], k_ref[t]) < 1e-2
        assert torch.equal(vc[rows[t], :, pos[t]], x[t, Hq + Hkv:].bfloat16())


@pytest.mark.parametrize('G,N', [(8, 1), (8, 37), (8, 2304), (4, 513), (1, 100), (16, 300)])
def test_attn_decode(cuda_ops, G, N):
    torch.manual_seed(2)
    B, Hkv, D, L = 2, 2, 128, 4096
    Hq = Hkv * G
    q = torch.randn(B, Hq, D, device='cuda').bfloat16()
    kc = torch.randn(B, Hkv, L, D, device='cuda').bfloat16()
    vc = torch.randn(B, Hkv, L, D, device='cuda').bfloat16()
    lens = torch.tensor([N, max(1, N // 2)], dtype=torch.int32, device='cuda')
    splits = cuda_ops.attn_decode_splits(B, Hkv, L)
    ws_o = torch.empty(B * Hkv * splits * G * D, device='cuda')
    ws_ml = torch.empty(B * Hkv * splits * G * 2, device='cuda')
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device='cuda')
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    for _ in range(2):   # the arrival counters must reset themselves
        cuda_ops.attn_decode(q, kc, vc, lens, out, ws_o, ws_ml, cnt, splits, scale)
    for b in range(B):
        n = int(lens[b])
        k = kc[b, :, :n].float().repeat_interleave(G, 0)
        v = vc[b, :, :n].float().repeat_interleave(G, 0)
        s = torch.einsum('hd,hnd->hn', q[b].float(), k) * scale
        ref = torch.einsum('hn,hnd->hd', s.softmax(-1), v)
        assert _rel(out[b], ref) < 1e-2, (b, _rel(out[b], ref))
    assert int(cnt.sum()) == 0


def _moe_case(E, H, I, k, m, fmt, hot=None, n_shared=0, seed=0, mode=0):
    from xtier_b200.cache.pool import TieredMoE
    torch.manual_seed(seed)
    ex = formats.random_experts(E, H, I, fmt, seed=seed, std=0.05)
    sh = formats.random_experts(n_shared, H, I, fmt, seed=seed + 1, std=0.05) if n_shared else None
    router = (torch.randn(E, H) * 0.02).bfloat16()
    x = torch.randn(m, H).bfloat16()
    return ex, sh, router, x


@pytest.mark.parametrize('fmt,E,H,I,k,m', [(formats.NVFP4, 16, 2048, 768, 8, 1), (formats.NVFP4, 16, 512, 256, 4, 5),
                                           (formats.MXFP4, 16, 1024, 512, 4, 3), (formats.MXFP4, 8, 256, 128, 2, 16)])
def test_moe_decode_all_hot(cuda_ops, fmt, E, H, I, k, m):
    from xtier_b200.cache.pool import TieredMoE
    ex, _, router, x = _moe_case(E, H, I, k, m, fmt)
    layer = TieredMoE(0, router, ex, k, device='cuda')
    out = layer.forward(x.cuda())
    ids, w = layer.ids[:m].cpu(), layer.w[:m].cpu()
    p = (x.float() @ router.float().T).softmax(-1)
    tw, tid = p.topk(k, -1)
    assert torch.equal(ids.sort(-1).values, tid.int().sort(-1).values)
    assert torch.allclose(w.sort(-1).values, (tw / tw.sum(-1, keepdim=True)).sort(-1).values, atol=1e-5)
    ref = formats.reference_moe(x, ids, w, ex)
    assert _rel(out.cpu(), ref) < 1e-2, _rel(out.cpu(), ref)


def test_moe_decode_grouped_sigmoid_with_shared(cuda_ops):
    from xtier_b200.cache.pool import TieredMoE
    E, H, I, k, m = 32, 512, 256, 4, 3
    ex, sh, router, x = _moe_case(E, H, I, k, m, formats.MXFP4, n_shared=1, seed=3)
    corr = torch.randn(E) * 0.1
    layer = TieredMoE(0, router, ex, k, shared=sh, mode=1, n_group=4, topk_group=2, renorm=True, scale=2.5,
                      corr_bias=corr, device='cuda')
    out = layer.forward(x.cuda())
    s = torch.sigmoid(x.float() @ router.float().T)
    sel = s + corr
    gs = sel.view(m, 4, 8).topk(2, -1).values.sum(-1)
    keep = torch.zeros(m, 4, dtype=torch.bool).scatter_(1, gs.topk(2, -1).indices, True)
    sel = sel.masked_fill(~keep.repeat_interleave(8, 1), float('-inf'))
    tid = sel.topk(k, -1).indices
    tw = s.gather(1, tid)
    tw = tw / tw.sum(-1, keepdim=True) * 2.5
    ids = layer.ids[:m, :k].cpu()
    assert torch.equal(ids.sort(-1).values, tid.int().sort(-1).values)
    ref = formats.reference_moe(x, tid.int(), tw, ex, shared=sh)
    assert _rel(out.cpu(), ref) < 1e-2


def test_moe_decode_with_cpu_tier_and_graph(cuda_ops):
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    E, H, I, k, m = 16, 512, 256, 4, 2
    ex, _, router, x = _moe_case(E, H, I, k, m, formats.NVFP4, seed=4)
    mb = Mailbox(H, timeout_s=10.0)
    eng = CpuEngine(ex, threads=2)
    layer = TieredMoE(3, router, ex, k, hot=[0, 2, 4, 6, 8, 10, 12, 14], mailbox=mb, engine=eng, device='cuda')
    mb.start()
    try:
        xc = x.cuda()
        out = layer.forward(xc)
        torch.cuda.synchronize()
        mb.check()
        ids, w = layer.ids[:m].cpu(), layer.w[:m].cpu()
        assert (layer.slots[:m].cpu() < 0).any(), 'the case should route something to the CPU'
        ref = formats.reference_moe(x, ids, w, ex)
        assert _rel(out.cpu(), ref) < 1e-2
        # the same call captured in a CUDA graph, replayed twice
        out_g = torch.empty_like(out)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            layer.forward(xc, out=out_g)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer.forward(xc, out=out_g)
        for _ in range(2):
            out_g.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out_g, out)
        mb.check()
        counts, st = mb.layer_stats(3, E)
        assert st['calls'] >= 3 and counts.sum() > 0
        del g
    finally:
        mb.stop()
        mb.close()


def test_moe_layer_without_gpu_slots(cuda_ops):
    """A layer with no hot and no shared expert: every route goes to the CPU engine through the mailbox, decode
    (eager and graph-replayed) and a prefill-sized call both match the fp32 reference."""
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    E, H, I, k, m = 16, 512, 256, 4, 2
    ex, _, router, x = _moe_case(E, H, I, k, m, formats.NVFP4, seed=9)
    mb = Mailbox(H, timeout_s=10.0)
    eng = CpuEngine(ex, threads=2)
    layer = TieredMoE(5, router, ex, k, hot=[], mailbox=mb, engine=eng, device='cuda')
    assert layer.slotless and layer.gpu_bytes() == 0
    mb.start()
    try:
        xc = x.cuda()
        out = layer.forward(xc)
        torch.cuda.synchronize()
        mb.check()
        ids, w = layer.ids[:m].cpu(), layer.w[:m].cpu()
        assert bool((layer.slots[:m].cpu() < 0).all())
        assert _rel(out.cpu(), formats.reference_moe(x, ids, w, ex)) < 1e-2
        out_g = torch.empty_like(out)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            layer.forward(xc, out=out_g)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer.forward(xc, out=out_g)
        out_g.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out_g, out)
        del g
        xp = torch.randn(40, H, generator=torch.Generator().manual_seed(10)).bfloat16()
        outp = layer.forward(xp.cuda())        # prefill-sized: the CPU engine computes every route
        torch.cuda.synchronize()
        from xtier_b200.cache.pool import _PREFILL_BUFS   # the prefill call's own route buffers
        pf = _PREFILL_BUFS[(layer.kk, E, I, H, layer.device)]
        idp, wp = pf['ids'][:40, :k].cpu(), pf['w'][:40, :k].cpu()
        refp = formats.reference_moe(xp, idp, wp, ex)
        assert _rel(outp.cpu(), refp) < 1e-2
        mb.check()
    finally:
        mb.stop()
        mb.close()


def test_mailbox_wait_times_out_without_hanging(cuda_ops):
    """Nothing answers the mailbox (no dispatcher): the GPU wait gives up after its deadline and reports it."""
    import time
    from xtier_b200.cache.pool import TieredMoE
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox, MailboxError
    E, H, I, k = 8, 256, 128, 2
    ex, _, router, x = _moe_case(E, H, I, k, 1, formats.NVFP4, seed=5)
    mb = Mailbox(H, timeout_s=0.5)
    eng = CpuEngine(ex, threads=1)
    layer = TieredMoE(0, router, ex, k, hot=[0], mailbox=mb, engine=eng, device='cuda')
    t0 = time.time()
    layer.forward(x.cuda())
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    with pytest.raises(MailboxError, match='timed out'):
        mb.check()
    mb.check()   # cleared
    mb.close()


def test_tiny_qwen3_decode_graph_matches_eager(cuda_ops):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    cfg = Qwen3MoeConfig.tiny()
    model = Qwen3MoeModel(cfg, device='cuda', seed=0)
    prompt = torch.randint(0, cfg.vocab, (1, 40))
    g1 = Generator(model, 1, 128, use_graph=False)
    a = g1.generate(prompt, 12)
    g2 = Generator(model, 1, 128, use_graph=True)
    b = g2.generate(prompt, 12)
    assert torch.equal(a, b)


def test_tiny_qwen3_prefill_and_decode_match_fp32_reference(cuda_ops):
    """Logits of the prefill path and of the decode path (KV cache + decode kernels) against an fp32 PyTorch forward
    of the whole sequence."""
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    cfg = Qwen3MoeConfig.tiny(std=0.05)
    model = Qwen3MoeModel(cfg, device='cuda', seed=1, synthetic_experts=False)
    prompt = torch.randint(0, cfg.vocab, (1, 24), generator=torch.Generator().manual_seed(0))
    st = model.alloc_state(1, 64)
    _, lp = model.prefill(st, prompt[0].cuda(), return_logits=True)
    ref = model.reference_logits(prompt[0].cuda())
    assert _rel(lp, ref) < 3e-2, _rel(lp, ref)
    gen = Generator(model, 1, 64, use_graph=False)
    new = gen.generate(prompt, 3)
    # the decode step's logits after the last generated token vs the reference over prompt + generated tokens
    seq = torch.cat([prompt, new[:, :2]], 1)[0]
    gen2 = Generator(model, 1, 64, use_graph=False)
    gen2.prefill(seq[:-1].view(1, -1))
    gen2.buf['tokens'].fill_(int(seq[-1]))
    gen2.step()
    ref2 = model.reference_logits(seq.cuda())
    assert _rel(gen2.buf['logits'][0], ref2) < 3e-2, _rel(gen2.buf['logits'][0], ref2)


@pytest.mark.parametrize('G,N,splits', [(8, 2084, 36), (8, 33, 37), (16, 1000, 8), (8, 32768, 37), (8, 5000, 3)])
def test_attn_decode_tensor_core_path(cuda_ops, G, N, splits):
    """The mma.sync path (query groups of 8 / 16 heads): uneven splits, blocks past the end of a split, more keys per
    warp than one block (double-buffered loads), against the fp32 reference."""
    torch.manual_seed(G + N)
    B, Hkv, D = 2, 2, 128
    L = N + 64
    Hq = Hkv * G
    q = torch.randn(B, Hq, D, device='cuda').bfloat16()
    kc = torch.randn(B, Hkv, L, D, device='cuda').bfloat16()
    vc = torch.randn(B, Hkv, L, D, device='cuda').bfloat16()
    lens = torch.tensor([N, max(1, N // 3)], dtype=torch.int32, device='cuda')
    ws_o = torch.empty(B * Hkv * splits * G * D, device='cuda')
    ws_ml = torch.empty(B * Hkv * splits * G * 2, device='cuda')
    cnt = torch.zeros(B * Hkv, dtype=torch.int32, device='cuda')
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(D)
    for _ in range(2):
        cuda_ops.attn_decode(q, kc, vc, lens, out, ws_o, ws_ml, cnt, splits, scale)
    torch.cuda.synchronize()
    for b in range(B):
        n = int(lens[b])
        k = kc[b, :, :n].float().repeat_interleave(G, 0)
        v = vc[b, :, :n].float().repeat_interleave(G, 0)
        s = torch.einsum('hd,hnd->hn', q[b].float(), k) * scale
        ref = torch.einsum('hn,hnd->hd', s.softmax(-1), v)
        assert _rel(out[b], ref) < 1e-2, (b, _rel(out[b], ref))
    assert int(cnt.sum()) == 0
