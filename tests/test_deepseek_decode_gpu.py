"""The DeepSeek-shaped batched decode step on B200: the MLA projection kernels against fp32 PyTorch, the tiered EP MoE
(GPU pool + CPU tier through the mailbox, one rank) against the fp32 dequant reference, and the captured decode step
against the model's eager forward."""
import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _rope_ref(x, pos, theta):
    d = x.shape[-1]
    inv = theta ** (-torch.arange(0, d // 2, dtype=torch.float64, device=x.device) * 2 / d)
    ang = pos.double()[:, None] * inv[None]
    cos, sin = ang.cos().float(), ang.sin().float()
    while cos.dim() < x.dim():
        cos, sin = cos.unsqueeze(-2), sin.unsqueeze(-2)
    a, b = x[..., :d // 2], x[..., d // 2:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)


def test_mla_prep_matches_reference(cuda_ops):
    from xtier_b200.attention.mla import LatentCache
    torch.manual_seed(0)
    T, ql = 5, 1536
    inp = torch.randn(T, ql + 576 + 40, device='cuda').bfloat16()[:, :ql + 576]   # strided rows
    qn = (torch.rand(ql, device='cuda') + .5).bfloat16()
    kn = (torch.rand(512, device='cuda') + .5).bfloat16()
    pos = torch.tensor([0, 3, 17, 900, 4095], dtype=torch.int32, device='cuda')
    slot = torch.tensor([2, 9, 4, 0, 7], dtype=torch.int64, device='cuda')
    cache = LatentCache(1, 16, 'cuda')
    q_out = torch.empty(T, ql, dtype=torch.bfloat16, device='cuda')
    lat = torch.empty(T, 576, dtype=torch.bfloat16, device='cuda')
    cuda_ops.mla_prep(inp, ql, qn, kn, pos, slot, 1e-6, 10000.0, q_out, cache.codes, cache.scales, cache.rope, lat)
    x = inp.float()
    rms = lambda v, w: v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert _rel(q_out, rms(x[:, :ql], qn)) < 1e-2
    assert _rel(lat[:, :512], rms(x[:, ql:ql + 512], kn)) < 1e-2
    assert _rel(lat[:, 512:], _rope_ref(x[:, ql + 512:], pos, 10000.0)) < 1e-2
    # the cache holds the NVFP4 image of the same latent rows (the encoder of mla_kv_write)
    ref_cache = LatentCache(1, 16, 'cuda')
    ref_cache.write(lat, slot)
    assert torch.equal(cache.codes[slot], ref_cache.codes[slot])
    assert torch.equal(cache.scales[slot], ref_cache.scales[slot])
    assert torch.equal(cache.rope[slot], ref_cache.rope[slot])


@pytest.mark.parametrize('T', [1, 4, 37])
def test_head_gemm_absorb_and_unabsorb(cuda_ops, T):
    torch.manual_seed(T)
    Hh = 128
    q = torch.randn(T, Hh, 192, device='cuda').bfloat16()
    w_uk = (torch.randn(Hh, 128, 512, device='cuda') * 0.05).bfloat16()
    pos = torch.randint(0, 5000, (T,), dtype=torch.int32, device='cuda')
    qf = torch.empty(T, Hh, 576, dtype=torch.bfloat16, device='cuda')
    cuda_ops.head_gemm(q, w_uk, qf, pos, 128, 512, 64, 10000.0)
    ref = torch.einsum('thn,hnl->thl', q[..., :128].float(), w_uk.float())
    assert _rel(qf[..., :512], ref) < 1e-2
    assert _rel(qf[..., 512:], _rope_ref(q[..., 128:].float(), pos, 10000.0)) < 1e-2
    o_lat = torch.randn(T, Hh, 512, device='cuda').bfloat16()
    w_uvT = (torch.randn(Hh, 512, 128, device='cuda') * 0.05).bfloat16()
    out = torch.empty(T, Hh, 128, dtype=torch.bfloat16, device='cuda')
    cuda_ops.head_gemm(o_lat, w_uvT, out)
    assert _rel(out, torch.einsum('thl,hlv->thv', o_lat.float(), w_uvT.float())) < 1e-2


def test_silu_mul(cuda_ops):
    torch.manual_seed(3)
    g = torch.randn(6, 2 * 1024, device='cuda').bfloat16()
    out = torch.empty(6, 1024, dtype=torch.bfloat16, device='cuda')
    cuda_ops.silu_mul(g, out)
    a, b = g[:, :1024].float(), g[:, 1024:].float()
    assert _rel(out, torch.nn.functional.silu(a) * b) < 1e-2


def test_linear_two_pass_gemv(cuda_ops):
    torch.manual_seed(4)
    x = torch.randn(10, 16384, device='cuda').bfloat16()     # 6 rows per pass fit the GEMV's shared memory
    w = (torch.randn(768, 16384, device='cuda') * 0.02).bfloat16()
    assert _rel(cuda_ops.linear(x, w), x.float() @ w.float().T) < 1e-2


def test_ep_tiered_moe_one_rank(cuda_ops):
    """GPU pool for part of the experts, the rest on the CPU engine through the mailbox: the EP kernels at world 1
    against the fp32 dequant reference, eager and replayed from a CUDA graph."""
    from xtier_b200.engine import CpuEngine
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.deepseek_v3 import ep_layout
    from xtier_b200.parallel import dist as xdist
    from xtier_b200.parallel.ep import EPComm, EPMoE
    xdist.init()
    H, I, E, k, T = 1024, 512, 16, 4, 12
    ex = formats.random_experts(E, H, I, formats.MXFP4, seed=5, std=0.05)
    table, pools, cpu_ids = ep_layout(E, 1, 10, seed=9)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(6)) * 0.02).bfloat16()
    mb = Mailbox(H, timeout_s=10.0)
    comm = EPComm(H, I, E, k, 16, torch.device('cuda'), timeout_s=5.0, slots_per_rank=10)
    engine = CpuEngine(ex.select(torch.tensor(cpu_ids)), threads=2, slots=len(cpu_ids), resident=cpu_ids,
                       total_experts=E)
    layer = EPMoE(3, comm, router, ex.select(torch.tensor(pools[0])), k, table=table, mailbox=mb, engine=engine,
                  mode=1, n_group=4, topk_group=2, renorm=True, scale=2.5)
    mb.start()
    try:
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(7)).bfloat16().cuda()
        out = layer.forward(x)
        torch.cuda.synchronize()
        comm.check()
        mb.check()
        ids, w = layer.router.ids[:T].cpu(), layer.router.wt[:T].cpu()
        slots = layer.router.slots[:T].cpu()
        assert bool((slots < 0).any()) and bool((slots >= 0).any())   # both tiers took routes
        ref = formats.reference_moe(x.cpu(), ids, w, ex)
        assert _rel(out.cpu(), ref) < 2e-2, _rel(out.cpu(), ref)
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
            out_g.zero_()
            g.replay()
            torch.cuda.synchronize()
            assert torch.equal(out_g, out)
        comm.check()
        mb.check()
        del g
    finally:
        mb.stop()
        comm.close()


def _small_cfg(**kw):
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Config
    base = dict(hidden=1024, layers=3, dense_layers=1, dense_inter=2048, heads=128, q_lora=256, kv_lora=512,
                qk_nope=128, qk_rope=64, v_head=128, experts=16, top_k=4, inter=512, n_group=4, topk_group=2,
                vocab=2000, attn='mla')
    base.update(kw)
    return DeepSeekV3Config(**base)


def test_batched_decode_step_matches_forward(cuda_ops):
    """The kernel decode step (mla_prep, head_gemm, MLA, EP MoE with a CPU tier) against the model's eager forward on
    the same state, then the same step captured and replayed by the Generator."""
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Model
    from xtier_b200.runtime.decode import Generator
    cfg = _small_cfg()
    mb = Mailbox(cfg.hidden, timeout_s=10.0)
    model = DeepSeekV3Model(cfg, device='cuda', seed=2, ep=True, gpu_experts=11, mailbox=mb, engine_threads=2,
                            decode_tokens=8, pcie_slots=0)   # every CPU-tier route on the engine
    mb.start()
    try:
        B, L0 = 3, 40
        st = model.alloc_state(B, 256)
        model.fill_synthetic_cache(st, L0, seed=1)
        toks = torch.randint(0, cfg.vocab, (B,), generator=torch.Generator().manual_seed(3)).cuda()
        rows = torch.arange(B, dtype=torch.int32, device='cuda')
        pos = torch.full((B,), L0, dtype=torch.int32, device='cuda')
        ref = model.forward(st, toks, rows, pos, decode=True).float()
        buf = model.decode_buffers(B)
        buf['tokens'].copy_(toks)
        buf['pos'].fill_(L0)
        model.decode_step(st, buf)
        torch.cuda.synchronize()
        model.check()
        assert _rel(buf['logits'], ref) < 3e-2, _rel(buf['logits'], ref)
        eager_next = buf['next'].clone()
        # captured: the Generator's graph replays the same step (self-advancing)
        gen = Generator(model, batch=B, max_len=256)
        gen.state = st
        gen.buf = buf
        buf['tokens'].copy_(toks)
        buf['pos'].fill_(L0)
        gen.capture()
        gen.step()
        torch.cuda.synchronize()
        gen.check()
        assert torch.equal(buf['next'], eager_next)
        assert int(buf['pos'][0]) == L0 + 1
        gen.graph = None
    finally:
        mb.stop()
        model.close()


def test_ep_shared_expert_in_pool(cuda_ops):
    """Shared experts as routes to the last pool slots of every rank: the EP kernels at world 1 against the fp32
    dequant reference with the shared expert added at weight 1."""
    from xtier_b200.parallel import dist as xdist
    from xtier_b200.parallel.ep import EPComm, EPMoE
    xdist.init()
    H, I, E, k, T = 1024, 512, 16, 4, 9
    ex = formats.random_experts(E, H, I, formats.MXFP4, seed=15, std=0.05)
    sh = formats.random_experts(1, H, I, formats.MXFP4, seed=16, std=0.05)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(17)) * 0.02).bfloat16()
    comm = EPComm(H, I, E, k, 16, torch.device('cuda'), timeout_s=5.0, n_shared=1)
    layer = EPMoE(0, comm, router, ex, k, shared=sh, mode=1, n_group=4, topk_group=2, renorm=True, scale=2.5)
    try:
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(18)).bfloat16().cuda()
        add = torch.randn(T, H, generator=torch.Generator().manual_seed(19)).bfloat16().cuda()
        out = layer.forward(x, add=add)
        torch.cuda.synchronize()
        comm.check()
        ids, w = layer.router.ids[:T].cpu(), layer.router.wt[:T].cpu()
        assert bool((ids[:, k:] == -1).all()) and bool((w[:, k:] == 1).all())
        ref = formats.reference_moe(x.cpu(), ids[:, :k], w[:, :k], ex, shared=sh) + add.cpu().float()
        assert _rel(out.cpu(), ref) < 2e-2, _rel(out.cpu(), ref)
    finally:
        comm.close()


def test_chunked_prompt_prefill_and_served_decode(cuda_ops):
    """A prompt longer than the EP exchange's tokens prefills in chunks (each a continuation over the BF16 latent
    cache) and gives the logits of one pass; the server's backend (serve.GenBackend over the Generator, greedy, no
    prefix reuse) then decodes the tokens of the eager forward."""
    from xtier_b200 import serve
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Model
    from xtier_b200.runtime.decode import Generator
    cfg = _small_cfg()
    toks = torch.randint(0, cfg.vocab, (20,), generator=torch.Generator().manual_seed(9)).cuda()
    logits = {}
    for chunk in (8, 32):
        mb = Mailbox(cfg.hidden, timeout_s=10.0)
        model = DeepSeekV3Model(cfg, device='cuda', seed=6, ep=True, gpu_experts=11, mailbox=mb, engine_threads=2,
                                decode_tokens=chunk)
        model.keep_bf16_cache = True
        mb.start()
        try:
            st = model.alloc_state(1, 128)
            _, logits[chunk] = model.prefill(st, toks, all_logits=True)
            model.check()
            if chunk == 8:
                with pytest.raises(ValueError):
                    model.prefill({'batch': 1}, toks)          # chunks without the BF16 latent cache
                # eager greedy continuation from the same prompt
                want, cur = [], int(logits[chunk][-1].argmax())
                for i in range(4):
                    want.append(cur)
                    nxt = model.decode_tokens_step(st, torch.tensor([cur], device='cuda'),
                                                   torch.zeros(1, dtype=torch.int32, device='cuda'))
                    cur = int(nxt[0])
                be = serve.GenBackend(model, Generator(model, batch=1, max_len=128), None, mb, prefix_cache=False)
                got = [be.prefill(toks.tolist())] + [be.decode() for _ in range(3)]
                be.check()
                assert got[:2] == want[:2], (got, want)
                be.gen.graph = None
        finally:
            mb.stop()
            model.close()
    assert logits[8].shape == logits[32].shape == (20, cfg.vocab)
    assert _rel(logits[8], logits[32]) < 2e-2, _rel(logits[8], logits[32])


def test_pcie_staging_matches_cpu_tier(cuda_ops):
    """PCIe staging: the router hands up to 4 of the CPU-tier experts per call to the GPU, which copies them from the
    engine's own (CUDA-registered) host memory and computes them; the decode step's logits match the same model with
    every CPU-tier route on the engine, the claims are reset after every call, GPU routes grow, and the captured step
    replays the same tokens."""
    from xtier_b200.engine.mailbox import Mailbox
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Model
    from xtier_b200.runtime.decode import Generator
    cfg = _small_cfg()
    B, L0 = 4, 40
    toks = torch.randint(0, cfg.vocab, (B,), generator=torch.Generator().manual_seed(5)).cuda()
    res = {}
    for S in (0, 4):
        mb = Mailbox(cfg.hidden, timeout_s=10.0)
        model = DeepSeekV3Model(cfg, device='cuda', seed=8, ep=True, gpu_experts=6, mailbox=mb, engine_threads=2,
                                decode_tokens=8, pcie_slots=S)
        mb.start()
        try:
            assert model.pcie_slots == S and (S == 0 or len(model.host_maps) == len(model.engines))
            st = model.alloc_state(B, 256)
            model.fill_synthetic_cache(st, L0, seed=2)
            buf = model.decode_buffers(B)
            buf['tokens'].copy_(toks)
            buf['pos'].fill_(L0)
            model.decode_step(st, buf)
            torch.cuda.synchronize()
            model.check(st)
            layer = next(L['moe'] for L in model.layers if 'moe' in L)
            _, ls = mb.layer_stats(layer.layer, cfg.experts)
            res[S] = (buf['logits'].float().clone(), buf['next'].clone(), ls['gpu_routes'], ls['cpu_routes'])
            if S:
                assert bool((model.ep.claim == -1).all()) and int(model.ep.claim_count) == 0
                gen = Generator(model, batch=B, max_len=256)
                gen.state, gen.buf = st, buf
                buf['tokens'].copy_(toks)
                buf['pos'].fill_(L0)
                gen.capture()
                for _ in range(2):
                    gen.step()
                torch.cuda.synchronize()
                gen.check()
                assert bool((model.ep.claim == -1).all()) and int(model.ep.claim_count) == 0
                gen.graph = None
        finally:
            mb.stop()
            model.close()
    assert _rel(res[4][0], res[0][0]) < 3e-2, _rel(res[4][0], res[0][0])
    assert res[4][2] > res[0][2] and res[4][3] < res[0][3], (res[0][2:], res[4][2:])
