"""Grouped FP4 expert GEMM for prefill (tcgen05, W4A16 with in-shared-memory dequantization) against the fp32
reference MoE: both formats, uneven runs per expert (including runs longer than a tile), routes left to the CPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('fmt,H,I,E,m,k', [('nvfp4', 512, 256, 8, 300, 4), ('mxfp4', 1024, 512, 16, 200, 8),
                                           ('nvfp4', 2048, 768, 32, 257, 8)])
def test_grouped_experts_vs_reference(cuda_ops, fmt, H, I, E, m, k):
    from xtier_b200 import formats
    from xtier_b200.cache.prefill import grouped_experts
    g = torch.Generator().manual_seed(E + m)
    ex = formats.random_experts(E, H, I, fmt, seed=E, std=0.05)
    x = torch.randn(m, H, generator=g).bfloat16()
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(m)]).int()
    # skew: expert 0 takes many routes (runs longer than one 128-row tile)
    ids[: m // 2, 0] = 0
    w = torch.rand(m, k, generator=g)
    slots = ids.clone()
    slots[torch.rand(m, k, generator=g) < 0.2] = -1          # CPU routes are skipped here
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    out = grouped_experts(x.cuda(), slots.cuda(), w.cuda(), ex.to('cuda'), err)
    torch.cuda.synchronize()
    assert int(err) == 0
    ids_ref = torch.where(slots >= 0, ids, torch.full_like(ids, -1))
    ref = formats.reference_moe(x, ids_ref, w, ex)
    rel = float((out.cpu() - ref).norm() / ref.norm())
    assert rel < 1e-2, rel


def test_tiny_qwen3_grouped_prefill_matches_reference(cuda_ops, monkeypatch):
    """Model-level: with the grouped path forced for every prefill call, a tiered model (half the experts hot, the
    rest uploaded from pinned host memory for the call) matches the fp32 forward."""
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    monkeypatch.setenv('XTIER_GPU_PREFILL_MIN', '16')
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128)
    model = Qwen3MoeModel(cfg, device='cuda', seed=2, hot_fraction=0.5, synthetic_experts=False, engine_threads=2)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(3)).cuda()
    st = model.alloc_state(1, 64)
    _, lp = model.prefill(st, prompt, return_logits=True)
    ref = model.reference_logits(prompt)
    rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 3e-2, rel


def test_grouped_prefill_after_swaps(cuda_ops, monkeypatch):
    """After adaptive swaps move experts between the GPU slots and the CPU side, a grouped prefill still covers every
    route: a swapped-out expert takes over the staging index of the one swapped in."""
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    monkeypatch.setenv('XTIER_GPU_PREFILL_MIN', '16')
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128)
    model = Qwen3MoeModel(cfg, device='cuda', seed=5, hot_fraction=0.5, synthetic_experts=False, engine_threads=2)
    prompt = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(4)).cuda()
    st = model.alloc_state(1, 64)
    model.prefill(st, prompt)            # builds the staging copies
    for L in model.layers:
        moe = L['moe']
        hot = moe.resident()
        cold = [e for e in range(moe.E) if e not in hot]
        moe.swap(cold[0], hot[0])
        moe.swap(cold[1], hot[1])
    torch.cuda.synchronize()
    st = model.alloc_state(1, 64)
    _, lp = model.prefill(st, prompt, return_logits=True)
    ref = model.reference_logits(prompt)
    rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 3e-2, rel


@pytest.mark.parametrize('mode', [0, 1])
def test_prefill_router_gemm_matches_decode_router(cuda_ops, mode):
    """Prefill-sized calls take the router logits from the FP32-output tensor-core GEMM and only select in the route
    kernel; the routes equal the decode router's (which computes the logits itself) up to near-ties."""
    from xtier_b200 import formats
    from xtier_b200.cache.pool import TieredMoE
    E, H, I, k = 64, 1024, 256, 4
    g = torch.Generator().manual_seed(mode)
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=1, std=0.05)
    router = (torch.randn(E, H, generator=g) * 0.05).bfloat16()
    bias = torch.randn(E, generator=g) * 0.1
    kw = dict(mode=1, n_group=8, topk_group=4, scale=2.5, corr_bias=torch.randn(E, generator=g) * 0.01) if mode else {}
    layer = TieredMoE(0, router, ex, k, router_bias=bias, device='cuda', **kw)
    x = torch.randn(300, H, generator=g).bfloat16().cuda()
    layer._alloc(300)
    layer.route(x, False)                      # m > 16: GEMM logits + selection
    ids_p, w_p = layer.ids[:300, :k].clone(), layer.w[:300, :k].clone()
    layer._alloc(16)
    ids_d, w_d = [], []
    for s in range(0, 300, 16):                # the decode router, 16 tokens at a time
        xs = x[s:s + 16].contiguous()
        layer.route(xs, False)
        ids_d.append(layer.ids[:xs.shape[0], :k].clone())
        w_d.append(layer.w[:xs.shape[0], :k].clone())
    ids_d, w_d = torch.cat(ids_d), torch.cat(w_d)
    same = (ids_p == ids_d).all(dim=1).float().mean().item()
    assert same > 0.98, same
    rows = (ids_p == ids_d).all(dim=1)
    assert torch.allclose(w_p[rows], w_d[rows], rtol=1e-4, atol=1e-5)
