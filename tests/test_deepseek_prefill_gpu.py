"""DSA sparse prefill of the DeepSeek-shaped model on one B200 (the pipeline of the 64K TTFT, small shapes): the
expert-parallel prefill MoE against the fp32 dequant reference, and the sparse prefill (indexer -> top-k -> tcgen05
MLA over the NVFP4 latent cache) against dense causal attention when the top-k keeps every earlier key."""
import pytest
import torch

from xtier_b200 import formats

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize('mx,tol', [(False, 2e-2), (True, 6e-2)])
def test_ep_prefill_moe_matches_reference(cuda_ops, mx, tol):
    """Exact W4A16 path, and the block-scaled path with MXFP8 activations (the reference's prefill numerics)."""
    from xtier_b200.models.deepseek_prefill import EPPrefillMoE
    from xtier_b200.parallel import dist as xdist
    from xtier_b200.parallel.ep import EPComm, EPMoE
    xdist.init()
    H, I, E, k, T = 1024, 512, 16, 4, 300
    ex = formats.random_experts(E, H, I, formats.MXFP4, seed=21, std=0.05)
    sh = formats.random_experts(1, H, I, formats.MXFP4, seed=22, std=0.05)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(23)) * 0.02).bfloat16()
    comm = EPComm(H, I, E, k, 8, torch.device('cuda'), timeout_s=5.0, n_shared=1)
    layer = EPMoE(0, comm, router, ex, k, shared=sh, mode=1, n_group=4, topk_group=2, renorm=True, scale=2.5)
    try:
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(24)).bfloat16().cuda()
        add = torch.randn(T, H, generator=torch.Generator().manual_seed(25)).bfloat16().cuda()
        out = torch.empty_like(x)
        pm = EPPrefillMoE(chunk=512, mx=mx)
        pm.forward(layer, x, out, add)
        torch.cuda.synchronize()
        assert int(pm.err.item()) == 0
        ids, w = pm.last[0].cpu(), pm.last[1].cpu()
        assert bool((ids[:, k:] == -1).all())
        ref = formats.reference_moe(x.cpu(), ids[:, :k], w[:, :k], ex, shared=sh) + add.cpu().float()
        assert _rel(out.cpu(), ref) < tol, _rel(out.cpu(), ref)
    finally:
        comm.close()


def _cfg():
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Config
    return DeepSeekV3Config(hidden=1024, layers=3, dense_layers=1, dense_inter=2048, heads=128, q_lora=256, kv_lora=512,
                            qk_nope=128, qk_rope=64, v_head=128, experts=16, top_k=4, inter=512, n_group=4,
                            topk_group=2, vocab=2000, attn='mla', index_topk=256)


def test_sparse_prefill_matches_dense_when_topk_covers(cuda_ops):
    from xtier_b200.models.deepseek_prefill import SparsePrefill
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Model
    cfg = _cfg()
    model = DeepSeekV3Model(cfg, device='cuda', seed=5, ep=True, decode_tokens=8, indexer=True)
    try:
        T = 256
        ids = torch.randint(0, cfg.vocab, (T,), generator=torch.Generator().manual_seed(6)).cuda()
        # the exact W4A16 experts on both sides: the comparison is about the attention
        sp = SparsePrefill(model, T, q_chunk=128, moe_chunk=128, mx=False)
        lg = sp.run(ids, return_logits=True).float()
        torch.cuda.synchronize()
        sp.check()
        dn = SparsePrefill(model, T, q_chunk=128, moe_chunk=128, dense=True, mx=False)
        lg_d = dn.run(ids, return_logits=True).float()
        assert _rel(lg, lg_d) < 3e-2, _rel(lg, lg_d)
    finally:
        model.close()


def test_sparse_prefill_topk_below_length_runs(cuda_ops):
    """index_topk < prompt length: every query attends over its own top-k (no dense equivalent); the result stays
    finite and the caches are written at every position."""
    from xtier_b200.models.deepseek_prefill import SparsePrefill
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Model
    cfg = _cfg()
    cfg.index_topk = 128
    model = DeepSeekV3Model(cfg, device='cuda', seed=7, ep=True, decode_tokens=8, indexer=True)
    try:
        T = 384
        ids = torch.randint(0, cfg.vocab, (T,), generator=torch.Generator().manual_seed(8)).cuda()
        sp = SparsePrefill(model, T, q_chunk=128, moe_chunk=256)
        lg = sp.run(ids, return_logits=True).float()
        torch.cuda.synchronize()
        sp.check()
        assert bool(torch.isfinite(lg).all())
        assert int((sp.latent[0].scales.view(T, -1).sum(1) == 0).sum()) == 0
    finally:
        model.close()
