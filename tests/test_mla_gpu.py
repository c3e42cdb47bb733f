"""MLA over the NVFP4 latent cache on the tensor cores against the fp32 PyTorch oracle on the dequantized cache:
cache write (NVFP4 round trip), dense and sparse (index lists with holes) decode, several queries."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def test_latent_cache_roundtrip(cuda_ops):
    from xtier_b200.attention.mla import LatentCache
    cache = LatentCache(2, 256)
    lat = torch.randn(300, 576, device='cuda').bfloat16()
    slots = torch.randperm(512, device='cuda')[:300]
    cache.write(lat, slots)
    back = cache.dequant(slots)
    # NVFP4: 1 mantissa bit and a per-16 E4M3 scale -> relative RMS error around 10 %; rope exact
    assert _rel(back[:, :512], lat[:, :512]) < 0.15
    assert torch.equal(back[:, 512:], lat[:, 512:].float())


@pytest.mark.parametrize('Q,n,nsel,holes', [(1, 700, 512, 0.0), (3, 2000, 1024, 0.1), (2, 300, 384, 0.3)])
def test_mla_decode_sparse(cuda_ops, Q, n, nsel, holes):
    from xtier_b200.attention.mla import LatentCache, MlaWorkspace, default_scale, mla_decode, reference_decode
    g = torch.Generator(device='cuda').manual_seed(Q * 7 + n)
    cache = LatentCache(1, n)
    lat = torch.randn(n, 576, device='cuda', generator=g).bfloat16()
    cache.write(lat, torch.arange(n, device='cuda'))
    q = (torch.randn(Q, 128, 576, device='cuda', generator=g) * 0.5).bfloat16()
    idx = torch.stack([torch.randperm(n, device='cuda', generator=g)[:nsel] if nsel <= n else
                       torch.cat([torch.randperm(n, device='cuda', generator=g),
                                  torch.full((nsel - n,), -1, device='cuda', dtype=torch.int64)])
                       for _ in range(Q)]).int()
    if holes:
        drop = torch.rand(idx.shape, device='cuda', generator=g) < holes
        idx[drop] = -1
    ws = MlaWorkspace(Q, nsel)
    scale = default_scale()
    out = mla_decode(q, idx, cache, ws, scale)
    torch.cuda.synchronize()
    assert int(ws.err) == 0
    ref = reference_decode(q, idx, cache, scale)
    assert _rel(out, ref) < 2e-2, _rel(out, ref)


@pytest.mark.parametrize('Q,n,nsel,holes,splits', [(1, 700, 512, 0.0, 1), (3, 2000, 1024, 0.1, 1),
                                                   (2, 300, 384, 0.3, 1), (4, 5000, 4480, 0.05, 7),
                                                   (2, 900, 1024, 0.0, 3), (5, 4000, 2048, 0.0, 1)])
def test_mla_flash_matches_reference(cuda_ops, Q, n, nsel, holes, splits):
    """The one-pass tcgen05 kernel (online softmax with lazy O correction in TMEM, V read in place through the
    MN-major descriptor) against the fp32 oracle, one split and several."""
    from xtier_b200.attention.mla import FlashWorkspace, LatentCache, default_scale, mla_flash, reference_decode
    g = torch.Generator(device='cuda').manual_seed(Q * 11 + n)
    cache = LatentCache(1, n)
    lat = torch.randn(n, 576, device='cuda', generator=g).bfloat16()
    cache.write(lat, torch.arange(n, device='cuda'))
    q = (torch.randn(Q, 128, 576, device='cuda', generator=g) * 0.5).bfloat16()
    idx = torch.stack([torch.randperm(n, device='cuda', generator=g)[:nsel] if nsel <= n else
                       torch.cat([torch.randperm(n, device='cuda', generator=g),
                                  torch.full((nsel - n,), -1, device='cuda', dtype=torch.int64)])
                       for _ in range(Q)]).int()
    if holes:
        drop = torch.rand(idx.shape, device='cuda', generator=g) < holes
        idx[drop] = -1
    ws = FlashWorkspace(Q, splits)
    scale = default_scale()
    out = mla_flash(q, idx, cache, scale, splits, ws)
    torch.cuda.synchronize()
    assert int(ws.err) == 0
    ref = reference_decode(q, idx, cache, scale)
    assert _rel(out, ref) < 2e-2, _rel(out, ref)
    out2 = mla_flash(q, idx, cache, scale, splits, ws)   # repeatable
    assert torch.equal(out, out2)


def test_mla_flash_growing_scores_rescale(cuda_ops):
    """Keys ordered so that every block raises the running max far past the lazy-correction threshold: O must be
    rescaled in TMEM block after block."""
    from xtier_b200.attention.mla import FlashWorkspace, LatentCache, default_scale, mla_flash, reference_decode
    n = 1024
    g = torch.Generator(device='cuda').manual_seed(3)
    cache = LatentCache(1, n)
    base = torch.randn(n, 576, device='cuda', generator=g)
    grow = torch.linspace(0.2, 3.0, n, device='cuda')[:, None]    # later keys score ever higher
    lat = (base * 0.3 + grow).bfloat16()
    cache.write(lat, torch.arange(n, device='cuda'))
    q = torch.ones(2, 128, 576, device='cuda').bfloat16() * 0.3
    idx = torch.arange(n, device='cuda', dtype=torch.int32)[None].repeat(2, 1).contiguous()
    ws = FlashWorkspace(2, 1)
    out = mla_flash(q, idx, cache, default_scale(), 1, ws)
    torch.cuda.synchronize()
    assert int(ws.err) == 0
    ref = reference_decode(q, idx, cache, default_scale())
    assert _rel(out, ref) < 2e-2, _rel(out, ref)
