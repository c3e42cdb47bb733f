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


def test_mla_flash_strided_query_and_output(cuda_ops):
    """Flash MLA through head-major views (latent and rotary query parts as separate strided tensors, strided output)
    equals the contiguous [Q, 128, 576] call bit for bit."""
    from xtier_b200.attention.mla import LatentCache, default_scale, mla_flash
    g = torch.Generator(device='cuda').manual_seed(41)
    Q, n = 5, 1000
    lc = LatentCache(1, n)
    lc.write(torch.randn(n, 576, device='cuda', generator=g).bfloat16(), torch.arange(n, device='cuda'))
    q = (torch.randn(Q, 128, 576, device='cuda', generator=g) * 0.5).bfloat16()
    idx = torch.stack([torch.randperm(n, device='cuda', generator=g)[:256] for _ in range(Q)]).int()
    ref = mla_flash(q, idx, lc, default_scale())
    q_lat = q[..., :512].transpose(0, 1).contiguous()          # [128, Q, 512] head-major
    q_pe = q[..., 512:].transpose(0, 1).contiguous()           # [128, Q, 64]
    o = torch.zeros(128, Q, 512, dtype=torch.bfloat16, device='cuda')
    mla_flash(q_lat.transpose(0, 1), idx, lc, default_scale(), out=o.transpose(0, 1), q_rope=q_pe.transpose(0, 1))
    assert torch.equal(o.transpose(0, 1), ref)


def test_rope_heads_and_fp8_query_quantization(cuda_ops):
    """RoPE kernel over strided (token, head) views against the fp32 PyTorch rotation; the fused FP8 query
    quantization against the PyTorch one (the same scales and weights; the E4M3 bytes agree but for a few in a
    thousand that PyTorch's conversion rounds the other way, one code step apart)."""
    from xtier_b200 import ops
    from xtier_b200.attention import dsa
    from xtier_b200.models.deepseek_v3 import _rope
    g = torch.Generator(device='cuda').manual_seed(42)
    T, H = 300, 128
    x = torch.randn(T, H, 192, device='cuda', generator=g).bfloat16()
    pos = torch.randint(0, 70000, (T,), device='cuda', generator=g).int()
    ref = _rope(x[..., 128:].transpose(0, 1), pos, 10000.0).transpose(0, 1).float()
    out = torch.empty(H, T, 64, dtype=torch.bfloat16, device='cuda')
    ops.rope_heads(x[..., 128:], pos, 10000.0, out.transpose(0, 1))
    assert float((out.transpose(0, 1).float() - ref).abs().max()) < 0.05
    assert float((out.transpose(0, 1).float() - ref).norm() / ref.norm()) < 5e-3
    q = torch.randn(T, 64, 128, device='cuda', generator=g).bfloat16()
    w = torch.randn(T, 64, device='cuda', generator=g).bfloat16()
    q8_ref, w8_ref = dsa.quantize_queries(q, w.float() * 0.125)
    q8 = torch.empty_like(q8_ref)
    w8 = torch.empty_like(w8_ref)
    torch.ops.xtier.dsa_quant_q(q, w, 0.125, q8, w8)
    assert torch.allclose(w8, w8_ref, rtol=1e-6, atol=0)
    diff = q8 != q8_ref
    assert float(diff.float().mean()) < 1e-2
    a = q8.view(torch.float8_e4m3fn).float()
    b = q8_ref.view(torch.float8_e4m3fn).float()
    assert bool(((a - b).abs() <= b.abs() * 0.125 + 2 ** -9).all())


def test_mla_flash_bounds_check_flags_bad_slot():
    """XTIER_DEBUG_BOUNDS: a selected slot past the cache is skipped and reported (error word 2), the rest of the
    query's keys still count. Runs in a child process: the switch is read once per process."""
    import os
    import subprocess
    import sys
    code = r"""
import copy
import torch
from xtier_b200 import ops
from xtier_b200.attention.mla import FlashWorkspace, LatentCache, default_scale, mla_flash
ops.load()
g = torch.Generator(device='cuda').manual_seed(3)
n = 300
big = LatentCache(1, 2 * n)   # the slot "past the cache" below stays inside this allocation
big.write(torch.randn(2 * n, 576, device='cuda', generator=g).bfloat16(), torch.arange(2 * n, device='cuda'))
lc = copy.copy(big)
lc.codes, lc.scales, lc.rope = big.codes[:n], big.scales[:n], big.rope[:n]
q = (torch.randn(2, 128, 576, device='cuda', generator=g) * 0.5).bfloat16()
idx = torch.stack([torch.randperm(n, device='cuda', generator=g)[:128] for _ in range(2)]).int()
good = idx.clone()
idx[1, 5] = n + 7                                    # past the n-slot cache, inside the allocation
good[1, 5] = -1
ws = FlashWorkspace(2, 1, 'cuda')
out = mla_flash(q, idx, lc, default_scale(), 1, ws)
ref = mla_flash(q, good, lc, default_scale(), 1, FlashWorkspace(2, 1, 'cuda'))
torch.cuda.synchronize()
assert int(ws.err) == 2, int(ws.err)
assert torch.equal(out, ref)
print('ok')
"""
    env = dict(os.environ, XTIER_DEBUG_BOUNDS='1')
    r = subprocess.run([sys.executable, '-c', code], env=env, capture_output=True, text=True, timeout=300,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0 and 'ok' in r.stdout, r.stdout + r.stderr
