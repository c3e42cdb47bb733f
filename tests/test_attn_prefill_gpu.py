"""Causal GQA prefill attention on the tcgen05 tensor cores (csrc/cuda/attn_prefill.cu) against a plain fp32 PyTorch
reference of the same op: first chunks and continuation chunks, partial tiles, GQA groups, strided query / output
views."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(q, k, v, row, start):
    """q [T, Hq, D], caches [B, Hkv, L, D] -> [T, Hq, D] fp32; query t sees keys 0 .. start + t."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    n = start + T
    kk = k[row, :, :n].float().repeat_interleave(Hq // Hkv, 0)        # [Hq, n, D]
    vv = v[row, :, :n].float().repeat_interleave(Hq // Hkv, 0)
    s = torch.einsum('thd,hnd->htn', q.float(), kk) / math.sqrt(D)
    mask = torch.arange(n, device=q.device)[None, :] > (start + torch.arange(T, device=q.device))[:, None]
    s = s.masked_fill(mask[None], float('-inf'))
    return torch.einsum('htn,hnd->thd', torch.softmax(s, -1), vv)


def _cache(B, Hkv, L, seed):
    g = torch.Generator(device='cuda').manual_seed(seed)
    k = torch.randn(B, Hkv, L, 128, generator=g, device='cuda').bfloat16()
    v = torch.randn(B, Hkv, L, 128, generator=g, device='cuda').bfloat16()
    return k, v


@pytest.mark.parametrize('T,start,Hq,Hkv,row', [
    (1, 0, 8, 2, 0), (100, 0, 8, 2, 1), (256, 0, 16, 2, 0), (700, 0, 32, 4, 1), (300, 77, 8, 8, 0),
    (1, 1000, 8, 1, 1), (513, 1111, 16, 4, 0)])
def test_attn_prefill_matches_fp32(cuda_ops, T, start, Hq, Hkv, row):
    from xtier_b200 import ops
    k, v = _cache(2, Hkv, 2048, seed=T + start)
    q = torch.randn(T, Hq, 128, device='cuda').bfloat16()
    err = ops.gemm_error_word(q.device)
    err.zero_()
    out = ops.attn_prefill(q, k, v, row, start, 1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = _reference(q, k, v, row, start)
    rel = float((out.float() - ref).norm() / ref.norm())
    assert rel < 1e-2, rel
    assert torch.isfinite(out.float()).all()


def test_attn_prefill_strided_views(cuda_ops):
    """q as a slice of a fused qkv row, out written into the [T, Hq * 128] input of the output projection."""
    from xtier_b200 import ops
    T, Hq, Hkv = 333, 16, 4
    k, v = _cache(1, Hkv, 1024, seed=5)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device='cuda').bfloat16()
    q = qkv[:, :Hq * 128].view(T, Hq, 128)
    flat = torch.full((T, Hq * 128), float('nan'), device='cuda').bfloat16()
    ops.attn_prefill(q, k, v, 0, 0, 1.0 / math.sqrt(128), out=flat.view(T, Hq, 128))
    torch.cuda.synchronize()
    ref = _reference(q, k, v, 0, 0).reshape(T, -1)
    assert float((flat.float() - ref).norm() / ref.norm()) < 1e-2


def test_attn_prefill_long_against_sdpa(cuda_ops):
    """8K causal tokens (many key tiles, the lazy rescale path) against PyTorch's fused attention in fp32."""
    from xtier_b200 import ops
    T, Hq, Hkv = 8192, 8, 1
    k, v = _cache(1, Hkv, T, seed=9)
    q = (torch.randn(T, Hq, 128, device='cuda') * 2).bfloat16()
    out = ops.attn_prefill(q, k, v, 0, 0, 1.0 / math.sqrt(128))
    ref = torch.nn.functional.scaled_dot_product_attention(
        q.float().transpose(0, 1)[None], k[:, :, :T].float().repeat_interleave(Hq // Hkv, 1),
        v[:, :, :T].float().repeat_interleave(Hq // Hkv, 1), is_causal=True)[0].transpose(0, 1)
    torch.cuda.synchronize()
    assert float((out.float() - ref).norm() / ref.norm()) < 1e-2
