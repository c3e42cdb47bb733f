"""Sparse GQA attention over an NVFP4 KV cache (QSA / MiniMax decode shape): the cache writer against the FP32 values
it encodes, and the split-key decode against an FP32 PyTorch attention over the dequantized cache -- Qwen4-exp's 24
query / 2 KV heads of dim 256 and a 128-dim 8-group shape, selections with unused (-1) entries and a query with no key."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize('Hq,Hkv,D,nsel', [(24, 2, 256, 300), (64, 8, 128, 2048)])
def test_qsa_decode_matches_fp32(cuda_ops, Hq, Hkv, D, nsel):
    from xtier_b200.attention import qsa
    g = torch.Generator(device='cuda').manual_seed(3)
    B, L = 3, 2304
    cache = qsa.KvCacheFP4(B, L, Hkv, D)
    k = torch.randn(B * L, Hkv, D, device='cuda', generator=g).bfloat16()
    v = torch.randn(B * L, Hkv, D, device='cuda', generator=g).bfloat16()
    cache.write(k, v, torch.arange(B * L, device='cuda'))
    # the cache holds the NVFP4 encoding of the rows: the dequantized values track them (E2M1: ~12 % relative error)
    kd, vd = cache.dequant(torch.arange(B * L, device='cuda'))
    assert _rel(kd, k) < 0.2 and _rel(vd, v) < 0.2
    idx = torch.full((B, nsel), -1, dtype=torch.int32, device='cuda')
    for b in range(B - 1):   # distinct slots of the query's own row; the tail left empty; the last query has none
        n = nsel - 37 * (b + 1)
        idx[b, :n] = (torch.randperm(L, device='cuda', generator=g)[:n] + b * L).int()
    q = torch.randn(B, Hq, D, device='cuda', generator=g).bfloat16()
    scale = D ** -0.5
    out = qsa.qsa_decode(q, idx, cache, scale)
    torch.cuda.synchronize()
    ref = qsa.reference(q, idx, cache, scale)
    assert _rel(out[:B - 1], ref[:B - 1]) < 1e-2, _rel(out[:B - 1], ref[:B - 1])
    assert float(out[B - 1].float().abs().max()) == 0.0
