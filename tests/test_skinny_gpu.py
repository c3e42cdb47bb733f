"""Skinny tcgen05 GEMM (decode projections, M <= 32 rows) against the fp32 PyTorch product: one and several K splits,
weight-row counts that are not multiples of 128, the fused residual add, and routing through ops.linear."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('M,N,K', [(1, 2112, 7168), (4, 576, 1536), (8, 7168, 16384), (16, 300, 512),
                                   (17, 1000, 2048), (32, 4096, 1024)])
def test_skinny_gemm_matches_fp32(cuda_ops, M, N, K):
    from xtier_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(M * 131 + N)
    x = torch.randn(M, K, device='cuda', generator=g).bfloat16()
    w = (torch.randn(N, K, device='cuda', generator=g) * K ** -0.5).bfloat16()
    add = torch.randn(M, N, device='cuda', generator=g).bfloat16()
    ref = x.float() @ w.float().t()
    y = ops.skinny_gemm(x, w)
    assert int(ops.gemm_error_word(x.device)) == 0
    assert float((y.float() - ref).abs().max()) <= 0.02 * float(ref.abs().max()) + 1e-3
    assert float((y.float() - ref).norm() / ref.norm()) < 8e-3
    y2 = ops.skinny_gemm(x, w, add=add)
    assert float((y2.float() - (ref + add.float())).norm() / (ref + add.float()).norm()) < 8e-3
    if M >= 3:
        assert torch.equal(ops.linear(x, w), y)   # routed through the skinny GEMM, deterministic


def test_skinny_gemm_deterministic_across_calls(cuda_ops):
    from xtier_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(7)
    x = torch.randn(8, 16384, device='cuda', generator=g).bfloat16()
    w = torch.randn(7168, 16384, device='cuda', generator=g).bfloat16()
    a = ops.skinny_gemm(x, w)
    for _ in range(3):
        assert torch.equal(ops.skinny_gemm(x, w), a)
