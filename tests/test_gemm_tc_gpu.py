"""tcgen05/TMEM/TMA BF16 GEMM vs an fp32 PyTorch matmul (B200 only)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize('M,N,K', [(128, 256, 64), (256, 2048, 512), (300, 1000, 200), (1, 4096, 2048),
                                   (2048, 5120, 2048), (777, 2304, 4096), (4096, 4096, 4096)])
def test_gemm_tc(cuda_ops, M, N, K):
    torch.manual_seed(M + N + K)
    a = torch.randn(M, K, device='cuda').bfloat16()
    b = (torch.randn(N, K, device='cuda') * K ** -0.5).bfloat16()
    out = torch.full((M, N), float('nan'), device='cuda', dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    torch.ops.xtier.gemm_tc(a, b, None, out, err)
    torch.cuda.synchronize()
    assert int(err) == 0
    ref = a.float() @ b.float().T
    assert _rel(out, ref) < 1e-2, _rel(out, ref)
    r = torch.randn(M, N, device='cuda').bfloat16()
    torch.ops.xtier.gemm_tc(a, b, r, out, err)
    assert _rel(out, ref + r.float()) < 1e-2


def test_gemm_tc_repeated_and_in_graph(cuda_ops):
    a = torch.randn(512, 1024, device='cuda').bfloat16()
    b = torch.randn(3072, 1024, device='cuda').bfloat16()
    out = torch.empty(512, 3072, device='cuda', dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    torch.ops.xtier.gemm_tc(a, b, None, out, err)
    first = out.clone()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        torch.ops.xtier.gemm_tc(a, b, None, out, err)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(g):
        torch.ops.xtier.gemm_tc(a, b, None, out, err)
    for _ in range(3):
        out.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, first) and int(err) == 0
