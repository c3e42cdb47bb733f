"""Dense MXFP8 GEMM (csrc/cuda/gemm_mx8.cu) against plain fp32 PyTorch: exactly against the product of the dequantized
operands (only the FP32 accumulation order differs), and within the E4M3 quantization error against the BF16 inputs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dequant(q8: torch.Tensor, sf: torch.Tensor) -> torch.Tensor:
    """E4M3 codes [R, K] and their scale atoms -> fp32 values (the atom layout of mx_quant_rows)."""
    R, K = q8.shape
    v = q8.view(torch.float8_e4m3fn).float()
    r = torch.arange(R, device=q8.device)[:, None]
    b = torch.arange(K // 32, device=q8.device)[None, :]
    idx = ((r // 128) * (K // 128) + b // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + b % 4
    e = sf.long()[idx].float() - 127.0
    return v * torch.exp2(e).repeat_interleave(32, 1)


@pytest.mark.parametrize('M,N,K', [(128, 128, 128), (300, 256, 512), (1000, 384, 1024), (64, 7168, 2048)])
def test_gemm_mx8_matches_fp32(cuda_ops, M, N, K):
    from xtier_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(M + N + K)
    x = torch.randn(M, K, device='cuda', generator=g).bfloat16()
    w = (torch.randn(N, K, device='cuda', generator=g) * 0.02).bfloat16()
    res = torch.randn(M, N, device='cuda', generator=g).bfloat16()
    wq = ops.MX8Weight(w)
    err = ops.gemm_error_word(x.device)
    err.zero_()
    y = ops.linear_mx8(x, wq)
    y_res = ops.linear_mx8(x, wq, residual=res)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # the quantized operands, as the kernel saw them
    Mp = (M + 127) // 128 * 128
    x8 = torch.empty(Mp, K, dtype=torch.uint8, device='cuda')
    sfx = torch.empty(Mp * K // 32, dtype=torch.uint8, device='cuda')
    xp = torch.zeros(Mp, K, device='cuda').bfloat16()
    xp[:M] = x
    torch.ops.xtier.mx_quant_rows(xp, None, x8, sfx)
    exact = _dequant(x8, sfx)[:M] @ _dequant(wq.w8, wq.sf).t()
    rel = float((y.float() - exact).norm() / exact.norm())
    assert rel < 5e-3, rel                 # BF16 output rounding only
    ref = x.float() @ w.float().t()
    rel_q = float((y.float() - ref).norm() / ref.norm())
    assert rel_q < 8e-2, rel_q             # E4M3 operands: ~3 % per element
    want = exact + res.float()
    assert float((y_res.float() - want).norm() / want.norm()) < 5e-3
