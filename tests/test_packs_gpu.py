"""Model-pack kernels (csrc/cuda/packs.cu) against plain PyTorch: the DeepSeek V4 mHC post-mix bit for bit, the V4
wo_a grouped projection over FP8 (32 x 32 block scales) and BF16 weights, and the Qwen4-exp hyper-connection mix."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('M,H', [(1, 4096), (7, 1024), (500, 7168)])
def test_mhc_post_bit_exact(cuda_ops, M, H):
    from xtier_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(M + H)
    x = torch.randn(M, H, device='cuda', generator=g).bfloat16()
    res = torch.randn(M, 4, H, device='cuda', generator=g).bfloat16()
    post = torch.randn(M, 4, device='cuda', generator=g)
    comb = torch.randn(M, 4, 4, device='cuda', generator=g)
    out = ops.mhc_post(x, res, post, comb)
    torch.cuda.synchronize()
    r = res.float()
    m = [comb[:, j, :, None] * r[:, j, None, :] for j in range(4)]     # [M, 4 (out i), H]
    ref = (post[:, :, None] * x.float()[:, None, :] + (((m[0] + m[1]) + m[2]) + m[3])).bfloat16()
    assert torch.equal(out, ref)


@pytest.mark.parametrize('T,G,R,D,fp8', [(1, 8, 1024, 4096, True), (6, 4, 256, 1024, True), (20, 2, 64, 512, True),
                                          (6, 4, 256, 1024, False)])
def test_wo_a_vs_fp32(cuda_ops, T, G, R, D, fp8):
    from xtier_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(T * 7 + R)
    big = torch.randn(T, G, D + 64, device='cuda', generator=g).bfloat16()
    o = big[:, :, :D]                                      # a strided view, as the attention output hands it over
    if fp8:
        w = (torch.randn(G, R, D, device='cuda', generator=g) * 2).to(torch.float8_e4m3fn)
        e = torch.randint(-9, -4, (G * R // 32, D // 32), device='cuda', generator=g).float()
        scale = torch.exp2(e)
        wf = w.float().view(G * R, D) * scale.repeat_interleave(32, 0).repeat_interleave(32, 1)
        wf = wf.view(G, R, D)
        out = ops.wo_a(o, w, scale)
    else:
        w = (torch.randn(G, R, D, device='cuda', generator=g) * 0.02).bfloat16()
        wf = w.float()
        out = ops.wo_a(o, w)
    torch.cuda.synchronize()
    ref = torch.einsum('tgh,grh->tgr', o.float(), wf)
    rel = float((out.float() - ref).norm() / ref.norm())
    assert rel < 4e-3, rel


@pytest.mark.parametrize('rows,hc,hs,L', [(1, 4, 2048, 512), (4, 4, 1024, 256), (20, 2, 512, 128)])
def test_hc_mix_vs_fp32(cuda_ops, rows, hc, hs, L):
    from xtier_b200 import ops
    g = torch.Generator(device='cuda').manual_seed(rows + hs)
    x = torch.randn(rows, hc * hs, device='cuda', generator=g).bfloat16()
    wd = (torch.randn(L, hc * hs, device='cuda', generator=g) * 0.02).bfloat16()
    wu = (torch.randn(hc * hs, L, device='cuda', generator=g) * 0.05).bfloat16()
    out = ops.hc_mix(x, wd, wu, hc)
    torch.cuda.synchronize()
    a = (x.float() @ wd.float().t()) / hc
    t = (a * torch.sigmoid(a)).bfloat16().float()
    gate = torch.sigmoid(t @ wu.float().t()).view(rows, hc, hs)
    ref = (gate * x.float().view(rows, hc, hs)).sum(1) / hc
    rel = float((out.float() - ref).norm() / ref.norm())
    assert rel < 1e-2, rel
