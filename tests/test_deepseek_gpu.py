"""DeepSeek-V3-shaped model (tiny shape): the absorbed MLA decode over the latent cache agrees with the expanded
prefill of the same sequence, with grouped-sigmoid MXFP4 MoE layers, a shared expert and a dense first layer."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_mla_decode_matches_prefill_recompute(cuda_ops):
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Config, DeepSeekV3Model
    cfg = DeepSeekV3Config.tiny()
    model = DeepSeekV3Model(cfg, device='cuda', seed=3)
    toks = torch.randint(0, cfg.vocab, (20,), generator=torch.Generator().manual_seed(1)).cuda()
    st = model.alloc_state(1, 64)
    model.prefill(st, toks[:19])
    rows = torch.zeros(1, dtype=torch.int32, device='cuda')
    pos = st['lengths'][rows.long()].clone()
    logits_dec = model.forward(st, toks[19:20], rows, pos, decode=True)
    st2 = model.alloc_state(1, 64)
    T = 20
    logits_pre = model.forward(st2, toks, torch.zeros(T, dtype=torch.int32, device='cuda'),
                               torch.arange(T, dtype=torch.int32, device='cuda'), decode=False)
    assert _rel(logits_dec[0], logits_pre[0]) < 3e-2, _rel(logits_dec[0], logits_pre[0])


def test_gemm_linear_dispatch_large_m(cuda_ops):
    x = torch.randn(300, 512, device='cuda').bfloat16()
    w = (torch.randn(768, 512, device='cuda') * 0.05).bfloat16()
    y = cuda_ops.linear(x, w)
    assert _rel(y, x.float() @ w.float().T) < 1e-2
    assert int(cuda_ops.gemm_error_word('cuda')) == 0
