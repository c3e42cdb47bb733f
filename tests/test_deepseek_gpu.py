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


def _mla_cfg(attn, **kw):
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Config
    return DeepSeekV3Config.tiny(heads=128, q_lora=256, kv_lora=512, qk_nope=128, qk_rope=64, v_head=128,
                                 layers=2, attn=attn, **kw)


def test_mla_kernel_decode_matches_torch_decode(cuda_ops):
    """Model-level: the tcgen05 MLA decode over the NVFP4 latent cache against the torch absorbed decode reading the
    same (dequantized) cached keys; and DSA with top-k >= the sequence (every key selected) against dense MLA."""
    from xtier_b200.models.deepseek_v3 import DeepSeekV3Model
    T = 40
    toks = torch.randint(0, 1000, (T,), generator=torch.Generator().manual_seed(2)).cuda()
    rows = torch.zeros(1, dtype=torch.int32, device='cuda')
    outs = {}
    for attn in ('mla', 'torch', 'dsa'):
        model = DeepSeekV3Model(_mla_cfg(attn, index_topk=128), device='cuda', seed=4)
        st = model.alloc_state(1, 512)
        model.prefill(st, toks[:T - 1])
        if attn == 'torch':   # the keys the kernel path sees: dequantized NVFP4 latent rows of the prefix
            ref_model = DeepSeekV3Model(_mla_cfg('mla'), device='cuda', seed=4)
            st_k = ref_model.alloc_state(1, 512)
            ref_model.prefill(st_k, toks[:T - 1])
            for li in range(len(model.layers)):
                deq = st_k['latent'][li].dequant(torch.arange(T - 1, device='cuda'))
                st['cache'][li][0, :T - 1] = deq.to(torch.bfloat16)
        pos = st['lengths'][rows.long()].clone()
        outs[attn] = model.forward(st, toks[T - 1:T], rows, pos, decode=True)[0].float()
        del model
    assert _rel(outs['mla'], outs['torch']) < 2e-2, _rel(outs['mla'], outs['torch'])
    assert _rel(outs['dsa'], outs['mla']) < 1e-3, _rel(outs['dsa'], outs['mla'])
