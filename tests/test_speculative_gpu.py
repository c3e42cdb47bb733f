"""Speculative decoding on the GPU: the truncation kernel against its PyTorch oracle, token flags in the MoE router
(a flagged-off token skips its routed experts), a continuation prefill chunk (causal over the cached prefix), and
chain speculative decoding whose greedy output equals the target model's own greedy decoding."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_truncate_kernel_matches_reference(cuda_ops):
    from xtier_b200.runtime.speculative import truncate, truncate_reference
    g = torch.Generator().manual_seed(0)
    B, S, V = 5, 4, 1000
    q = torch.softmax(torch.randn(B, S, V, generator=g) * 4, -1)
    tokens = torch.randint(0, V, (B, S + 1), generator=g)
    tokens[:, 1:] = torch.argmax(q, -1)                     # drafts = the draft's own argmax (mixed confidences)
    for greedy in (False, True):
        qd = q.cuda()
        flags = truncate(qd, tokens.cuda(), 0.2, greedy=greedy)
        torch.cuda.synchronize()
        qr, fr = truncate_reference(q, tokens, 0.2, greedy=greedy)
        assert torch.equal(flags.cpu(), fr)
        assert torch.equal(qd.cpu(), qr)


def test_token_flags_skip_routed_experts(cuda_ops):
    from xtier_b200 import formats
    from xtier_b200.cache.pool import TieredMoE
    E, H, I, k = 8, 256, 128, 2
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=3, std=0.05)
    router = (torch.randn(E, H) * 0.02).bfloat16()
    layer = TieredMoE(0, router, ex, k, device='cuda')
    x = torch.randn(3, H).bfloat16().cuda()
    add = torch.randn(3, H).bfloat16().cuda()
    active = torch.tensor([1, 0, 1], dtype=torch.int32, device='cuda')
    out = layer.forward(x, add=add, active=active)
    torch.cuda.synchronize()
    ids = layer.ids[:3, :k].cpu()
    assert bool((ids[1] == -1).all()) and bool((ids[[0, 2]] >= 0).all())
    assert torch.equal(out[1].cpu(), add[1].cpu())         # no routed expert: the residual only
    ref = formats.reference_moe(x.cpu(), ids, layer.w[:3, :k].cpu(), ex) + add.cpu().float()
    rel = float((out[[0, 2]].cpu().float() - ref[[0, 2]]).norm() / ref[[0, 2]].norm())
    assert rel < 1e-2, rel


def _tiny(seed, layers=2):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    cfg = Qwen3MoeConfig.tiny(std=0.05, hidden=256, inter=128)
    cfg.layers = layers
    return Qwen3MoeModel(cfg, device='cuda', seed=seed, hot_fraction=1.0, synthetic_experts=False)


def test_continuation_prefill_is_causal(cuda_ops):
    model = _tiny(11)
    prompt = torch.randint(0, model.cfg.vocab, (40,), generator=torch.Generator().manual_seed(1)).cuda()
    st = model.alloc_state(1, 64)
    model.prefill(st, prompt[:24])
    _, lp = model.prefill(st, prompt[24:], start=24, return_logits=True)
    ref = model.reference_logits(prompt)
    rel = float((lp.float() - ref.float()).norm() / ref.float().norm())
    assert rel < 3e-2, rel


def test_speculative_greedy_equals_target_greedy(cuda_ops):
    from xtier_b200.runtime.speculative import SpeculativeDecoder
    target = _tiny(21)
    draft = _tiny(21, layers=1)          # the target's first layer and head: a cheap, often-right draft
    prompt = torch.randint(0, target.cfg.vocab, (12,), generator=torch.Generator().manual_seed(2)).cuda()
    st = target.alloc_state(1, 128)
    want = []
    nxt = target.prefill(st, prompt)
    pos = prompt.shape[0]
    for _ in range(20):
        want.append(int(nxt))
        nxt = target.prefill(st, nxt.view(1), start=pos)
        pos += 1
    sd = SpeculativeDecoder(target, draft, steps=4, threshold=0.2, max_len=128)
    got = sd.generate(prompt, 20)
    assert got == want, (got, want)
    assert sd.stats['rounds'] < 20                      # some drafts were accepted


def test_fp8_draft_lm_head(cuda_ops):
    """A draft whose LM head is FP8 (W8A16 GEMV in decode, W8A8 block-scaled GEMM in prefill): its logits stay close
    to the BF16 head's, its decode graph runs, and speculative greedy output still equals the target's."""
    from xtier_b200.runtime.decode import Generator
    from xtier_b200.runtime.speculative import SpeculativeDecoder
    target = _tiny(41)
    draft = _tiny(41, layers=1)
    prompt = torch.randint(0, target.cfg.vocab, (150,), generator=torch.Generator().manual_seed(7)).cuda()
    st = draft.alloc_state(1, 256)
    _, ref = draft.prefill(st, prompt, all_logits=True)               # every position: the prefill GEMM
    draft.quantize_lm_head()
    assert draft.lm_head is None and draft.lm_head_fp8 is not None
    st = draft.alloc_state(1, 256)
    _, got = draft.prefill(st, prompt, all_logits=True)
    assert float((got.float() - ref.float()).norm() / ref.float().norm()) < 8e-2
    st = draft.alloc_state(1, 256)
    _, last = draft.prefill(st, prompt, return_logits=True)           # one position: the W8A16 GEMV
    assert float((last.float() - ref[-1].float()).norm() / ref[-1].float().norm()) < 8e-2
    gen = Generator(draft, batch=1, max_len=256)
    toks = gen.generate(prompt[None].cpu(), 4)
    assert toks.shape == (1, 4)
    gen.graph = None
    want = []
    st = target.alloc_state(1, 256)
    nxt, pos = target.prefill(st, prompt[:12]), 12
    for _ in range(16):
        want.append(int(nxt))
        nxt = target.prefill(st, nxt.view(1), start=pos)
        pos += 1
    sd = SpeculativeDecoder(target, draft, steps=4, threshold=0.0, max_len=256, draft_fp8_head=True)
    assert sd.generate(prompt[:12], 16) == want
