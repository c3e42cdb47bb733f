"""Prefix reuse on the GPU: a prefill that starts after a cached prefix gives the logits of a prefill of the whole
prompt, and the server backend's second request with a shared prefix computes only the new ids."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def test_continuation_prefill_matches_the_whole(cuda_ops):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    cfg = Qwen3MoeConfig.tiny(std=0.05)
    model = Qwen3MoeModel(cfg, device='cuda', seed=4, synthetic_experts=False)
    ids = torch.randint(0, cfg.vocab, (48,), generator=torch.Generator().manual_seed(5)).cuda()
    st1 = model.alloc_state(1, 128)
    _, whole = model.prefill(st1, ids, return_logits=True)
    st2 = model.alloc_state(1, 128)
    model.prefill(st2, ids[:30])
    _, part = model.prefill(st2, ids[30:], start=30, return_logits=True)
    assert _rel(part, whole) < 1e-2, _rel(part, whole)


def test_server_backend_reuses_the_prefix(cuda_ops):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    from xtier_b200.serve import GenBackend
    cfg = Qwen3MoeConfig.tiny()
    model = Qwen3MoeModel(cfg, device='cuda', seed=0)
    be = GenBackend(model, Generator(model, 1, 256))
    p = torch.randint(0, cfg.vocab, (40,), generator=torch.Generator().manual_seed(1)).tolist()
    out = [be.prefill(p)] + [be.decode() for _ in range(5)]
    assert be.reusable(p + out + [3, 4]) == len(p) + len(out) - 1
    first = be.prefill(p + out + [3, 4])
    assert be.reused == len(p) + len(out) - 1 and 0 <= first < cfg.vocab
