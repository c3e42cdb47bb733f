"""Continuous batching on the GPU: a request decoded in row 0 of the captured 3-row step gets the same tokens
whether another request runs in row 1 or the other rows are parked."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_rows_are_independent(cuda_ops):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    from xtier_b200.serve import BatchBackend
    cfg = Qwen3MoeConfig.tiny()
    model = Qwen3MoeModel(cfg, device='cuda', seed=0)
    be = BatchBackend(model, Generator(model, batch=3, max_len=128))
    be.capture()
    g = torch.Generator().manual_seed(2)
    a = torch.randint(0, cfg.vocab, (30,), generator=g).tolist()
    b = torch.randint(0, cfg.vocab, (17,), generator=g).tolist()
    alone = [be.prefill_row(0, a)]
    for _ in range(10):
        alone.append(be.step([0])[0])
    both_a = [be.prefill_row(0, a)]
    both_b = [be.prefill_row(1, b)]
    for _ in range(10):
        t = be.step([0, 1])
        both_a.append(t[0])
        both_b.append(t[1])
    assert both_a == alone
    assert all(0 <= t < cfg.vocab for t in both_b)
