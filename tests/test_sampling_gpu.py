"""Temperature / top-p sampling inside the captured decode step: temperature 0 reproduces the greedy tokens, a
positive temperature draws valid tokens that leave the greedy path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_sampling_in_the_decode_graph(cuda_ops):
    from xtier_b200.models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from xtier_b200.runtime.decode import Generator
    cfg = Qwen3MoeConfig.tiny()
    model = Qwen3MoeModel(cfg, device='cuda', seed=0)
    prompt = torch.randint(0, cfg.vocab, (1, 40), generator=torch.Generator().manual_seed(3))
    want = Generator(model, 1, 128).generate(prompt, 12)
    g = Generator(model, 1, 128, sampling=True)
    g.set_sampling(0.0)
    assert torch.equal(g.generate(prompt, 12), want)
    g.set_sampling(1.5, 0.95)
    out = g.generate(prompt, 24)
    assert int(out.min()) >= 0 and int(out.max()) < cfg.vocab
    assert not torch.equal(out[:, :12], want)
    plain = Generator(model, 1, 128)
    with pytest.raises(ValueError):
        plain.set_sampling(0.7)
