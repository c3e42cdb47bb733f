"""Temperature / top-p sampling on the CPU: each row's draws follow the nucleus distribution of its logits, rows with
temperature 0 take the argmax, and a seeded generator repeats its draws."""
import torch

from xtier_b200.runtime.sampling import nucleus_probs, sample


def _empirical(logits, temp, top_p, n=40000, seed=0):
    g = torch.Generator().manual_seed(seed)
    rows = logits[None].expand(n, -1)
    ids = sample(rows, torch.full((n,), temp), torch.full((n,), top_p), generator=g)
    return torch.bincount(ids, minlength=logits.shape[0]).double() / n


def test_distribution_matches_the_nucleus():
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(12, generator=g) * 2
    for temp, top_p in [(1.0, 1.0), (0.7, 1.0), (1.0, 0.8), (1.3, 0.5)]:
        want = nucleus_probs(logits, temp, top_p)
        got = _empirical(logits, temp, top_p)
        assert float((got - want).abs().max()) < 0.012, (temp, top_p)
        assert float(got[want == 0].sum()) == 0.0            # nothing outside the nucleus


def test_greedy_rows_and_mixed_batches():
    g = torch.Generator().manual_seed(2)
    logits = torch.randn(5, 30, generator=g)
    temp = torch.tensor([0.0, 1.0, 0.0, 0.5, 0.0])
    out = torch.empty(5, dtype=torch.int64)
    sample(logits, temp, torch.ones(5), out=out, generator=g)
    greedy = torch.argmax(logits, -1)
    assert torch.equal(out[temp == 0], greedy[temp == 0])
    tiny = sample(logits, torch.ones(5), torch.full((5,), 1e-6), generator=g)   # top_p -> 0 keeps only the best
    assert torch.equal(tiny, greedy)
    a = sample(logits, torch.ones(5), torch.ones(5), generator=torch.Generator().manual_seed(9))
    b = sample(logits, torch.ones(5), torch.ones(5), generator=torch.Generator().manual_seed(9))
    assert torch.equal(a, b)
