"""Speculative decoding on the host: the chain verifier's output distribution equals the target's (lossless), greedy
verification returns the target's greedy tokens, and the truncation rule's plain-PyTorch oracle."""
import torch

from xtier_b200.runtime.speculative import truncate_reference, verify_chain


def test_verify_chain_is_lossless():
    V, S, N = 6, 3, 20000
    g = torch.Generator().manual_seed(0)
    p = torch.softmax(torch.randn(S + 1, V, generator=g) * 1.5, -1)
    q = torch.softmax(torch.randn(S, V, generator=g) * 1.5, -1)
    first = torch.zeros(V)
    for _ in range(N):
        drafts = torch.stack([torch.multinomial(q[j], 1, generator=g)[0] for j in range(S)])
        out = verify_chain(p, q, drafts, g)
        assert 1 <= len(out) <= S + 1
        first[out[0]] += 1
    emp = first / N
    assert float((emp - p[0]).abs().max()) < 0.015, (emp, p[0])


def test_verify_zero_q_row_never_accepts():
    V = 5
    p = torch.softmax(torch.randn(3, V), -1)
    q = torch.softmax(torch.randn(2, V), -1)
    q[1] = 0                                   # truncated at the second draft
    g = torch.Generator().manual_seed(1)
    for _ in range(200):
        out = verify_chain(p, q, torch.tensor([int(torch.argmax(q[0])), 2]), g)
        assert len(out) <= 2                   # the second draft is never accepted


def test_greedy_verify():
    p = torch.zeros(4, 8)
    p[0, 3] = p[1, 5] = p[2, 1] = p[3, 7] = 1
    assert verify_chain(p, torch.zeros(3, 8), torch.tensor([3, 5, 1]), greedy=True) == [3, 5, 1, 7]
    assert verify_chain(p, torch.zeros(3, 8), torch.tensor([3, 4, 1]), greedy=True) == [3, 5]


def test_truncate_reference_rule():
    q = torch.full((2, 4, 10), 0.05)
    tokens = torch.tensor([[0, 1, 2, 3, 4], [0, 5, 6, 7, 8]])
    q[0, 0, 1], q[0, 1, 2], q[0, 2, 3] = 0.9, 0.5, 0.1       # third draft under 0.2
    q[1, 0, 5] = 0.1                                          # first draft low: keep one anyway
    q2, flags = truncate_reference(q, tokens, 0.2)
    assert flags.tolist() == [[1, 1, 1, 0, 0], [1, 1, 0, 0, 0]]
    assert float(q2[0, 2].abs().sum()) == 0 and float(q2[1, 1].abs().sum()) == 0
    _, fg = truncate_reference(q, tokens, 0.2, greedy=True)
    assert fg.tolist() == [[1] * 5, [1] * 5]


class _Bigram:
    """Stand-in model: a position's logits depend on its token only; `cols` restricts the head (a hot vocabulary)."""

    def __init__(self, W, cols=None):
        self.W = W if cols is None else W[:, cols]
        self.vocab = W.shape[1]
        self.device = torch.device('cpu')

    def alloc_state(self, b, n):
        return {}

    def prefill(self, st, tokens, start=0, return_logits=False, all_logits=False, active=None):
        lg = self.W[tokens.long()]
        nxt = torch.argmax(lg, -1)
        if all_logits:
            return nxt, lg
        return (nxt[-1:], lg[-1]) if return_logits else nxt[-1:]


def test_hot_vocab_draft_is_scattered_and_lossless():
    from xtier_b200.runtime.speculative import SpeculativeDecoder
    g = torch.Generator().manual_seed(4)
    V = 48
    W = torch.randn(V, V, generator=g) * 3
    hot = torch.randperm(V, generator=g)[:20]
    W[:, hot] += 2.0                                   # the hot tokens carry most of the mass
    target = _Bigram(W)
    draft = _Bigram(W + 0.3 * torch.randn(V, V, generator=g), cols=hot)   # a close model over the hot vocab
    prompt = torch.tensor([1, 2, 3])
    seq = [3]
    for _ in range(30):
        seq.append(int(torch.argmax(W[seq[-1]])))
    sd = SpeculativeDecoder(target, draft, steps=4, threshold=0.0, hot_ids=hot)
    assert sd.generate(prompt, 30) == seq[1:]          # greedy: the target's own tokens
    assert sd.stats['accepted'] > 0
    # the scattered q: a distribution over the target vocabulary that is zero outside the hot ids
    q = sd.draft_probs(torch.randn(len(hot), generator=g), V)
    outside = torch.ones(V, dtype=torch.bool)
    outside[hot] = False
    assert abs(float(q.sum()) - 1) < 1e-6 and float(q[outside].abs().max()) == 0
    sd = SpeculativeDecoder(target, draft, steps=4, threshold=0.0, hot_ids=hot, temperature=1.0, seed=2,
                            draft_temp_scale=0.8)
    out = sd.generate(prompt, 40)
    assert len(out) == 40 and all(0 <= t < V for t in out)
    assert 0.8 * 1.0 == sd.temp * sd.draft_scale


def test_hot_vocab_verify_matches_target_distribution():
    """verify_chain with a scattered q (zero outside the hot ids) keeps the target's distribution."""
    g = torch.Generator().manual_seed(7)
    V, N = 8, 20000
    hot = torch.tensor([1, 4, 6])
    p = torch.softmax(torch.randn(2, V, generator=g), -1)
    qh = torch.softmax(torch.randn(1, 3, generator=g), -1)
    q = torch.zeros(1, V)
    q[:, hot] = qh
    first = torch.zeros(V)
    for _ in range(N):
        d = hot[torch.multinomial(qh[0], 1, generator=g)]
        out = verify_chain(p, q, d, g)
        first[out[0]] += 1
    assert float((first / N - p[0]).abs().max()) < 0.015


def test_top_p_nucleus_in_verification_probs():
    from xtier_b200.runtime.sampling import nucleus_probs
    from xtier_b200.runtime.speculative import SpeculativeDecoder
    g = torch.Generator().manual_seed(3)
    W = torch.randn(16, 16, generator=g) * 2
    sd = SpeculativeDecoder(_Bigram(W), _Bigram(W), threshold=0.0, temperature=0.9)
    sd.top_p = 0.7
    logits = torch.randn(3, 16, generator=g)
    got = sd._probs(logits)
    for r in range(3):
        assert torch.allclose(got[r].double(), nucleus_probs(logits[r], 0.9, 0.7), atol=1e-6)
