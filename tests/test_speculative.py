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
