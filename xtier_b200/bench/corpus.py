"""Fixed prompts for the bench tools: token-id segments cut deterministically from a text corpus through a tokenizer,
or, without one, from a seeded id stream (a random-init model has no tokenizer; every configuration still scores
exactly the same ids)."""
from __future__ import annotations

import random


def tokenizer(path: str | None):
    if not path:
        return None
    from transformers import AutoTokenizer
    return AutoTokenizer.from_pretrained(path)


def id_stream(n: int, vocab: int, seed: int = 0) -> list[int]:
    """n ids of a seeded stream with some repetition (short phrases recur, as in text)."""
    rng = random.Random(seed)
    phrases = [[rng.randrange(vocab) for _ in range(rng.randint(2, 12))] for _ in range(256)]
    out: list[int] = []
    while len(out) < n:
        out += phrases[rng.randrange(len(phrases))] if rng.random() < 0.6 else [rng.randrange(vocab)]
    return out[:n]


def corpus_ids(tok, path: str, limit_chars: int = 4_000_000) -> list[int]:
    with open(path, encoding='utf-8', errors='ignore') as f:
        text = f.read(limit_chars)
    return tok.encode(text, add_special_tokens=False)


def segments(count: int, length: int, vocab: int, tok=None, corpus: str | None = None, seed: int = 0):
    """`count` segments of `length` ids spread evenly over the corpus (or the seeded stream): [(index, ids)]."""
    ids = corpus_ids(tok, corpus) if (tok is not None and corpus) else id_stream(max(count, 1) * length * 2, vocab,
                                                                                  seed)
    n = min(count, max(1, len(ids) // length))
    stride = max(length, (len(ids) - length) // max(1, n))
    out = []
    for i in range(n):
        s = ids[i * stride:i * stride + length]
        if len(s) == length:
            out.append((i, s))
    return out


def prompt(length: int, vocab: int, tok=None, corpus: str | None = None, salt: int = 0) -> list[int]:
    """One prompt of `length` ids; `salt` makes it differ from every other one (nothing can be reused)."""
    if tok is not None and corpus:
        ids = corpus_ids(tok, corpus)
        head = tok.encode(f'[run {salt}]\n', add_special_tokens=False)
        off = (salt * 9973) % max(1, len(ids) - length)
        return (head + ids[off:off + length])[:length]
    return id_stream(length, vocab, seed=1_000_003 + salt)
