"""Parallel encoding of long prompts with a Hugging Face fast tokenizer.

A fast tokenizer encodes one text on one CPU core (a 500K-character prompt takes over a second); a batch of texts is
encoded by its Rust engine on all cores. `parallel_encode` cuts a long text into slices at positions where the
byte-level BPE pre-tokenizers of the supported model families always start a new pre-token -- right after a newline
that is followed by an ASCII letter or digit -- and never inside an added token that contains a newline, encodes the
slices as one batch without special tokens and concatenates the ids: the same ids as encoding the whole text.
`supported(tok)` checks the property on a probe text once per tokenizer; an unsupported tokenizer (or a short text)
is encoded in one piece.
(Reference parity: xtier/platform.py `_try_parallel_bpe_encode` -- the split rule and the one-time probe.)
"""
from __future__ import annotations

import re

_SPLIT = re.compile(r'\n(?=[A-Za-z0-9])')
_PROBE = ('def f(x):\n    return x\nclass A:\n  pass\nThe end.\n\nimport os\n# comment\n12 apples\n\tz = 1\n'
          'naïve café\nx\n')


def _cuts(text: str, target: int, guarded) -> list[int]:
    cuts, last = [], 0
    for m in _SPLIT.finditer(text):
        pos = m.end()
        if pos - last >= target and not any(a < pos < b for a, b in guarded):
            cuts.append(pos)
            last = pos
    return cuts


def _guarded(tok, text: str) -> list[tuple[int, int]]:
    """Spans of added tokens that contain a newline (a cut there would split them)."""
    spans = []
    for s in (getattr(tok, 'added_tokens_encoder', None) or {}):
        if '\n' in s:
            i = text.find(s)
            while i >= 0:
                spans.append((i, i + len(s)))
                i = text.find(s, i + 1)
    return spans


def _split_encode(tok, text: str, target: int) -> list[int]:
    cuts = _cuts(text, target, _guarded(tok, text))
    if not cuts:
        return tok(text, add_special_tokens=False)['input_ids']
    bounds = [0] + cuts + [len(text)]
    pieces = [text[a:b] for a, b in zip(bounds, bounds[1:])]
    out: list[int] = []
    for ids in tok(pieces, add_special_tokens=False)['input_ids']:
        out += ids
    return out


def supported(tok) -> bool:
    """Whether cutting at the split rule gives the same ids on a probe text (cached on the tokenizer)."""
    ok = getattr(tok, '_xtier_parallel_ok', None)
    if ok is None:
        try:
            ok = bool(getattr(tok, 'is_fast', False)) and \
                _split_encode(tok, _PROBE * 4, 1) == tok(_PROBE * 4, add_special_tokens=False)['input_ids']
        except Exception:   # noqa: BLE001 -- any tokenizer that cannot batch is encoded in one piece
            ok = False
        try:
            tok._xtier_parallel_ok = ok
        except AttributeError:
            pass
    return ok


def parallel_encode(tok, text: str, target_chars: int = 16384) -> list[int]:
    """Ids of `text` without special tokens; slices of about `target_chars` characters encoded as one batch when the
    tokenizer supports it and the text is long."""
    if len(text) < 4 * target_chars or not supported(tok):
        return tok(text, add_special_tokens=False)['input_ids'] if callable(tok) else tok.encode(
            text, add_special_tokens=False)
    return _split_encode(tok, text, target_chars)
