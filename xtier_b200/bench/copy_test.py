"""Verbatim-copy test of a running `xtier_b200.serve` with a real instruction-tuned checkpoint and its tokenizer: the
model must echo windows of a source file exactly (greedy). Any changed span points at the decode path.

    python -m xtier_b200.bench.copy_test --url URL --tokenizer DIR --source FILE [--chunks 8] [--lines 90]
        [--ignore-first-indent] [--out FILE]

The prompt is the tokenizer's chat template around an instruction and the window between <src> tags (thinking off
where the template has the switch); generation stops at the template's end-of-turn ids. Reported per window: the
differing spans (difflib opcodes); overall: how many windows differ. Exit status 1 when any does.
(Reference parity: bench/copy_test.py.)
"""
from __future__ import annotations

import argparse
import difflib
import json
import sys
from pathlib import Path

from .client import Client

INSTRUCTION = ('Output the text between <src> and </src> exactly as it is, character for character: add, remove or '
               'change nothing, no code fences, no explanation.')


def windows(text: str, count: int = 8, lines: int = 90) -> list[str]:
    rows = text.splitlines()
    if len(rows) <= lines:
        return [text] if text.strip() else []
    step = max(1, (len(rows) - lines) // max(1, count))
    out = []
    for i in range(count):
        w = '\n'.join(rows[i * step:i * step + lines])
        if w.strip():
            out.append(w)
    return out


def chat_ids(tok, content: str) -> list[int]:
    msgs = [{'role': 'user', 'content': content}]
    try:
        return list(tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True,
                                            enable_thinking=False))
    except TypeError:
        return list(tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=True))


def compare(src: str, out: str, ignore_first_indent: bool = False) -> list:
    o = out.strip('\n')
    if o.startswith('```') and '\n' in o:
        o = o.split('\n', 1)[1].rsplit('```', 1)[0].strip('\n')
    s = src.strip('\n')
    if ignore_first_indent:
        s, o = s.lstrip(' '), o.lstrip(' ')
    return [list(op) for op in difflib.SequenceMatcher(None, s, o, autojunk=False).get_opcodes() if op[0] != 'equal']


def run(cl: Client, tok, source_text: str, chunks: int = 8, lines: int = 90, ignore_first_indent: bool = False,
        log=print) -> dict:
    st, info = cl.request('GET', '/health')
    stop = [t for t in {getattr(tok, 'eos_token_id', None)} if t is not None]
    rows = []
    for w in windows(source_text, chunks, lines):
        ids = chat_ids(tok, f'{INSTRUCTION}\n<src>\n{w}\n</src>')
        n = min(len(tok.encode(w, add_special_tokens=False)) + 64, info['max_len'] - len(ids) - 16)
        if n < 8:
            log(json.dumps(dict(skipped='window longer than the server max length')))
            continue
        got = cl.generate(ids, n, stop_ids=stop)['ids']
        got = [t for t in got if t not in stop]
        out = tok.decode(got, skip_special_tokens=True)
        diffs = compare(w, out, ignore_first_indent)
        rows.append(dict(expected=w, actual=out, diffs=diffs))
        log(json.dumps(dict(window=len(rows) - 1, differs=bool(diffs), spans=len(diffs))))
    bad = sum(1 for r in rows if r['diffs'])
    return dict(test='copy', windows=len(rows), differ=bad, rows=rows)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--url', default='http://127.0.0.1:18180')
    ap.add_argument('--tokenizer', required=True)
    ap.add_argument('--source', required=True)
    ap.add_argument('--chunks', type=int, default=8)
    ap.add_argument('--lines', type=int, default=90)
    ap.add_argument('--ignore-first-indent', action='store_true')
    ap.add_argument('--out')
    a = ap.parse_args(argv)
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(a.tokenizer)
    res = run(Client(a.url), tok, Path(a.source).read_text(encoding='utf-8'), a.chunks, a.lines,
              a.ignore_first_indent)
    print(f'COPY {res["differ"]}/{res["windows"]} windows differ')
    if a.out:
        with open(a.out, 'w') as f:
            json.dump(res, f, ensure_ascii=False, indent=1)
    return 1 if res['differ'] else 0


if __name__ == '__main__':
    sys.exit(main())
