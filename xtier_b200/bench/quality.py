"""Precision checks against a running `xtier_b200.serve`: fixed-text perplexity, the distance between two
configurations' predictions, and whether a prompt's tokens depend on anything but its text.

    python -m xtier_b200.bench.quality ppl  --url URL --tag NAME [--segments 6 --tokens 4096] [--top 20]
        [--tokenizer DIR --corpus NAME=FILE ...] [--out DIR]
    python -m xtier_b200.bench.quality kl   REF.top.json TEST.top.json
    python -m xtier_b200.bench.quality flip --url URL [--cycles 12] [--prompt-len 512] [--tokens 64]

ppl: segments cut deterministically from each corpus (or the seeded id stream), each scored as a cold prefill through
/v1/logprobs; mean NLL and PPL per corpus and overall, per-segment rows, and with --top N a dump of every scored
position's N most likely tokens (DIR/NAME.top.json). kl: per scored position of two dumps of the same segments (the
reference first), KL(reference || test) over the tokens both list, the rest of each distribution merged into one
outcome -- merging outcomes never raises a KL (log-sum inequality), so this is a lower bound of the full KL, tight when
the N tokens carry most of the mass; reported: mean, 99th percentile, share of positions whose most likely token
changed, mean NLL difference. flip: the same prompt --cycles times, cache flushed each time, greedy; the generated
ids and their logprobs must be identical across cycles (this framework's kernels sum in a fixed order).
(Reference parity: bench/ppl_eval.py, bench/kl_compare.py, bench/token_flip.py.)
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import zlib

from . import corpus
from .client import Client


# ---------------------------------------------------------------------------------------------------- ppl
def ppl(cl: Client, tag: str, segments: int = 6, tokens: int = 4096, top: int = 0, tok=None, corpora=None,
        log=print) -> tuple[dict, dict | None]:
    st, info = cl.request('GET', '/health')
    if st != 200 or not info.get('ready'):
        raise SystemExit(f'server not ready: {info}')
    tokens = min(tokens, info['max_len'] - 16)
    sources = corpora or {'ids': None}
    rows, dumps = [], []
    for name, path in sources.items():
        seed = zlib.crc32(name.encode()) & 0xFFFF
        for i, ids in corpus.segments(segments, tokens, info['vocab'], tok, path, seed=seed):
            cl.flush()
            r = cl.logprobs(ids, top)
            nll = sum(r['nll']) / len(r['nll'])
            rows.append(dict(corpus=name, seg=i, n=len(r['nll']), nll=round(nll, 6)))
            log(json.dumps(rows[-1]))
            if top:
                dumps.append(dict(corpus=name, seg=i, lp=[round(-x, 6) for x in r['nll']],
                                  top=[[[int(t), round(lp, 6)] for t, lp in pos] for pos in r['top']]))
    summary = {}
    for name in list(sources) + ['all']:
        sel = [r for r in rows if name == 'all' or r['corpus'] == name]
        if sel:
            nll = sum(r['nll'] * r['n'] for r in sel) / sum(r['n'] for r in sel)
            summary[name] = dict(segments=len(sel), nll=round(nll, 5), ppl=round(math.exp(nll), 4))
    return dict(tag=tag, rows=rows, summary=summary), (dict(tag=tag, top=top, segments=dumps) if top else None)


# ---------------------------------------------------------------------------------------------------- kl
def kl_lower_bound(p_top, q_top) -> float:
    """KL(p || q) over the outcomes both top lists name plus one merged outcome for everything else; p_top / q_top:
    [[token, logprob], ...]."""
    p, q = {int(t): lp for t, lp in p_top}, {int(t): lp for t, lp in q_top}
    shared = [t for t in p if t in q]
    ps = [math.exp(p[t]) for t in shared]
    qs = [math.exp(q[t]) for t in shared]
    p_rest = max(1e-12, 1.0 - sum(ps))
    q_rest = max(1e-12, 1.0 - sum(qs))
    terms = [a * (math.log(a) - math.log(b)) for a, b in zip(ps, qs) if a > 0]
    return max(0.0, sum(terms) + p_rest * (math.log(p_rest) - math.log(q_rest)))


def kl_compare(ref: dict, test: dict) -> dict:
    key = [(s['corpus'], s['seg'], len(s['lp'])) for s in ref['segments']]
    if key != [(s['corpus'], s['seg'], len(s['lp'])) for s in test['segments']]:
        raise ValueError('the two dumps do not score the same segments')
    kls, changed, dnll, per = [], 0, 0.0, {}
    for a, b in zip(ref['segments'], test['segments']):
        acc = per.setdefault(a['corpus'], [0.0, 0])
        for la, lb, ta, tb in zip(a['lp'], b['lp'], a['top'], b['top']):
            k = kl_lower_bound(ta, tb)
            kls.append(k)
            acc[0] += k
            acc[1] += 1
            changed += max(ta, key=lambda x: x[1])[0] != max(tb, key=lambda x: x[1])[0]
            dnll += la - lb          # logprobs: reference minus test = test NLL minus reference NLL
    n = len(kls)
    srt = sorted(kls)
    return dict(ref=ref['tag'], test=test['tag'], positions=n, kl_mean=sum(kls) / n if n else 0.0,
                kl_p99=srt[int(0.99 * (n - 1))] if n else 0.0, top1_changed=changed / n if n else 0.0,
                nll_diff=dnll / n if n else 0.0, kl_by_corpus={c: s / m for c, (s, m) in per.items()})


# ---------------------------------------------------------------------------------------------------- flip
def flip(cl: Client, cycles: int = 12, prompt_len: int = 512, tokens: int = 64, log=print) -> dict:
    st, info = cl.request('GET', '/health')
    p = corpus.prompt(prompt_len, info['vocab'], salt=424242)
    runs = []
    for c in range(cycles):
        cl.flush()
        ids = cl.generate(p, tokens)['ids']
        cl.flush()
        lp = cl.logprobs(p + ids)['nll'][len(p) - 1:]
        runs.append((ids, lp))
        log(json.dumps(dict(cycle=c, first_ids=ids[:8], mean_nll=round(sum(lp) / len(lp), 6))))
    base_ids, base_lp = runs[0]
    differ = [c for c, (ids, _) in enumerate(runs) if ids != base_ids]
    spread = max(max(abs(a - b) for a, b in zip(lp, base_lp)) for _, lp in runs)
    return dict(test='token_flip', cycles=cycles, differing_cycles=differ, max_logprob_spread=spread,
                identical=not differ and spread == 0.0)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('mode', choices=('ppl', 'kl', 'flip'))
    ap.add_argument('files', nargs='*')
    ap.add_argument('--url', default='http://127.0.0.1:18180')
    ap.add_argument('--tag', default='run')
    ap.add_argument('--segments', type=int, default=6)
    ap.add_argument('--tokens', type=int, default=4096)
    ap.add_argument('--top', type=int, default=0)
    ap.add_argument('--tokenizer')
    ap.add_argument('--corpus', action='append', help='NAME=FILE (repeatable)')
    ap.add_argument('--cycles', type=int, default=12)
    ap.add_argument('--prompt-len', type=int, default=512)
    ap.add_argument('--out', default='.')
    a = ap.parse_args(argv)
    if a.mode == 'kl':
        if len(a.files) != 2:
            raise SystemExit('kl: give REF.top.json TEST.top.json')
        ref, test = (json.load(open(p)) for p in a.files)
        print(json.dumps(kl_compare(ref, test)))
        return 0
    cl = Client(a.url)
    if a.mode == 'flip':
        res = flip(cl, a.cycles, a.prompt_len, min(a.tokens, 256))
        print(json.dumps(res))
        return 0 if res['identical'] else 1
    corpora = dict(c.split('=', 1) for c in a.corpus) if a.corpus else None
    res, dump = ppl(cl, a.tag, a.segments, a.tokens, a.top, corpus.tokenizer(a.tokenizer), corpora)
    print('SUMMARY', json.dumps(res['summary']))
    os.makedirs(a.out, exist_ok=True)
    with open(os.path.join(a.out, f'{a.tag}.json'), 'w') as f:
        json.dump(res, f, indent=1)
    if dump is not None:
        with open(os.path.join(a.out, f'{a.tag}.top.json'), 'w') as f:
            json.dump(dump, f)
    return 0


if __name__ == '__main__':
    sys.exit(main())
