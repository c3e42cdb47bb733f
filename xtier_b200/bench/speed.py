"""Speed measurements against a running `xtier_b200.serve`: decode speed, prefill latency by prompt length, and
long-context prefill + decode.

    python -m xtier_b200.bench.speed decode  --url URL [--tokens 512] [--prompt-len 64] [--concurrency 1] [--rounds 2]
    python -m xtier_b200.bench.speed ttft    --url URL [--lengths 70,500,1000,2000,4096,8192] [--repeat 3]
    python -m xtier_b200.bench.speed context --url URL [--contexts 8192,65536] [--output 256] [--warmup 2048]
        [--repeats 3]
    python -m xtier_b200.bench.speed spec    --url URL [--tokens 256] [--prompts 8] [--rounds 2]   (--recall servers)
    common: [--tokenizer DIR --corpus FILE] (prompts cut from a text; default: seeded ids) [--out FILE]

decode: streamed requests with fixed prompts; per request decode tok/s from the first to the last streamed token, per
round the aggregate (tokens of all requests / wall time of the round). ttft: cold prefill (cache flushed) of prompts
of each length, one output token, median of --repeat. context: per context length a cold prefill (prefill tok/s =
prompt tokens / time to the first token) and an answer of --output tokens, then --repeats more answers to the same
prompt; decode tok/s is the median over the answers. A first request of --warmup tokens takes one-time costs.
Every line printed is JSON; the last one is the summary, also written to --out.
spec: per request of a speculative server, target forwards, ms per forward and tokens per forward.
(Reference parity: bench/decode_speed.py, bench/ttft_probe.py, bench/context_speed.py, bench/verify_step_bench.py --
the same measures against this framework's server.)
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import statistics
import sys
import time

from . import corpus
from .client import Client


def _info(cl: Client) -> dict:
    st, h = cl.request('GET', '/health')
    if st != 200 or not h.get('ready'):
        raise SystemExit(f'server not ready: {h}')
    return h


def decode_speed(cl: Client, tokens: int = 512, prompt_len: int = 64, concurrency: int = 1, rounds: int = 2,
                 tok=None, corpus_path=None, log=print) -> dict:
    info = _info(cl)
    out = []
    for r in range(rounds):
        prompts = [corpus.prompt(prompt_len, info['vocab'], tok, corpus_path, salt=r * 1000 + i)
                   for i in range(concurrency)]
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(concurrency) as ex:
            res = list(ex.map(lambda p: cl.stream(p, tokens), prompts))
        wall = time.perf_counter() - t0
        for i, x in enumerate(res):
            log(json.dumps(dict(round=r, request=i, tokens=len(x['ids']), ttft_s=round(x['ttft_s'], 4),
                                decode_tok_s=x['decode_tok_s'] and round(x['decode_tok_s'], 2))))
        agg = sum(len(x['ids']) for x in res) / wall
        out.append(dict(round=r, aggregate_tok_s=round(agg, 2),
                        median_decode_tok_s=round(statistics.median(x['decode_tok_s'] or 0 for x in res), 2)))
        log(json.dumps(out[-1]))
    return dict(test='decode_speed', tokens=tokens, concurrency=concurrency, rounds=out,
                decode_tok_s=max(r['median_decode_tok_s'] for r in out))


def ttft(cl: Client, lengths=(70, 500, 1000, 2000, 4096, 8192), repeat: int = 3, tok=None, corpus_path=None,
         log=print) -> dict:
    info = _info(cl)
    rows = []
    for n in lengths:
        if n + 16 > info['max_len']:
            log(json.dumps(dict(tokens=n, skipped='longer than the server max length')))
            continue
        times = []
        for r in range(repeat):
            cl.flush()
            x = cl.stream(corpus.prompt(n, info['vocab'], tok, corpus_path, salt=n * 100 + r), 1)
            times.append(x['ttft_s'])
        rows.append(dict(tokens=n, ttft_s=round(statistics.median(times), 4),
                         prefill_tok_s=round(n / statistics.median(times), 1)))
        log(json.dumps(rows[-1]))
    return dict(test='ttft', rows=rows)


def context_speed(cl: Client, contexts=(8192, 65536), output: int = 256, warmup: int = 2048, repeats: int = 3,
                  tok=None, corpus_path=None, log=print) -> dict:
    info = _info(cl)
    if warmup:
        cl.stream(corpus.prompt(min(warmup, info['max_len'] - 32), info['vocab'], tok, corpus_path, salt=7), 16)
    rows = []
    for n in contexts:
        if n + output + 8 > info['max_len']:
            log(json.dumps(dict(context=n, skipped='longer than the server max length')))
            continue
        p = corpus.prompt(n, info['vocab'], tok, corpus_path, salt=n)
        cl.flush()
        first = cl.stream(p, output)
        dec = [first['decode_tok_s']] + [cl.stream(p, output)['decode_tok_s'] for _ in range(repeats)]
        dec = [d for d in dec if d]
        rows.append(dict(context=n, ttft_s=round(first['ttft_s'], 3), prefill_tok_s=round(n / first['ttft_s'], 1),
                         decode_tok_s=round(statistics.median(dec), 2) if dec else None, answers=len(dec)))
        log(json.dumps(rows[-1]))
    return dict(test='context_speed', output=output, rows=rows)


def spec_steps(cl: Client, tokens: int = 256, prompts: int = 8, rounds: int = 2, prompt_len: int = 64, tok=None,
               corpus_path=None, log=print) -> dict:
    """Cost of one speculative step of a server started with --recall (or a draft model): per request the target
    forwards it took (the `spec_forwards` metric), ms per forward = decode time / forwards, tokens per forward. The
    same prompts run every round, so later rounds can copy from what earlier ones wrote."""
    info = _info(cl)
    rows = []
    for r in range(rounds):
        for i in range(prompts):
            f0 = cl.metrics().get('spec_forwards')
            if f0 is None:
                raise SystemExit('the server does not report spec_forwards: start it with --recall')
            x = cl.stream(corpus.prompt(prompt_len, info['vocab'], tok, corpus_path, salt=3000 + i), tokens)
            fw = cl.metrics()['spec_forwards'] - f0
            n = len(x['ids'])
            rows.append(dict(round=r, request=i, tokens=n, forwards=fw,
                             ms_per_step=round(1000.0 * x['decode_s'] / fw, 3) if fw else None,
                             tokens_per_step=round((n - 1) / fw, 3) if fw else None))
            log(json.dumps(rows[-1]))
    summary = []
    for r in range(rounds):
        sel = [x for x in rows if x['round'] == r and x['forwards']]
        fw = sum(x['forwards'] for x in sel)
        summary.append(dict(round=r, forwards=fw, tokens_per_step=round(sum(x['tokens'] - 1 for x in sel) / fw, 3)
                            if fw else None,
                            ms_per_step=round(statistics.median(x['ms_per_step'] for x in sel), 3) if sel else None))
    return dict(test='spec_steps', rounds=summary, rows=rows)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('mode', choices=('decode', 'ttft', 'context', 'spec'))
    ap.add_argument('--prompts', type=int, default=8)
    ap.add_argument('--url', default='http://127.0.0.1:18180')
    ap.add_argument('--tokenizer')
    ap.add_argument('--corpus')
    ap.add_argument('--tokens', type=int, default=512)
    ap.add_argument('--prompt-len', type=int, default=64)
    ap.add_argument('--concurrency', type=int, default=1)
    ap.add_argument('--rounds', type=int, default=2)
    ap.add_argument('--lengths', default='70,500,1000,2000,4096,8192')
    ap.add_argument('--repeat', type=int, default=3)
    ap.add_argument('--contexts', default='8192,65536')
    ap.add_argument('--output', type=int, default=256)
    ap.add_argument('--warmup', type=int, default=2048)
    ap.add_argument('--repeats', type=int, default=3)
    ap.add_argument('--out')
    a = ap.parse_args(argv)
    cl = Client(a.url)
    tok = corpus.tokenizer(a.tokenizer)
    if a.mode == 'decode':
        res = decode_speed(cl, a.tokens, a.prompt_len, a.concurrency, a.rounds, tok, a.corpus)
    elif a.mode == 'ttft':
        res = ttft(cl, [int(x) for x in a.lengths.split(',')], a.repeat, tok, a.corpus)
    elif a.mode == 'spec':
        res = spec_steps(cl, a.tokens, a.prompts, a.rounds, a.prompt_len, tok, a.corpus)
    else:
        res = context_speed(cl, [int(x) for x in a.contexts.split(',')], a.output, a.warmup, a.repeats, tok,
                            a.corpus)
    print(json.dumps(res))
    if a.out:
        with open(a.out, 'w') as f:
            json.dump(res, f, indent=1)
    return 0


if __name__ == '__main__':
    sys.exit(main())
