"""What clients do to a running `xtier_b200.serve` that it must survive, and what a long prompt does to a request
decoding beside it.

    python -m xtier_b200.bench.robustness abuse      --url URL [--quick] [--out FILE]
    python -m xtier_b200.bench.robustness interleave --url URL [--tokens 16384] [--delay 2.0] [--out FILE]

abuse: (1) streamed requests whose client goes away after a few tokens: the server must notice, stop the decode and
count it; (2) requests it must refuse with 400 / 404 / 413 (too long, bad parameters, ids outside the vocabulary, an
empty prompt, broken JSON, an unknown path, a body declared larger than the limit); (3) three requests at once, all
answered in full. After every group a small request must still be answered. One JSON line per case; exit status 1
when any case failed.
interleave: request A streams a long answer; --delay seconds in, request B sends a cold prompt of --tokens ids.
Reported: B's time to its first token, A's longest wait between two tokens while B is read, A's token rate before,
during and after. A server started with --batch 1 runs one request at a time, so B waits for A (and A is never paused
by B); with --batch N > 1, B's prefill runs between two of A's decode steps, and A's longest wait is its cost.
(Reference parity: bench/abuse_test.py and bench/interleave_probe.py.)
"""
from __future__ import annotations

import argparse
import http.client
import json
import sys
import threading
import time

from . import corpus
from .client import Client, ServerError


def _small(cl: Client, vocab: int) -> bool:
    try:
        return len(cl.generate(corpus.prompt(8, vocab, salt=99), 4)['ids']) == 4
    except (ServerError, OSError):
        return False


def _raw(cl: Client, method: str, path: str, body: bytes, headers: dict) -> int:
    c = http.client.HTTPConnection(cl.host, cl.port, timeout=60)
    try:
        c.putrequest(method, path)
        for k, v in headers.items():
            c.putheader(k, v)
        c.endheaders()
        if body:
            c.send(body)
        r = c.getresponse()
        r.read()
        return r.status
    finally:
        c.close()


def abuse(cl: Client, quick: bool = False, log=print) -> dict:
    st, info = cl.request('GET', '/health')
    if st != 200 or not info.get('ready'):
        raise SystemExit(f'server not ready: {info}')
    V, L = info['vocab'], info['max_len']
    cases = []

    def case(group, name, ok, **kw):
        cases.append(dict(group=group, case=name, ok=bool(ok), **kw))
        log(json.dumps(cases[-1]))

    # 1. aborted streams
    before = cl.metrics().get('aborted', 0)
    for k in ([1, 4] if quick else [1, 2, 4, 8, 16]):
        x = cl.stream(corpus.prompt(32, V, salt=k), max_new_tokens=min(256, L - 64), abort_after=k)
        case('abort', f'after {k} tokens', x['aborted'] and len(x['ids']) == k)
    t0 = time.monotonic()
    ok = _small(cl, V)
    case('abort', 'small request after the aborts', ok, wait_s=round(time.monotonic() - t0, 3))
    want = 2 if quick else 5
    t_end = time.monotonic() + 30.0
    counted = cl.metrics().get('aborted', 0) - before
    while counted < want and time.monotonic() < t_end:   # the last abort may still be finishing its token
        time.sleep(0.05)
        counted = cl.metrics().get('aborted', 0) - before
    case('abort', 'aborts counted', counted == want, counted=counted)

    # 2. requests to refuse
    refuse = [
        ('too long', {'prompt_ids': [1] * (L - 4), 'max_new_tokens': 64}, 400),
        ('max_new_tokens 0', {'prompt_ids': [1, 2], 'max_new_tokens': 0}, 400),
        ('max_new_tokens text', {'prompt_ids': [1, 2], 'max_new_tokens': 'ten'}, 400),
        ('id outside the vocabulary', {'prompt_ids': [1, V + 5]}, 400),
        ('negative id', {'prompt_ids': [-3]}, 400),
        ('empty prompt', {'prompt_ids': []}, 400),
        ('no prompt', {'max_new_tokens': 4}, 400),
        ('not an object', [1, 2, 3], 400),
    ]
    for name, body, want in refuse:
        got, _ = cl.request('POST', '/v1/generate', body)
        case('refuse', name, got == want, status=got)
    got, _ = cl.request('POST', '/v1/generate', raw=b'{"prompt_ids": [1, 2')
    case('refuse', 'broken JSON', got == 400, status=got)
    got, _ = cl.request('POST', '/v1/nothing', {})
    case('refuse', 'unknown path', got == 404, status=got)
    got = _raw(cl, 'POST', '/v1/generate', b'{}', {'Content-Type': 'application/json',
                                                   'Content-Length': str(1 << 30)})
    case('refuse', 'declared body over the limit', got == 413, status=got)
    got, _ = cl.request('POST', '/v1/logprobs', {'prompt_ids': [1]})
    case('refuse', 'scoring one token', got == 400, status=got)
    case('refuse', 'small request after the refusals', _small(cl, V))

    # 3. three at once
    res = [None] * 3

    def one(i):
        try:
            res[i] = cl.generate(corpus.prompt(24, V, salt=500 + i), 12)
        except (ServerError, OSError) as e:
            res[i] = e
    th = [threading.Thread(target=one, args=(i,)) for i in range(3)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    case('concurrent', 'three requests answered in full',
         all(isinstance(r, dict) and len(r['ids']) == 12 for r in res))
    case('concurrent', 'small request after', _small(cl, V))
    failed = [c for c in cases if not c['ok']]
    return dict(test='abuse', cases=len(cases), failed=len(failed), failures=failed)


def interleave(cl: Client, tokens: int = 16384, delay: float = 2.0, answer: int = 4096, log=print) -> dict:
    st, info = cl.request('GET', '/health')
    V, L = info['vocab'], info['max_len']
    tokens = min(tokens, L - 16)
    answer = min(answer, L - 80)
    a_times: list[float] = []
    b_box: dict = {}

    def run_a():
        b_box['a'] = cl.stream(corpus.prompt(64, V, salt=1), answer, on_token=lambda m: a_times.append(
            time.perf_counter()))

    ta = threading.Thread(target=run_a)
    ta.start()
    while not a_times and ta.is_alive():
        time.sleep(0.01)
    time.sleep(delay)
    b_sent = time.perf_counter()
    b = cl.stream(corpus.prompt(tokens, V, salt=2), 8)
    b_first = b_sent + (b['ttft_s'] or 0.0)
    ta.join()

    def rate(t0, t1):
        n = sum(1 for t in a_times if t0 <= t < t1)
        return n / (t1 - t0) if t1 > t0 else None
    during = [t for t in a_times if b_sent <= t <= b_first]
    gaps = [y - x for x, y in zip(a_times, a_times[1:]) if x >= b_sent - 1e-9 and y <= b_first + 1e-9]
    res = dict(test='interleave', prompt_tokens=tokens, b_ttft_s=b['ttft_s'],
               a_tok_s_before=rate(max(a_times[0], b_sent - 10.0), b_sent) if a_times else None,
               a_tok_s_during=len(during) / (b_first - b_sent) if b_first > b_sent else None,
               a_tok_s_after=rate(b_first, a_times[-1]) if a_times and a_times[-1] > b_first else None,
               a_longest_wait_s=max(gaps) if gaps else 0.0, a_tokens=len(a_times),
               b_waited_for_a=bool(a_times) and b_first >= a_times[-1])
    log(json.dumps(res))
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('mode', choices=('abuse', 'interleave'))
    ap.add_argument('--url', default='http://127.0.0.1:18180')
    ap.add_argument('--quick', action='store_true')
    ap.add_argument('--tokens', type=int, default=16384)
    ap.add_argument('--delay', type=float, default=2.0)
    ap.add_argument('--answer', type=int, default=4096)
    ap.add_argument('--out')
    a = ap.parse_args(argv)
    cl = Client(a.url)
    res = abuse(cl, a.quick) if a.mode == 'abuse' else interleave(cl, a.tokens, a.delay, a.answer)
    print(json.dumps(res))
    if a.out:
        with open(a.out, 'w') as f:
            json.dump(res, f, indent=1)
    return 1 if res.get('failed') else 0


if __name__ == '__main__':
    sys.exit(main())
