"""The generation server's HTTP behaviour and the bench tools, against a stand-in backend on the CPU: validation,
streaming, scoring, aborts, the queue limit; speed, perplexity / KL / token stability, abuse and interleave probes,
and the verbatim-copy test."""
import math
import random
import time

import numpy as np
import pytest

from xtier_b200 import serve
from xtier_b200.bench import copy_test, quality, robustness, speed
from xtier_b200.bench.client import Client, ServerError

V = 1000


class Fake:
    """A deterministic model: next token = (31 * last + 7) % vocab; position logits a fixed function of the token."""

    def __init__(self, vocab=V, max_len=4096, delay=0.0005, shift=0.0, tokenizer=None, corrupt=False):
        self.vocab, self.max_len, self.delay, self.shift = vocab, max_len, delay, shift
        self.tokenizer, self.corrupt = tokenizer, corrupt
        self.queue = None

    def prefill(self, ids):
        time.sleep(self.delay * (1 + len(ids) / 256))
        self.last = ids[-1]
        if self.tokenizer is not None:      # echo what sits between <src> and </src>
            text = self.tokenizer.decode(ids)
            a, b = text.index('<src>\n') + 6, text.index('\n</src>')
            body = text[a:b]
            if self.corrupt:
                body = body.replace('e', 'E', 1)
            self.queue = self.tokenizer.encode(body) + [self.tokenizer.eos_token_id]
            return self.queue.pop(0)
        return self.decode(sleep=False)

    def decode(self, sleep=True):
        if sleep:
            time.sleep(self.delay)
        if self.queue is not None:
            return self.queue.pop(0) if self.queue else self.tokenizer.eos_token_id
        self.last = (31 * self.last + 7) % self.vocab
        return self.last

    def _lp(self, t):
        x = np.sin(np.arange(self.vocab) * (t + 1) * 0.01) * 3.0 + self.shift * np.cos(np.arange(self.vocab) * 0.37)
        x = x - x.max()
        return x - np.log(np.exp(x).sum())

    def logprobs(self, ids, top):
        nll, tops = [], []
        for i in range(len(ids) - 1):
            lp = self._lp(ids[i])
            nll.append(float(-lp[ids[i + 1]]))
            if top:
                idx = np.argsort(-lp)[:top]
                tops.append([(int(j), float(lp[j])) for j in idx])
        return nll, tops

    def check(self):
        pass


class CharTok:
    eos_token_id = 3

    def encode(self, s, add_special_tokens=False):
        return [ord(c) for c in s]

    def decode(self, ids, skip_special_tokens=False):
        return ''.join(chr(t) for t in ids if t != self.eos_token_id)

    def apply_chat_template(self, msgs, add_generation_prompt=True, tokenize=True, **kw):
        return [1] + self.encode('user: ' + msgs[0]['content'] + '\nassistant: ')


@pytest.fixture
def server():
    made = []

    def make(backend, max_queue=8):
        s = serve.Server(backend, max_queue)
        srv = serve.serve(s, '127.0.0.1', 0)
        made.append(srv)
        return s, Client(f'http://127.0.0.1:{srv.server_address[1]}', timeout=60)
    yield make
    for srv in made:
        srv.shutdown()
        srv.server_close()


def test_endpoints_validation_and_streaming(server):
    s, cl = server(Fake())
    st, h = cl.request('GET', '/health')
    assert st == 200 and h['ready'] and h['vocab'] == V and h['max_len'] == 4096
    full = cl.generate([5, 6, 7], 10)
    assert len(full['ids']) == 10 and full['prompt_tokens'] == 3 and full['decode_tok_s'] > 0
    x = cl.stream([5, 6, 7], 10)
    assert x['ids'] == full['ids'] and x['server']['done'] and x['ttft_s'] > 0
    stop = full['ids'][3]
    assert cl.generate([5, 6, 7], 10, stop_ids=[stop])['ids'] == full['ids'][:4]
    r = cl.logprobs(list(range(20)), top=3)
    assert len(r['nll']) == 19 and len(r['top']) == 19 and len(r['top'][0]) == 3
    assert cl.flush() == {'ok': True}
    for body, code in [({'prompt_ids': [1] * 4090, 'max_new_tokens': 8}, 400), ({'prompt_ids': [V]}, 400),
                       ({'prompt_ids': [1], 'max_new_tokens': True}, 400), ({'prompt': 'text'}, 400),
                       ({'prompt_ids': 'abc'}, 400)]:
        assert cl.request('POST', '/v1/generate', body)[0] == code, body
    assert cl.request('GET', '/nowhere')[0] == 404
    m = cl.metrics()
    assert m['requests'] == 4 and m['tokens'] == 24
    _, cl0 = server(Fake(), max_queue=0)
    with pytest.raises(ServerError) as e:
        cl0.generate([1, 2], 2)
    assert e.value.status == 503


def test_speed_tools(server):
    _, cl = server(Fake())
    quiet = dict(log=lambda s: None)
    d = speed.decode_speed(cl, tokens=16, prompt_len=8, concurrency=2, rounds=1, **quiet)
    assert d['rounds'][0]['aggregate_tok_s'] > 0 and d['decode_tok_s'] > 0
    t = speed.ttft(cl, lengths=[16, 64, 5000], repeat=2, **quiet)
    assert [r['tokens'] for r in t['rows']] == [16, 64] and all(r['ttft_s'] > 0 for r in t['rows'])
    c = speed.context_speed(cl, contexts=[256], output=8, warmup=32, repeats=1, **quiet)
    assert c['rows'][0]['prefill_tok_s'] > 0 and c['rows'][0]['answers'] == 2


def test_ppl_kl_and_flip(server):
    _, ref = server(Fake())
    _, test = server(Fake(shift=0.3))
    quiet = dict(log=lambda s: None)
    r1, d1 = quality.ppl(ref, 'ref', segments=3, tokens=64, top=8, **quiet)
    r2, d2 = quality.ppl(test, 'test', segments=3, tokens=64, top=8, **quiet)
    assert r1['summary']['all']['segments'] == 3 and r1['summary']['all']['ppl'] > 1
    assert [r['seg'] for r in r1['rows']] == [r['seg'] for r in r2['rows']]    # the same segments
    same = quality.kl_compare(d1, d1)
    assert same['kl_mean'] == 0 and same['top1_changed'] == 0 and same['nll_diff'] == 0
    diff = quality.kl_compare(d1, d2)
    assert diff['kl_mean'] > 0 and diff['positions'] == 3 * 63
    assert abs(diff['nll_diff'] - (r2['summary']['all']['nll'] - r1['summary']['all']['nll'])) < 1e-3
    f = quality.flip(ref, cycles=3, prompt_len=32, tokens=8, **quiet)
    assert f['identical']


def test_kl_lower_bound_never_exceeds_the_full_kl():
    rng = random.Random(0)
    for _ in range(200):
        n = 30
        p = [rng.random() ** 3 for _ in range(n)]
        q = [rng.random() ** 3 for _ in range(n)]
        sp, sq = sum(p), sum(q)
        p, q = [x / sp for x in p], [x / sq for x in q]
        full = sum(a * math.log(a / b) for a, b in zip(p, q))
        top = 5
        pt = sorted(range(n), key=lambda i: -p[i])[:top]
        qt = sorted(range(n), key=lambda i: -q[i])[:top]
        lb = quality.kl_lower_bound([[i, math.log(p[i])] for i in pt], [[i, math.log(q[i])] for i in qt])
        assert lb <= full + 1e-9


def test_abuse_and_interleave(server):
    _, cl = server(Fake(delay=0.001))
    res = robustness.abuse(cl, quick=True, log=lambda s: None)
    assert res['failed'] == 0, res['failures']
    it = robustness.interleave(cl, tokens=128, delay=0.05, answer=80, log=lambda s: None)
    assert it['b_waited_for_a'] and it['a_tokens'] == 80


def test_copy_test(server):
    src = '\n'.join(f'def f{i}(x):\n    return x + {i}' for i in range(40))
    tok = CharTok()
    _, good = server(Fake(vocab=70000, tokenizer=tok))
    res = copy_test.run(good, tok, src, chunks=3, lines=20, log=lambda s: None)
    assert res['windows'] == 3 and res['differ'] == 0
    _, bad = server(Fake(vocab=70000, tokenizer=tok, corrupt=True))
    res = copy_test.run(bad, tok, src, chunks=3, lines=20, log=lambda s: None)
    assert res['differ'] == 3


def test_speculative_serving_with_recall(server):
    """A --recall server: one target forward per step, several tokens when a copy lands; the tokens equal the
    target's greedy ones; repeated prompts copy from the record."""
    import torch
    from xtier_b200 import recall

    class Bigram:
        def __init__(self, V=64):
            self.W = torch.randn(V, V, generator=torch.Generator().manual_seed(0)) * 4
            self.vocab, self.device = V, torch.device('cpu')

        def alloc_state(self, b, n):
            return {}

        def prefill(self, st, tokens, start=0, return_logits=False, all_logits=False, active=None):
            lg = self.W[tokens.long()]
            nxt = torch.argmax(lg, -1)
            if all_logits:
                return nxt, lg
            return (nxt[-1:], lg[-1]) if return_logits else nxt[-1:]

    tgt = Bigram()
    be = serve.SpecBackend(tgt, recall.RecallEngine(recall.Record(), gamma=8, min_n=1.0), max_len=512)
    _, cl = server(be)
    prompt = [3, 9, 27, 17, 40]
    want, t = [], prompt[-1]
    for _ in range(40):
        t = int(torch.argmax(tgt.W[t]))
        want.append(t)
    assert cl.generate(prompt, 40)['ids'] == want
    x = cl.stream(prompt, 40)
    assert x['ids'] == want
    res = speed.spec_steps(cl, tokens=32, prompts=2, rounds=2, prompt_len=24, log=lambda s: None)
    assert res['rounds'][1]['tokens_per_step'] > 1.0
    m = cl.metrics()
    assert m['spec_copy_landed'] > 0 and m['recall_record_ids'] > 0
    r = cl.logprobs(prompt + want[:5], top=2)
    assert len(r['nll']) == 9


class Canned:
    """A backend that answers every prompt with the same text, then its end-of-turn id."""

    def __init__(self, reply, tok):
        self.tokenizer, self.vocab, self.max_len = tok, 70000, 4096
        self.reply = tok.encode(reply) + [tok.eos_token_id]

    def prefill(self, ids):
        self.i = 0
        return self.decode()

    def decode(self):
        t = self.reply[min(self.i, len(self.reply) - 1)]
        self.i += 1
        return t

    def check(self):
        pass


def _sse(cl, body):
    import http.client
    import json
    c = http.client.HTTPConnection(cl.host, cl.port, timeout=30)
    c.request('POST', '/v1/chat/completions', json.dumps(body).encode(), {'Content-Type': 'application/json'})
    r = c.getresponse()
    assert r.status == 200 and r.getheader('Content-Type') == 'text/event-stream'
    events = [line[6:] for line in r.read().decode().split('\n') if line.startswith('data: ')]
    c.close()
    return events


def test_chat_completions(server):
    import json
    tok = CharTok()
    reply = 'Hello <tool_call>\n{"name": "read_file", "arguments": {"path": "a.py"}}\n</tool_call>'
    _, cl = server(Canned(reply, tok))
    msgs = [{'role': 'user', 'content': 'read a.py'}]
    tools = [{'type': 'function', 'function': {'name': 'read_file', 'parameters': {}}}]
    st, r = cl.request('POST', '/v1/chat/completions', {'messages': msgs, 'tools': tools})
    assert st == 200 and r['object'] == 'chat.completion'
    ch = r['choices'][0]
    assert ch['message']['content'] == 'Hello' and ch['finish_reason'] == 'tool_calls'
    call = ch['message']['tool_calls'][0]['function']
    assert call['name'] == 'read_file' and json.loads(call['arguments']) == {'path': 'a.py'}
    assert r['usage']['completion_tokens'] == len(reply) and r['usage']['prompt_tokens'] > 0
    st, r = cl.request('POST', '/v1/chat/completions', {'messages': msgs})          # no tools: plain text
    assert r['choices'][0]['message']['content'] == reply and r['choices'][0]['finish_reason'] == 'stop'
    st, r = cl.request('POST', '/v1/chat/completions', {'messages': msgs, 'max_tokens': 3})
    assert r['choices'][0]['message']['content'] == 'Hel' and r['choices'][0]['finish_reason'] == 'length'
    ev = _sse(cl, {'messages': msgs, 'stream': True, 'stream_options': {'include_usage': True}})
    assert ev[-1] == '[DONE]'
    chunks = [json.loads(e) for e in ev[:-1]]
    text = ''.join(c['choices'][0]['delta'].get('content', '') for c in chunks if c['choices'])
    assert text == reply
    assert chunks[-2]['choices'][0]['finish_reason'] == 'stop' and chunks[-1]['usage']['completion_tokens'] == len(reply)
    for body in ({'messages': msgs, 'temperature': 0.7}, {'messages': []}, {'messages': msgs, 'max_tokens': 0}):
        st, r = cl.request('POST', '/v1/chat/completions', body)
        assert st == 400 and 'message' in r['error'], body
    assert cl.request('GET', '/v1/models')[1]['data'][0]['id'] == 'xtier-b200'
    _, plain = server(Fake())
    assert plain.request('POST', '/v1/chat/completions', {'messages': msgs})[0] == 400     # no tokenizer


class JsonChatTok(CharTok):
    """Chat template: the messages as ASCII JSON, one id per character."""

    def apply_chat_template(self, msgs, add_generation_prompt=True, tokenize=True, **kw):
        import json
        return self.encode(json.dumps(msgs))


class Scripted:
    """Answers the n-th request with the n-th scripted reply."""

    def __init__(self, replies, tok):
        self.tokenizer, self.vocab, self.max_len = tok, 70000, 1 << 20
        self.replies = [tok.encode(r) + [tok.eos_token_id] for r in replies]
        self.n = -1

    def prefill(self, ids):
        self.n += 1
        self.cur = self.replies[min(self.n, len(self.replies) - 1)]
        self.i = 0
        return self.decode()

    def decode(self):
        t = self.cur[min(self.i, len(self.cur) - 1)]
        self.i += 1
        return t

    def check(self):
        pass


def test_agent_bench_session(server):
    import json
    from pathlib import Path
    from xtier_b200.bench import agent
    src = Path(agent.__file__).resolve().parents[1]
    before = (src / 'bench' / 'corpus.py').read_text()

    def call(name, **args):
        return '<tool_call>\n' + json.dumps({'name': name, 'arguments': args}) + '\n</tool_call>'
    replies = ['Reading. ' + call('read_file', path='bench/corpus.py', start_line=1, end_line=5),
               call('edit_file', path='bench/corpus.py', old_string='def tokenizer(path: str | None):',
                    new_string='def tokenizer(path: str | None):  # edited'),
               call('check_python', path='bench/corpus.py') + call('grep', pattern='edited', path='bench'),
               'Done: the function is edited and the file checks.']
    _, cl = server(Scripted(replies, JsonChatTok()))
    res = agent.run_session(cl, 'tiny', (500, 'Edit the corpus module.', ['bench/corpus.py']), src, steps=6,
                            count=len, run_id='t1', context_limit=1 << 24, log=lambda s: None)
    rows = res['requests']
    assert [r['tools'] for r in rows] == [['read_file'], ['edit_file'], ['check_python', 'grep'], []]
    assert rows[0]['prefill_tps'] > 0 and all(r['output_tokens'] > 0 for r in rows)
    assert (src / 'bench' / 'corpus.py').read_text() == before          # the edit stayed in the sandbox
    t = agent.table([{'sessions': [res]}])
    assert t['all']['requests'] == 4 and t['sessions']['tiny']['cold_prefill_tps'] > 0
    sb = agent.Sandbox(src)
    try:
        assert 'outside' in sb.call('read_file', {'path': '../../etc/passwd'})
        assert sb.call('edit_file', {'path': 'bench/corpus.py', 'old_string': 'import', 'new_string': 'x'}).startswith(
            'error: old_string occurs')
        assert sb.call('write_file', {'path': 'new/x.py', 'content': 'def f(:\n'}).startswith('ok')
        assert sb.call('check_python', {'path': 'new/x.py'}).startswith('syntax error')
        assert sb.call('nope', {}) == 'error: no tool nope'
    finally:
        sb.close()
    assert not sb.root.exists()


def test_sampling_parameters(server):
    class Sampler(Fake):
        sampling = True

        def set_sampling(self, t, p):
            self.seen = (t, p)

    be = Sampler()
    _, cl = server(be)
    cl.request('POST', '/v1/generate', {'prompt_ids': [1, 2], 'max_new_tokens': 2, 'temperature': 0.7, 'top_p': 0.9})
    assert be.seen == (0.7, 0.9)
    cl.generate([1, 2], 2)
    assert be.seen == (0.0, 1.0)
    for bad in ({'temperature': -1}, {'top_p': 0}, {'top_p': 1.5}, {'temperature': 'hot'}):
        assert cl.request('POST', '/v1/generate', {'prompt_ids': [1], **bad})[0] == 400, bad
    _, greedy = server(Fake())
    st, r = greedy.request('POST', '/v1/generate', {'prompt_ids': [1], 'temperature': 0.5})
    assert st == 400 and 'greedily' in r['error']


def test_prefix_reuse_across_requests(server):
    """A prompt that starts with the previous request's prompt and reply prefills only the rest; a flush or a
    different prompt starts from the first token."""
    import torch

    class FakeGen:
        sampling, use_graph, max_len = False, False, 4096

        def __init__(self):
            self.graph, self.starts, self.state = 'captured', [], {}
            self.buf = {'tokens': torch.zeros(1, dtype=torch.int64)}
            self.host_tokens = torch.zeros(1, dtype=torch.int64)

        def prefill(self, prompts, start=0):
            self.starts.append(start)
            self.buf['tokens'].fill_(int(prompts[0, -1]) + 1)

        def decode_one(self):
            self.host_tokens += 1
            return self.host_tokens

        def between_steps(self):
            pass

        def check(self):
            pass

    class FakeModel:
        class cfg:
            vocab = 1000
        bigram = None

    gen = FakeGen()
    _, cl = server(serve.GenBackend(FakeModel(), gen))
    p = [5, 6, 7, 8]
    out = cl.generate(p, 4)['ids']
    assert out == [9, 10, 11, 12] and gen.starts == [0]
    cl.generate(p + out + [40, 41], 2)            # the cache holds p and the reply's first three tokens
    assert gen.starts[-1] == len(p) + len(out) - 1
    cl.generate(p, 2)                             # a prefix of the cache: all but the last id reused
    assert gen.starts[-1] == len(p) - 1
    cl.generate([1, 2, 3], 2)
    assert gen.starts[-1] == 0
    cl.flush()
    cl.generate([1, 2, 3], 2)
    assert gen.starts[-1] == 0
    assert cl.metrics()['prefix_reused_tokens'] == (len(p) + len(out) - 1) + (len(p) - 1)
    be = serve.GenBackend(FakeModel(), FakeGen(), prefix_cache=False)
    be.cached = [1, 2, 3]
    assert be.reusable([1, 2, 3, 4]) == 0


def test_continuous_batching(server):
    """Concurrent requests share decode steps (at most `rows` at once); each gets exactly its own sequence; an
    aborted stream frees its row."""
    import threading
    import time as _t

    class FakeBatch:
        vocab, max_len, rows, tokenizer, sampling = 1000, 4096, 3, None, False

        def __init__(self):
            self.last, self.steps, self.max_active = {}, 0, 0

        def prefill_row(self, row, ids):
            self.last[row] = sum(ids) % 1000
            return self.last[row]

        def step(self, active):
            _t.sleep(0.003)
            self.steps += 1
            self.max_active = max(self.max_active, len(active))
            out = [0] * self.rows
            for r in active:
                self.last[r] = (31 * self.last[r] + 7) % 1000
                out[r] = self.last[r]
            return out

        def check(self):
            pass

    def expect(ids, n):
        t = sum(ids) % 1000
        seq = [t]
        while len(seq) < n:
            t = (31 * t + 7) % 1000
            seq.append(t)
        return seq

    be = FakeBatch()
    srv = serve.BatchServer(be, max_queue=16)
    hs = serve.serve(srv, '127.0.0.1', 0)
    try:
        cl = Client(f'http://127.0.0.1:{hs.server_address[1]}', timeout=60)
        prompts = [[i + 1, 2 * i + 5, 7] for i in range(6)]
        res = [None] * 6

        def one(i):
            res[i] = cl.generate(prompts[i], 20 + i)['ids']
        th = [threading.Thread(target=one, args=(i,)) for i in range(6)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        for i in range(6):
            assert res[i] == expect(prompts[i], 20 + i), i
        assert 1 < be.max_active <= 3
        assert be.steps < sum(20 + i for i in range(6)) - 6          # steps were shared
        x = cl.stream([9, 9, 9], 200, abort_after=2)
        assert x['aborted']
        assert cl.generate([1, 2, 3], 5)['ids'] == expect([1, 2, 3], 5)
        t_end = _t.time() + 10
        while cl.metrics()['aborted'] < 1 and _t.time() < t_end:
            _t.sleep(0.05)
        assert cl.metrics()['aborted'] == 1
    finally:
        hs.shutdown()
        hs.server_close()
