"""Generation server over the framework's public API (the process the console launches, and what xtier_b200.bench
measures).

    python -m xtier_b200.serve --model qwen3-moe [--layers 48] [--hot 0.4] [--max-len 8192] --port 18180
    python -m xtier_b200.serve --checkpoint DIR [--hot 0.4] ...       # a Hugging Face qwen3_moe checkpoint
    python -m xtier_b200.serve --model deepseek-v3 [--layers 61] [--hot 0.44] ...   # DeepSeek-V3 shape, random init
    ... [--recall DIR|memory]        # speculative serving: Recall copy drafts verified by the target (one forward
                                     # per step, several tokens when a copy lands)

Endpoints
  GET  /health               {"ready": true, "vocab": V, "max_len": L, "tokenizer": bool} once the model is built and its
                             decode step captured
  GET  /metrics              decode counters, mailbox statistics, per-layer hit rates (JSON);
                             /metrics/prometheus: the same in the Prometheus text format
  POST /flush_cache          {"ok": true}; forgets the cached prefix (the next prompt is a cold prefill). A request whose
                             prompt starts with ids of the previous request (its prompt and reply) prefills only the
                             rest (--no-prefix-cache: never)
  POST /v1/generate          {"prompt_ids": [...] | "prompt": "text" (with a tokenizer), "max_new_tokens": n,
                              "stream": false, "stop_ids": [...], "temperature": 0, "top_p": 1 (a server started
                              with --sampling draws tokens; otherwise a temperature is refused)}
                             -> {"ids": [...], "text": ..., "prompt_tokens": T, "ttft_s": ..., "decode_tok_s": ...};
                             with "stream": true, newline-delimited JSON in a chunked response: {"id": t, "text": s}
                             per token, then {"done": true, ...the summary above}. A client that goes away ends the
                             decode at the next token.
  POST /v1/chat/completions  OpenAI chat format (with a tokenizer that has a chat template): messages, max_tokens,
                             stream (server-sent events, stream_options.include_usage), tools (Qwen-style
                             <tool_call> blocks in the reply come back as tool_calls), chat_template_kwargs; GET
                             /v1/models lists the one model
  POST /v1/logprobs          {"prompt_ids": [...], "top": N} -> {"nll": [-log p(ids[i+1] | ids[:i+1])],
                             "top": [[[id, logprob], ...] per position]} (fixed-text perplexity, A/B of configurations)

Requests run one at a time on the model (batch 1 decode, the CUDA graph of the tiered MoE model), or with --batch N
share the decode steps of N rows (continuous batching: a new request is prefilled into a free row between two steps);
at most --max-queue wait, the next ones get 503. Bad requests get 400 with the reason, unknown paths 404, bodies over 64 MiB 413.
(Reference parity: the reference serves through SGLang's HTTP server; the endpoints its bench tools use -- streamed
generation, /flush_cache, prompt logprobs, /metrics -- have these counterparts.)
"""
from __future__ import annotations

import argparse
import json
import re
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

MODELS = ('qwen3-moe', 'deepseek-v3')
MAX_BODY = 64 << 20


class BadRequest(ValueError):
    pass


STAGES = ('boot', 'weights', 'pool', 'graphs', 'ready')


class Stages:
    """Startup stages of the server with their times, printed as one log line each (the console reads the last one
    for its progress bar) and reported by /health and /metrics: boot, weights (layer i of n), pool (expert pools,
    CPU engines, mailbox), graphs (decode step capture), ready; `fail(reason)` records why a start died."""

    def __init__(self, emit=print):
        self.t0 = time.time()
        self.emit = emit
        self.phase, self.done, self.total, self.error = 'boot', 0, 0, None
        self.times = {'boot': 0.0}

    def set(self, phase: str, done: int = 0, total: int = 0):
        if phase not in STAGES:
            raise ValueError(f'unknown stage {phase!r}')
        first = phase != self.phase
        self.phase, self.done, self.total = phase, done, total
        if first:
            self.times[phase] = round(time.time() - self.t0, 3)
        if first or total:
            self.emit(f'[xtier_b200] stage {phase} {done}/{total} {time.time() - self.t0:.1f}s', flush=True)

    def fail(self, reason: str):
        self.error = str(reason)[:300]
        self.emit(f'[xtier_b200] FATAL: {self.error}', flush=True)

    def info(self) -> dict:
        return {'phase': self.phase, 'done': self.done, 'total': self.total, 'times': dict(self.times),
                'error': self.error}


class GenBackend:
    """The model and its decode runner behind the server: prefill a prompt, decode one token, score a text."""

    def __init__(self, model, gen, tokenizer=None, mailbox=None, prefix_cache: bool = True):
        self.model, self.gen, self.tokenizer, self.mailbox = model, gen, tokenizer, mailbox
        self.vocab = model.cfg.vocab
        self.max_len = gen.max_len
        self.sampling = gen.sampling
        # hashed n-gram rows read the previous token of a prefill's first one, which a reused prefix does not keep
        self.prefix_cache = prefix_cache and getattr(model, 'bigram', None) is None
        self.cached: list[int] = []      # ids whose KV sits in the cache at positions 0.. (the last request's)
        self.reused = 0                  # prompt tokens not computed again, over all requests

    def set_sampling(self, temperature: float, top_p: float):
        if self.sampling:                # a greedy generator has nothing to set (temperatures were refused)
            self.gen.set_sampling(temperature, top_p)

    def reusable(self, ids: list[int]) -> int:
        """How many leading ids of a prompt the cache already holds (at least one id is always computed)."""
        if not self.prefix_cache:
            return 0
        n = 0
        for a, b in zip(self.cached, ids):
            if a != b:
                break
            n += 1
        return min(n, len(ids) - 1)

    def prefill(self, ids: list[int]) -> int:
        import torch
        gen = self.gen
        start = self.reusable(ids)
        self.cached = []                 # invalid until this prefill is done
        gen.prefill(torch.tensor([ids]), start=start)
        if gen.graph is None and gen.use_graph:
            gen.capture()
        gen.host_tokens.copy_(gen.buf['tokens'].cpu())
        self.reused += start
        self.cached = list(ids)
        self.last = int(gen.host_tokens[0])
        return self.last

    def decode(self) -> int:
        t = int(self.gen.decode_one()[0])
        self.cached.append(self.last)    # the step wrote the KV of the token it was fed
        self.last = t
        self.gen.between_steps()
        return t

    def flush(self):
        self.cached = []

    def logprobs(self, ids: list[int], top: int):
        self.cached = []
        out = score(self.model, self.gen.state, ids, top)
        self.cached = list(ids)          # the scoring forward left the KV of exactly these ids
        return out

    def check(self):
        self.gen.check()

    def snapshot(self, state) -> dict:
        from .utils.metrics import snapshot
        snap = snapshot(self.model, self.mailbox, state)
        snap['prefix_reused_tokens'] = self.reused
        return snap


def score(model, state, ids: list[int], top: int):
    """(-log p(ids[i+1] | ids[:i+1]) per position, the `top` most likely (id, logprob) per position) from one
    forward of `model` over `ids` with every position's logits."""
    import torch
    dev = model.device
    _, logits = model.prefill(state, torch.tensor(ids, device=dev), all_logits=True)
    nll, tops = [], []
    tgt = torch.tensor(ids[1:], device=dev)
    for s in range(0, len(ids) - 1, 512):
        lp = torch.log_softmax(logits[s:min(s + 512, len(ids) - 1)].float(), dim=-1)
        nll += (-lp.gather(1, tgt[s:s + lp.shape[0], None])[:, 0]).tolist()
        if top > 0:
            v, i = lp.topk(top, dim=-1)
            tops += [list(zip(a, b)) for a, b in zip(i.tolist(), v.tolist())]
    return nll, tops


class SpecBackend:
    """Speculative serving: each step is one target forward that verifies copy drafts from a Recall engine (and / or
    a draft model's chain); a step yields one or more tokens. The stream's text goes to the recall record when the
    request ends."""

    def __init__(self, model, recall=None, draft=None, max_len: int = 8192, tokenizer=None, temperature: float = 0.0,
                 mailbox=None):
        from .runtime.speculative import SpeculativeDecoder
        self.model, self.recall, self.tokenizer, self.mailbox = model, recall, tokenizer, mailbox
        cfg = getattr(model, 'cfg', None)
        self.vocab = cfg.vocab if cfg is not None else int(model.vocab)
        self.max_len = max_len
        self.dec = SpeculativeDecoder(model, draft, recall=recall, max_len=max_len, temperature=temperature)
        self.active = False
        self.sampling = True             # verification is lossless at any temperature / top-p

    def set_sampling(self, temperature: float, top_p: float):
        self.dec.temp, self.dec.top_p = float(temperature), float(top_p)

    def prefill(self, ids: list[int]) -> int:
        import torch
        if self.active:
            self.dec.end()
        self.active = True
        return self.dec.begin(torch.tensor(ids))

    def decode(self) -> list[int]:
        return self.dec.step()

    def finish(self):
        if self.active:
            self.dec.end()
            self.active = False

    def logprobs(self, ids: list[int], top: int):
        return score(self.model, self.dec.st_t, ids, top)

    def check(self):
        mb = self.mailbox or getattr(self.model, 'mailbox', None)
        if mb is not None:
            mb.check()

    def snapshot(self, state) -> dict:
        snap = {}
        if self.mailbox is not None:
            from .utils.metrics import snapshot
            snap = snapshot(self.model, self.mailbox, state)
        snap.update({f'spec_{k}': v for k, v in self.dec.stats.items()})
        if self.recall is not None:
            st = self.recall.stats()
            snap.update(recall_offers=st['offers'], recall_landed=st['landed'], recall_probes=st['probes'])
            if st['record'] is not None:
                snap['recall_record_ids'] = st['record']['ids']
            if st['replies'] is not None:
                snap.update(recall_reply_hits=st['replies']['prompt_hits'], recall_replies=st['replies']['entries'])
        return snap


class Server:
    """Request handling of the HTTP endpoints over a backend (GenBackend, or a stand-in in the tests)."""

    def __init__(self, backend=None, max_queue: int = 8):
        self.backend = backend
        self.lock = threading.Lock()      # one request at a time on the model
        self.qlock = threading.Lock()     # the queue count
        self.max_queue = max_queue
        self.waiting = 0
        self.state = {'ready': backend is not None, 'requests': 0, 'tokens': 0, 'aborted': 0, 'rejected': 0,
                      'prompt_tokens': 0}
        self.stages = Stages()
        self._tele = (time.time(), 0, 0)   # (time, requests, tokens) of the last telemetry line

    def set_backend(self, backend):
        self.backend = backend
        self.state['ready'] = True
        self.stages.set('ready')

    def telemetry(self, every_s: float = 5.0, force: bool = False):
        """One log line with the counters' rates since the last line (at most one per `every_s`)."""
        now = time.time()
        t, r, n = self._tele
        if not force and now - t < every_s:
            return None
        dt = max(now - t, 1e-9)
        line = (f'[xtier_b200] decode {self.state["requests"] - r} req {self.state["tokens"] - n} tok '
                f'{(self.state["tokens"] - n) / dt:.1f} tok/s queue {self.waiting}')
        be = self.backend
        mb = getattr(be, 'mailbox', None)
        if mb is not None:
            st = mb.stats()
            line += f' cpu {st.get("calls", 0):.0f} calls {st.get("mean_us", 0) or 0:.0f} us'
        self._tele = (now, self.state['requests'], self.state['tokens'])
        print(line, flush=True)
        return line

    # ------------------------------------------------------------------ validation
    def _ids(self, req: dict) -> list[int]:
        be = self.backend
        if 'prompt_ids' in req:
            ids = req['prompt_ids']
            if not isinstance(ids, list) or not all(isinstance(t, int) and not isinstance(t, bool) for t in ids):
                raise BadRequest('prompt_ids must be a list of integers')
        elif 'prompt' in req:
            tok = getattr(be, 'tokenizer', None)
            if tok is None:
                raise BadRequest('this server has no tokenizer: send prompt_ids')
            if not isinstance(req['prompt'], str):
                raise BadRequest('prompt must be a string')
            from .utils.tokenize import parallel_encode
            ids = parallel_encode(tok, req['prompt'])
        else:
            raise BadRequest('prompt_ids (or prompt) is required')
        if not ids:
            raise BadRequest('empty prompt')
        bad = [t for t in ids if t < 0 or t >= be.vocab]
        if bad:
            raise BadRequest(f'token id {bad[0]} outside the vocabulary [0, {be.vocab})')
        return ids

    def parse_generate(self, req: dict):
        if not isinstance(req, dict):
            raise BadRequest('the body must be a JSON object')
        ids = self._ids(req)
        n = req.get('max_new_tokens', 16)
        if not isinstance(n, int) or isinstance(n, bool) or n < 1:
            raise BadRequest('max_new_tokens must be a positive integer')
        if len(ids) + n + 8 > self.backend.max_len:
            raise BadRequest(f'prompt ({len(ids)}) + max_new_tokens ({n}) exceed the server max length '
                             f'{self.backend.max_len}')
        stop = req.get('stop_ids', [])
        if not isinstance(stop, list) or not all(isinstance(t, int) for t in stop):
            raise BadRequest('stop_ids must be a list of integers')
        self.sampling_of(req)
        return ids, n, set(stop), bool(req.get('stream', False))

    def sampling_of(self, req: dict) -> tuple[float, float]:
        """(temperature, top_p) of a request; 400 when the backend decodes greedily and a temperature is asked."""
        temp = req.get('temperature', 0.0)
        top_p = req.get('top_p', 1.0)
        if temp is None:
            temp = 0.0
        if top_p is None:
            top_p = 1.0
        if not isinstance(temp, (int, float)) or isinstance(temp, bool) or not 0 <= temp <= 10:
            raise BadRequest('temperature must be a number in [0, 10]')
        if not isinstance(top_p, (int, float)) or isinstance(top_p, bool) or not 0 < top_p <= 1:
            raise BadRequest('top_p must be a number in (0, 1]')
        if temp > 0 and not getattr(self.backend, 'sampling', False):
            raise BadRequest('this server decodes greedily (start it with --sampling): send temperature 0 or none')
        return float(temp), float(top_p)

    def parse_chat(self, req: dict):
        """OpenAI chat request -> (prompt ids, max tokens, stop ids, stream, include usage, tools given)."""
        if not isinstance(req, dict):
            raise BadRequest('the body must be a JSON object')
        tok = getattr(self.backend, 'tokenizer', None)
        if tok is None or not hasattr(tok, 'apply_chat_template'):
            raise BadRequest('this server has no tokenizer with a chat template: use /v1/generate with prompt_ids')
        msgs = req.get('messages')
        if not isinstance(msgs, list) or not msgs or not all(isinstance(m, dict) and 'role' in m for m in msgs):
            raise BadRequest('messages must be a non-empty list of {"role": ..., "content": ...}')
        self.sampling_of(req)
        n = req.get('max_completion_tokens', req.get('max_tokens', 512))
        if not isinstance(n, int) or isinstance(n, bool) or n < 1:
            raise BadRequest('max_tokens must be a positive integer')
        tools = req.get('tools')
        kw = dict(req.get('chat_template_kwargs') or {})
        try:   # rendered to text, then encoded (in parallel slices when long)
            ids = tok.apply_chat_template(msgs, tools=tools, add_generation_prompt=True, tokenize=False, **kw)
        except TypeError:
            ids = tok.apply_chat_template(msgs, add_generation_prompt=True, tokenize=False)
        except Exception as e:   # noqa: BLE001 -- a template that refuses the messages
            raise BadRequest(f'chat template: {type(e).__name__}: {e}')
        if isinstance(ids, str):
            from .utils.tokenize import parallel_encode
            ids = parallel_encode(tok, ids)
        ids = list(ids['input_ids'] if isinstance(ids, dict) else ids)
        n = min(n, self.backend.max_len - len(ids) - 8)
        if n < 1:
            raise BadRequest(f'the prompt ({len(ids)} tokens) leaves no room under the server max length')
        stop = set()
        for t in (getattr(tok, 'eos_token_id', None), ):
            if isinstance(t, int):
                stop.add(t)
        conv = getattr(tok, 'convert_tokens_to_ids', None)
        if conv is not None:
            for name in ('<|im_end|>', '<|endoftext|>', '<|eot_id|>'):
                t = conv(name)
                if isinstance(t, int) and t >= 0 and t != getattr(tok, 'unk_token_id', None):
                    stop.add(t)
        opts = req.get('stream_options') or {}
        return ids, n, stop, bool(req.get('stream', False)), bool(opts.get('include_usage')), bool(tools)

    # ------------------------------------------------------------------ work
    def enter(self) -> bool:
        """Takes a place in the queue (False: full)."""
        with self.qlock:
            if self.waiting >= self.max_queue:
                self.state['rejected'] += 1
                return False
            self.waiting += 1
            return True

    def _started(self):
        with self.qlock:
            self.waiting -= 1

    def generate(self, ids, n, stop, emit=None, sampling=(0.0, 1.0)) -> dict:
        """Runs one request; emit(token) per new token returns False when the client is gone; sampling:
        (temperature, top_p)."""
        be = self.backend
        with self.lock:
            self._started()
            if hasattr(be, 'set_sampling'):
                be.set_sampling(*sampling)
            t0 = time.perf_counter()
            tok = be.prefill(ids)
            t_first = time.perf_counter()
            out, aborted = [tok], False
            if emit is not None and emit(tok) is False:
                aborted = True
            t_last = t_first
            try:
                while not aborted and len(out) < n and out[-1] not in stop:
                    got = be.decode()          # one token, or several (a speculative step)
                    for tok in (got if isinstance(got, list) else [got]):
                        if len(out) >= n or out[-1] in stop:
                            break
                        out.append(tok)
                        if emit is not None and emit(tok) is False:
                            aborted = True
                            break
                    t_last = time.perf_counter()
            finally:
                if hasattr(be, 'finish'):
                    be.finish()
            be.check()
            self.state['requests'] += 1
            self.state['tokens'] += len(out)
            self.state['prompt_tokens'] += len(ids)
            self.telemetry()
            if aborted:
                self.state['aborted'] += 1
        dec = t_last - t_first
        res = {'ids': out, 'prompt_tokens': len(ids), 'completion_tokens': len(out), 'ttft_s': t_first - t0,
               'decode_s': dec, 'decode_tok_s': (len(out) - 1) / dec if dec > 0 and len(out) > 1 else None,
               'aborted': aborted}
        tokz = getattr(be, 'tokenizer', None)
        if tokz is not None:
            res['text'] = tokz.decode(out)
        return res

    def parse_logprobs(self, req: dict):
        if not isinstance(req, dict):
            raise BadRequest('the body must be a JSON object')
        ids = self._ids(req)
        top = req.get('top', 0)
        if not isinstance(top, int) or isinstance(top, bool) or top < 0 or top > 100:
            raise BadRequest('top must be an integer in [0, 100]')
        if len(ids) < 2:
            raise BadRequest('scoring needs at least two tokens')
        if len(ids) + 8 > self.backend.max_len:
            raise BadRequest(f'{len(ids)} tokens exceed the server max length {self.backend.max_len}')
        return ids, top

    def logprobs(self, ids, top) -> dict:
        with self.lock:
            self._started()
            nll, tops = self.backend.logprobs(ids, top)
            self.backend.check()
            self.state['requests'] += 1
            self.state['prompt_tokens'] += len(ids)
        return {'nll': nll, 'top': tops, 'prompt_tokens': len(ids)}


class BatchBackend:
    """Continuous batching over a Generator of `gen.batch` decode rows: a request is prefilled into a free row while
    the others keep their KV; one replay of the captured decode step advances every row. Rows without a request decode
    a throw-away token at position 0 of their own KV row."""

    def __init__(self, model, gen, tokenizer=None, mailbox=None):
        import torch
        self.model, self.gen, self.tokenizer, self.mailbox = model, gen, tokenizer, mailbox
        self.vocab, self.max_len, self.rows = model.cfg.vocab, gen.max_len, gen.batch
        self.sampling = False
        pin = torch.cuda.is_available()
        self.host_pos = torch.zeros(self.rows, dtype=torch.int32, pin_memory=pin)
        self.score_state = None

    def capture(self):
        if self.gen.use_graph and self.gen.graph is None:
            self.gen.capture()

    def prefill_row(self, row: int, ids: list[int]) -> int:
        import torch
        g = self.gen
        t = int(self.model.prefill(g.state, torch.tensor(ids, device=self.model.device), row=row)[0])
        g.host_tokens[row] = t
        if 'prev' in g.buf:
            g.buf['prev'][row] = ids[-1]
        self.host_pos[row] = len(ids)
        return t

    def step(self, active: list[int]) -> list[int]:
        """One decode step of every row; the next token of each row (rows not in `active` are parked at 0)."""
        g = self.gen
        for r in range(self.rows):
            if r not in active:
                self.host_pos[r] = 0
        g.buf['pos'].copy_(self.host_pos, non_blocking=True)
        nxt = g.decode_one().tolist()
        for r in active:
            self.host_pos[r] += 1
        g.between_steps()
        return nxt

    def logprobs(self, ids: list[int], top: int):
        if self.score_state is None:
            self.score_state = self.model.alloc_state(1, self.max_len)
        return score(self.model, self.score_state, ids, top)

    def check(self):
        self.gen.check()

    def snapshot(self, state) -> dict:
        from .utils.metrics import snapshot
        return snapshot(self.model, self.mailbox, state)


class _Req:
    def __init__(self, ids, n, stop):
        import queue
        self.ids, self.n, self.stop = ids, n, stop
        self.q = queue.Queue()
        self.count, self.last, self.aborted, self.error, self.done = 0, None, False, None, False


class BatchServer(Server):
    """Server whose requests share the decode steps of a BatchBackend: a scheduler thread admits waiting requests
    into free rows (their prefill runs between two decode steps) and hands every step's tokens to the requests."""

    def __init__(self, backend=None, max_queue: int = 8):
        import collections
        super().__init__(backend, max_queue)
        self.cond = threading.Condition()
        self.pending = collections.deque()
        self.rows: dict = {}
        self.gpu = threading.Lock()
        self.thread = None
        if backend is not None:
            self._start()

    def set_backend(self, backend):
        super().set_backend(backend)
        self._start()

    def _start(self):
        if self.thread is None:
            self.thread = threading.Thread(target=self._loop, daemon=True, name='xtier-batch')
            self.thread.start()

    def _finish(self, row):
        req = self.rows.pop(row)
        req.done = True
        req.q.put(None)

    def _give(self, row, t):
        req = self.rows[row]
        req.count += 1
        req.last = t
        req.q.put(t)
        if req.count >= req.n or t in req.stop:
            self._finish(row)

    def _loop(self):
        be = self.backend
        while True:
            with self.cond:
                while not self.pending and not self.rows:
                    self.cond.wait()
                admit = []
                while self.pending and len(self.rows) < be.rows:
                    req = self.pending.popleft()
                    row = next(r for r in range(be.rows) if r not in self.rows)
                    self.rows[row] = req
                    admit.append((row, req))
            for row, req in admit:
                self._started()
                try:
                    with self.gpu:
                        t = be.prefill_row(row, req.ids)
                except Exception as e:   # noqa: BLE001 -- the request fails, the server goes on
                    req.error = e
                    self._finish(row)
                    continue
                self._give(row, t)
            for row in [r for r, q in self.rows.items() if q.aborted]:
                self._finish(row)
            active = sorted(self.rows)
            if not active:
                continue
            try:
                with self.gpu:
                    toks = be.step(active)
                    be.check()
            except Exception as e:   # noqa: BLE001 -- every running request fails with the step
                for row in active:
                    self.rows[row].error = e
                    self._finish(row)
                continue
            for row in active:
                self._give(row, toks[row])

    def generate(self, ids, n, stop, emit=None, sampling=(0.0, 1.0)) -> dict:
        req = _Req(ids, n, stop)
        t0 = time.perf_counter()
        with self.cond:
            self.pending.append(req)
            self.cond.notify()
        out, times = [], []
        while True:
            t = req.q.get()
            if t is None:
                break
            out.append(t)
            times.append(time.perf_counter())
            if emit is not None and emit(t) is False:
                req.aborted = True
                break
        if req.error is not None:
            raise req.error
        with self.qlock:
            self.state['requests'] += 1
            self.state['tokens'] += len(out)
            self.state['prompt_tokens'] += len(ids)
            self.telemetry()
            self.state['aborted'] += int(req.aborted)
        dec = times[-1] - times[0] if len(times) > 1 else 0.0
        res = {'ids': out, 'prompt_tokens': len(ids), 'completion_tokens': len(out),
               'ttft_s': (times[0] - t0) if times else None, 'decode_s': dec,
               'decode_tok_s': (len(out) - 1) / dec if dec > 0 else None, 'aborted': req.aborted}
        tokz = getattr(self.backend, 'tokenizer', None)
        if tokz is not None:
            res['text'] = tokz.decode(out)
        return res

    def logprobs(self, ids, top) -> dict:
        self._started()
        with self.gpu:
            nll, tops = self.backend.logprobs(ids, top)
        with self.qlock:
            self.state['requests'] += 1
            self.state['prompt_tokens'] += len(ids)
        return {'nll': nll, 'top': tops, 'prompt_tokens': len(ids)}


_TOOL_CALL = re.compile(r'<tool_call>\s*(\{.*?\})\s*</tool_call>', re.S)


def split_tool_calls(text: str):
    """(content without the <tool_call>{json}</tool_call> blocks or None, OpenAI tool_calls) of a reply; a block
    whose JSON does not parse stays in the content."""
    calls = []

    def take(m):
        try:
            obj = json.loads(m.group(1))
            name = obj['name']
        except (ValueError, KeyError, TypeError):
            return m.group(0)
        args = obj.get('arguments', {})
        calls.append({'id': f'call_{len(calls)}', 'type': 'function',
                      'function': {'name': name, 'arguments': args if isinstance(args, str) else json.dumps(args)}})
        return ''
    rest = _TOOL_CALL.sub(take, text).strip()
    return (rest or None) if calls else text, calls


def make_handler(server: Server):
    class Handler(BaseHTTPRequestHandler):
        server_version = 'xtier-b200'
        protocol_version = 'HTTP/1.1'

        def log_message(self, fmt, *a):
            pass

        def _send(self, code, data: bytes, ctype='application/json'):
            self.send_response(code)
            self.send_header('Content-Type', ctype)
            self.send_header('Content-Length', str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def _json(self, code, obj):
            self._send(code, json.dumps(obj).encode())

        def _chat(self):
            if not server.state['ready']:
                return self._json(503, {'error': {'message': 'loading'}})
            try:
                req = self._body()
                if req is None:
                    self.close_connection = True
                    return self._json(413, {'error': {'message': 'body too large'}})
                ids, n, stop, stream, usage, tools = server.parse_chat(req)
            except BadRequest as e:
                return self._json(400, {'error': {'message': str(e), 'type': 'invalid_request_error'}})
            if not server.enter():
                return self._json(503, {'error': {'message': 'queue full'}})
            tok = server.backend.tokenizer
            model = req.get('model') or 'xtier-b200'
            cid = f'chatcmpl-{time.time_ns():x}'
            created = int(time.time())

            def finish_reason(res):
                if res['ids'] and res['ids'][-1] in stop:
                    return 'stop'
                return 'length' if len(res['ids']) >= n else 'stop'

            def text_of(out):
                return tok.decode([t for t in out if t not in stop], skip_special_tokens=True)

            if not stream:
                try:
                    res = server.generate(ids, n, stop, sampling=server.sampling_of(req))
                except Exception as e:   # noqa: BLE001
                    return self._json(500, {'error': {'message': f'{type(e).__name__}: {e}'}})
                text = text_of(res['ids'])
                content, calls = split_tool_calls(text) if tools else (text, [])
                msg = {'role': 'assistant', 'content': content}
                if calls:
                    msg['tool_calls'] = calls
                done = len([t for t in res['ids'] if t not in stop])
                return self._json(200, {
                    'id': cid, 'object': 'chat.completion', 'created': created, 'model': model,
                    'choices': [{'index': 0, 'message': msg,
                                 'finish_reason': 'tool_calls' if calls else finish_reason(res)}],
                    'usage': {'prompt_tokens': len(ids), 'completion_tokens': done,
                              'total_tokens': len(ids) + done}})
            self.send_response(200)
            self.send_header('Content-Type', 'text/event-stream')
            self.send_header('Cache-Control', 'no-cache')
            self.send_header('Transfer-Encoding', 'chunked')
            self.end_headers()

            def event(obj) -> bool:
                data = b'data: ' + (obj if isinstance(obj, bytes) else json.dumps(obj).encode()) + b'\n\n'
                try:
                    self.wfile.write(b'%x\r\n%s\r\n' % (len(data), data))
                    self.wfile.flush()
                    return True
                except (BrokenPipeError, ConnectionResetError, OSError):
                    return False

            def chunk(delta, reason=None):
                return {'id': cid, 'object': 'chat.completion.chunk', 'created': created, 'model': model,
                        'choices': [{'index': 0, 'delta': delta, 'finish_reason': reason}]}
            out, sent = [], ['']

            def emit(t):
                out.append(t)
                text = text_of(out)
                if text.endswith('\ufffd'):      # an incomplete multi-byte character: wait for the next token
                    return True
                piece, sent[0] = text[len(sent[0]):], text
                return event(chunk({'content': piece})) if piece else True
            try:
                if not event(chunk({'role': 'assistant', 'content': ''})):
                    return None
                res = server.generate(ids, n, stop, emit, sampling=server.sampling_of(req))
                ok = event(chunk({}, finish_reason(res)))
                if ok and usage:
                    done = len([t for t in res['ids'] if t not in stop])
                    u = chunk({})
                    u['choices'] = []
                    u['usage'] = {'prompt_tokens': len(ids), 'completion_tokens': done,
                                  'total_tokens': len(ids) + done}
                    ok = event(u)
                if ok and event(b'[DONE]'):
                    self.wfile.write(b'0\r\n\r\n')
            except Exception as e:   # noqa: BLE001
                event({'error': {'message': f'{type(e).__name__}: {e}'}})
            self.close_connection = True
            return None

        def do_GET(self):
            if self.path == '/v1/models':
                return self._json(200, {'object': 'list', 'data': [{'id': 'xtier-b200', 'object': 'model',
                                                                    'owned_by': 'xtier-b200'}]})
            if self.path == '/health':
                be = server.backend
                info = {'ready': server.state['ready'], 'stage': server.stages.info()}
                if be is not None and server.state['ready']:
                    info.update(vocab=be.vocab, max_len=be.max_len, tokenizer=getattr(be, 'tokenizer', None) is not None)
                return self._json(200, info)
            if self.path in ('/metrics', '/metrics/prometheus'):
                from .utils.metrics import prometheus_text
                be = server.backend
                snap = be.snapshot(server.state) if be is not None and hasattr(be, 'snapshot') else {}
                snap.update({k: server.state[k] for k in ('requests', 'tokens', 'aborted', 'rejected',
                                                          'prompt_tokens')})
                snap['startup_s'] = server.stages.times
                if self.path == '/metrics':
                    return self._json(200, snap)
                return self._send(200, prometheus_text(snap).encode(), 'text/plain; version=0.0.4')
            self._json(404, {'error': 'not found'})

        def _body(self):
            try:
                n = int(self.headers.get('Content-Length', '0'))
            except ValueError:
                raise BadRequest('bad Content-Length')
            if n > MAX_BODY:
                return None
            raw = self.rfile.read(n) if n else b''
            try:
                return json.loads(raw or b'{}')
            except ValueError as e:
                raise BadRequest(f'body is not JSON: {e}')

        def do_POST(self):
            if self.path == '/flush_cache':
                self.rfile.read(int(self.headers.get('Content-Length', '0') or 0))
                be = server.backend
                if be is not None and hasattr(be, 'flush'):
                    with server.lock:
                        be.flush()
                return self._json(200, {'ok': True})
            if self.path == '/v1/chat/completions':
                return self._chat()
            if self.path not in ('/v1/generate', '/v1/logprobs'):
                return self._json(404, {'error': 'not found'})
            if not server.state['ready']:
                return self._json(503, {'error': 'loading'})
            try:
                req = self._body()
                if req is None:
                    self.close_connection = True
                    return self._json(413, {'error': 'body too large'})
                if self.path == '/v1/logprobs':
                    ids, top = server.parse_logprobs(req)
                else:
                    ids, n, stop, stream = server.parse_generate(req)
            except BadRequest as e:
                return self._json(400, {'error': str(e)})
            if not server.enter():
                return self._json(503, {'error': 'queue full'})
            if self.path == '/v1/logprobs':
                try:
                    return self._json(200, server.logprobs(ids, top))
                except Exception as e:   # noqa: BLE001 -- reported to the client, the server stays up
                    return self._json(500, {'error': f'{type(e).__name__}: {e}'})
            if not stream:
                try:
                    res = server.generate(ids, n, stop, sampling=server.sampling_of(req))
                except Exception as e:   # noqa: BLE001 -- reported to the client, the server stays up
                    return self._json(500, {'error': f'{type(e).__name__}: {e}'})
                return self._json(200, res)
            self.send_response(200)
            self.send_header('Content-Type', 'application/x-ndjson')
            self.send_header('Transfer-Encoding', 'chunked')
            self.end_headers()
            tokz = getattr(server.backend, 'tokenizer', None)

            def chunk(obj) -> bool:
                data = (json.dumps(obj) + '\n').encode()
                try:
                    self.wfile.write(b'%x\r\n%s\r\n' % (len(data), data))
                    self.wfile.flush()
                    return True
                except (BrokenPipeError, ConnectionResetError, OSError):
                    return False

            def emit(t):
                return chunk({'id': t, 'text': tokz.decode([t]) if tokz is not None else None})
            try:
                res = server.generate(ids, n, stop, emit, sampling=server.sampling_of(req))
                res['done'] = True
                if chunk(res):
                    self.wfile.write(b'0\r\n\r\n')
            except Exception as e:   # noqa: BLE001
                chunk({'done': True, 'error': f'{type(e).__name__}: {e}'})
            self.close_connection = True

    return Handler


def build_deepseek(args, stages: Stages):
    """The DeepSeek-V3-shaped model (MLA over the NVFP4 latent cache, 256 MXFP4 experts with grouped sigmoid top-8
    routing and a shared expert; random-init weights) on this GPU: `--hot` of each MoE layer's experts in HBM slots,
    the rest in the CPU engine through the mailbox. One request at a time, greedy; a prompt prefills in one forward
    and every token after it is a replay of the captured decode step."""
    from .engine.mailbox import Mailbox
    from .models.deepseek_v3 import DeepSeekV3Config, DeepSeekV3Model
    from .runtime.decode import Generator
    if args.checkpoint or args.sampling or args.batch > 1 or args.recall:
        raise ValueError('deepseek-v3 serves random-init weights greedily, one request at a time '
                         '(no --checkpoint, --sampling, --batch or --recall)')
    import torch
    cfg = DeepSeekV3Config(layers=args.layers or 61, attn='mla')
    # HBM slots: the --hot share, capped by what fits beside the dense weights with 6 GB kept for the KV cache, the
    # exchange and staging buffers and the workspaces
    free, _ = torch.cuda.mem_get_info()
    fit = (free - cfg.dense_bytes() - (6 << 30)) // max(1, cfg.expert_bytes() * cfg.moe_layers())
    gpu = max(1, min(cfg.experts, round(args.hot * cfg.experts), int(fit)))
    mailbox = Mailbox(cfg.hidden) if gpu < cfg.experts else None
    stages.set('weights')
    # the exchange buffers take a prompt chunk of up to 32 tokens (the mailbox's limit); decode uses one
    model = DeepSeekV3Model(cfg, device='cuda', seed=args.seed, ep=True, gpu_experts=gpu, mailbox=mailbox,
                            decode_tokens=32)
    model.keep_bf16_cache = True   # prompts prefill in chunks, each continuing the cached prefix
    stages.set('pool')
    if mailbox is not None:
        mailbox.start()
    stages.set('graphs')
    gen = Generator(model, batch=1, max_len=args.max_len)
    # no prefix reuse: the decode step writes only the NVFP4 latent cache, and a continuation prefill reads the BF16 one
    be = GenBackend(model, gen, None, mailbox, prefix_cache=False)
    be.prefill([0])        # captures the decode graph before the server says it is ready
    return be


def build(args, stages: Stages | None = None):
    from .engine.mailbox import Mailbox
    from .models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from .runtime.decode import Generator
    stages = stages or Stages(emit=lambda *a, **k: None)
    if args.model == 'deepseek-v3':
        return build_deepseek(args, stages)
    progress = lambda li, n: stages.set('weights', li, n)   # noqa: E731
    tok = None
    if args.checkpoint:
        from .models.hf import HFWeights
        cfg = HFWeights(args.checkpoint).cfg
        mailbox = Mailbox(cfg.hidden) if args.hot < 1.0 else None
        model = Qwen3MoeModel.from_pretrained(args.checkpoint, device='cuda', hot_fraction=args.hot, mailbox=mailbox,
                                              progress=progress)
        try:
            from transformers import AutoTokenizer
            tok = AutoTokenizer.from_pretrained(args.tokenizer or args.checkpoint)
        except Exception as e:   # noqa: BLE001 -- a checkpoint without tokenizer files serves token ids only
            print(f'[xtier_b200] no tokenizer ({type(e).__name__}); prompt_ids only', flush=True)
    else:
        cfg = Qwen3MoeConfig(layers=args.layers or 48)
        mailbox = Mailbox(cfg.hidden) if args.hot < 1.0 else None
        model = Qwen3MoeModel(cfg, device='cuda', seed=args.seed, hot_fraction=args.hot, mailbox=mailbox,
                              progress=progress)
    stages.set('pool')
    if mailbox is not None:
        mailbox.start()
    if args.recall:
        from . import recall
        ident = (recall.tokenizer_identity(tok, args.checkpoint or args.model) if tok is not None
                 else {'model': args.checkpoint or f'{args.model}-seed{args.seed}', 'vocab': model.cfg.vocab})
        rec = recall.Record(None if args.recall == 'memory' else args.recall, identity=ident,
                            budget_ids=int(args.recall_gib * (1 << 28)))
        eng = recall.RecallEngine(rec, gamma=args.recall_gamma)
        return SpecBackend(model, eng, max_len=args.max_len, tokenizer=tok, mailbox=mailbox)
    stages.set('graphs')
    if args.batch > 1:
        be = BatchBackend(model, Generator(model, batch=args.batch, max_len=args.max_len), tok, mailbox)
        be.capture()
        return be
    gen = Generator(model, batch=1, max_len=args.max_len, sampling=args.sampling)
    be = GenBackend(model, gen, tok, mailbox, prefix_cache=not args.no_prefix_cache)
    be.prefill([0])        # captures the decode graph before the server says it is ready
    return be


def serve(server: Server, host: str, port: int) -> ThreadingHTTPServer:
    """Starts the HTTP server on a thread; returns it (its server_address has the bound port)."""
    srv = ThreadingHTTPServer((host, port), make_handler(server))
    srv.daemon_threads = True
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--model', default='qwen3-moe', choices=MODELS)
    ap.add_argument('--checkpoint', default=None, help='a Hugging Face qwen3_moe checkpoint directory')
    ap.add_argument('--tokenizer', default=None, help='tokenizer directory (default: the checkpoint)')
    ap.add_argument('--layers', type=int, default=None, help='decoder layers (default: 48 qwen3-moe, 61 deepseek-v3)')
    ap.add_argument('--hot', type=float, default=0.4, help='fraction of each MoE layer\'s experts in HBM slots')
    ap.add_argument('--max-len', type=int, default=8192)
    ap.add_argument('--max-queue', type=int, default=8)
    ap.add_argument('--no-prefix-cache', action='store_true', help='prefill every prompt from its first token')
    ap.add_argument('--batch', type=int, default=1,
                    help='decode rows shared by concurrent requests (continuous batching; greedy, no prefix reuse)')
    ap.add_argument('--sampling', action='store_true',
                    help='temperature / top-p sampling in the decode step (requests without a temperature stay greedy)')
    ap.add_argument('--recall', default=None,
                    help='serve with Recall copy drafts verified by the target: a record directory, or "memory"')
    ap.add_argument('--recall-gib', type=float, default=1.0 / 16, help='record size budget (GiB of int32 ids)')
    ap.add_argument('--recall-gamma', type=int, default=16, help='longest copy draft')
    ap.add_argument('--seed', type=int, default=0)
    ap.add_argument('--host', default='127.0.0.1')
    ap.add_argument('--port', type=int, default=18180)
    args = ap.parse_args(argv)
    server = (BatchServer if args.batch > 1 else Server)(None, args.max_queue)
    serve(server, args.host, args.port)
    print(f'[xtier_b200] loading {args.checkpoint or args.model} ...', flush=True)
    server.stages.set('boot')
    try:
        server.set_backend(build(args, server.stages))
    except Exception as e:   # noqa: BLE001 -- the console shows why the start died
        server.stages.fail(f'{type(e).__name__}: {e}')
        raise
    from . import config
    if config.get('XTIER_GC_FREEZE'):
        from .utils.platform import freeze_gc
        print(f'[xtier_b200] GC heap frozen ({freeze_gc()} objects)', flush=True)
    print(f'[xtier_b200] ready on http://{args.host}:{args.port}', flush=True)
    try:
        threading.Event().wait()
    except KeyboardInterrupt:
        pass


if __name__ == '__main__':
    main()
