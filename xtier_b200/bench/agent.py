"""Coding-agent benchmark against a running `xtier_b200.serve` (chat completions with tools, streamed): sessions that
start at a given context size and then work as an agent for a number of requests, each re-reading a growing prefix.

    python -m xtier_b200.bench.agent --url URL --tokenizer DIR [--sessions 8k,32k,64k] [--steps 12]
        [--source DIR] [--context-limit N] [--out FILE]
    python -m xtier_b200.bench.agent --table RESULT.json [RESULT.json ...]

Each session copies a source tree (default: this package's Python sources) into a temporary sandbox, gives the model a
task on it, and a history of earlier read_file calls that brings the prompt to the session's target size. Tools:
read_file / list_dir / grep / edit_file / write_file / check_python (py_compile only); nothing the model writes is
executed, every path stays inside the sandbox, which is removed afterwards. Every system prompt starts with the run's
own id. Per request: prompt tokens, time to the first streamed token, output tokens, decode tok/s (first to last
chunk), the tool calls; the first request of a session is its cold prefill (prefill tok/s = prompt tokens / TTFT).
A session ends when the model answers without a tool call, after --steps requests, or before a request could pass
--context-limit. `--table` prints per-session and overall summaries of result files.
(Reference parity: bench/agent_bench.py and bench/agent_table.py: the session shape, the sandboxed tools and the
per-request measures; the tasks, sizes and sources here are this project's own.)
"""
from __future__ import annotations

import argparse
import http.client
import json
import py_compile
import re
import shutil
import statistics
import sys
import tempfile
import time
from pathlib import Path

from .client import Client

TOOLS = [
    {'type': 'function', 'function': {'name': 'read_file', 'description': 'Read a file (with line numbers).',
     'parameters': {'type': 'object', 'properties': {'path': {'type': 'string'}, 'start_line': {'type': 'integer'},
                                                     'end_line': {'type': 'integer'}}, 'required': ['path']}}},
    {'type': 'function', 'function': {'name': 'list_dir', 'description': 'List a directory.',
     'parameters': {'type': 'object', 'properties': {'path': {'type': 'string'}}, 'required': ['path']}}},
    {'type': 'function', 'function': {'name': 'grep', 'description': 'Search a regex; returns path:line:text.',
     'parameters': {'type': 'object', 'properties': {'pattern': {'type': 'string'}, 'path': {'type': 'string'}},
                    'required': ['pattern']}}},
    {'type': 'function', 'function': {'name': 'edit_file', 'description': 'Replace the unique old_string by new_string.',
     'parameters': {'type': 'object', 'properties': {'path': {'type': 'string'}, 'old_string': {'type': 'string'},
                                                     'new_string': {'type': 'string'}},
                    'required': ['path', 'old_string', 'new_string']}}},
    {'type': 'function', 'function': {'name': 'write_file', 'description': 'Write (overwrite) a file.',
     'parameters': {'type': 'object', 'properties': {'path': {'type': 'string'}, 'content': {'type': 'string'}},
                    'required': ['path', 'content']}}},
    {'type': 'function', 'function': {'name': 'check_python', 'description': 'Syntax-check a Python file.',
     'parameters': {'type': 'object', 'properties': {'path': {'type': 'string'}}, 'required': ['path']}}},
]

SYSTEM = ('You are a coding agent working in a terminal on a Python project (a tiered MoE inference framework). Read '
          'the relevant code with the tools before changing it; change files with edit_file (old_string must match '
          'the file exactly and once) or write_file; check with check_python. Files read earlier in this '
          'conversation need no second read. When the task is done, give a short summary without a tool call.')

# name -> (target prompt tokens, task, files of the pre-filled history: task files first, then padding)
SESSIONS = {
    '8k': (8_000, 'Add a function `summary()` to bench/corpus.py that returns the number of ids and distinct ids of '
                  'a list; keep everything else unchanged, then check the file.',
           ['bench/corpus.py', 'bench/client.py']),
    '32k': (32_000, 'In bench/quality.py, make kl_compare also report the median KL; keep the existing fields.',
            ['bench/quality.py', 'bench/client.py', 'serve.py', 'cache/cold.py']),
    '64k': (64_000, 'Write a pytest file tests_sandbox/test_corpus.py with at least six tests of bench/corpus.py '
                    '(segments, prompt, id_stream), no GPU or network; check it.',
            ['bench/corpus.py', 'cache/pool.py', 'models/qwen3_moe.py', 'cache/cold.py', 'serve.py']),
    '128k': (128_000, 'Document every public function of recall/__init__.py that has no docstring yet; change no '
                      'behaviour; check the file.',
             ['recall/__init__.py', 'cache/pool.py', 'models/qwen3_moe.py', 'cache/cold.py', 'serve.py',
              'parallel/ep.py', 'planner/auto.py']),
}


class Sandbox:
    def __init__(self, source: Path):
        self.root = Path(tempfile.mkdtemp(prefix='xtier_agent_'))
        for f in source.rglob('*.py'):
            if '__pycache__' in f.parts or f.stat().st_size > 2_000_000:
                continue
            t = self.root / f.relative_to(source)
            t.parent.mkdir(parents=True, exist_ok=True)
            shutil.copy2(f, t)

    def path(self, p) -> Path:
        q = (self.root / str(p).lstrip('/')).resolve()
        if q != self.root and self.root not in q.parents:
            raise ValueError('path outside the working directory')
        return q

    def call(self, name: str, args: dict) -> str:
        fn = getattr(self, 't_' + name, None)
        if fn is None:
            return f'error: no tool {name}'
        try:
            return fn(**args)
        except TypeError as e:
            return f'argument error: {e}'
        except Exception as e:   # noqa: BLE001 -- tool errors go back to the model
            return f'error: {type(e).__name__}: {e}'

    def t_read_file(self, path, start_line=None, end_line=None):
        lines = self.path(path).read_text(encoding='utf-8', errors='replace').splitlines()
        a = max(1, int(start_line or 1))
        b = min(len(lines), int(end_line or len(lines)), a + 1999)
        return '\n'.join(f'{i:6d}\t{lines[i - 1]}' for i in range(a, b + 1))

    def t_list_dir(self, path='.'):
        d = self.path(path)
        return '\n'.join(sorted(p.name + ('/' if p.is_dir() else '') for p in d.iterdir()))

    def t_grep(self, pattern, path='.'):
        rx = re.compile(pattern)
        base = self.path(path)
        files = [base] if base.is_file() else sorted(base.rglob('*.py'))
        out = []
        for f in files:
            for i, line in enumerate(f.read_text(encoding='utf-8', errors='replace').splitlines(), 1):
                if rx.search(line):
                    out.append(f'{f.relative_to(self.root)}:{i}:{line}')
                    if len(out) >= 200:
                        return '\n'.join(out) + '\n... (first 200 matches)'
        return '\n'.join(out) or 'no match'

    def t_edit_file(self, path, old_string, new_string):
        f = self.path(path)
        text = f.read_text(encoding='utf-8')
        n = text.count(old_string)
        if n != 1:
            return f'error: old_string occurs {n} times (it must occur exactly once)'
        f.write_text(text.replace(old_string, new_string, 1), encoding='utf-8')
        return 'ok'

    def t_write_file(self, path, content):
        f = self.path(path)
        f.parent.mkdir(parents=True, exist_ok=True)
        f.write_text(content, encoding='utf-8')
        return f'ok: {len(content)} characters'

    def t_check_python(self, path):
        try:
            py_compile.compile(str(self.path(path)), doraise=True)
            return 'ok'
        except py_compile.PyCompileError as e:
            return f'syntax error: {e.msg}'

    def close(self):
        shutil.rmtree(self.root, ignore_errors=True)


def _history(sb: Sandbox, files: list[str], target: int, count) -> list[dict]:
    """Earlier read_file calls (task files, then more files) until the conversation holds about `target` tokens."""
    msgs, total = [], 0
    pool = list(files) + sorted(str(p.relative_to(sb.root)) for p in sb.root.rglob('*.py')
                                if str(p.relative_to(sb.root)) not in files)
    for i, f in enumerate(pool):
        if total >= target:
            break
        body = sb.call('read_file', {'path': f})
        call = {'id': f'h{i}', 'type': 'function', 'function': {'name': 'read_file',
                                                                'arguments': json.dumps({'path': f})}}
        msgs += [{'role': 'assistant', 'content': None, 'tool_calls': [call]},
                 {'role': 'tool', 'tool_call_id': f'h{i}', 'content': body}]
        total += count(body) + 16
    return msgs


def _request(cl: Client, body: dict) -> dict:
    """One streamed chat request, timed on arrival."""
    c = http.client.HTTPConnection(cl.host, cl.port, timeout=cl.timeout)
    t0 = time.perf_counter()
    c.request('POST', '/v1/chat/completions', json.dumps(body).encode(), {'Content-Type': 'application/json'})
    r = c.getresponse()
    if r.status != 200:
        raise RuntimeError(f'HTTP {r.status}: {r.read()[:500]!r}')
    times, text, usage, reason = [], [], None, None
    for line in r:
        line = line.decode().strip()
        if not line.startswith('data: '):
            continue
        data = line[6:]
        if data == '[DONE]':
            break
        ev = json.loads(data)
        if ev.get('usage'):
            usage = ev['usage']
        for ch in ev.get('choices', []):
            piece = ch.get('delta', {}).get('content')
            if piece:
                times.append(time.perf_counter())
                text.append(piece)
            reason = ch.get('finish_reason') or reason
    c.close()
    dec = times[-1] - times[0] if len(times) > 1 else 0.0
    return dict(text=''.join(text), ttft_s=(times[0] - t0) if times else None, decode_s=dec, usage=usage,
                finish_reason=reason, chunks=len(times))


def run_session(cl: Client, name: str, spec, source: Path, steps: int, count, run_id: str,
                context_limit: int, log=print) -> dict:
    from ..serve import split_tool_calls
    target, task, files = spec
    sb = Sandbox(source)
    try:
        msgs = [{'role': 'system', 'content': f'[run {run_id}] {SYSTEM}'}]
        msgs += _history(sb, files, target, count)
        msgs.append({'role': 'user', 'content': task})
        rows = []
        for step in range(steps):
            body = {'messages': msgs, 'tools': TOOLS, 'stream': True, 'stream_options': {'include_usage': True},
                    'max_tokens': 2048}
            prompt_est = sum(count(json.dumps(m)) for m in msgs)
            if prompt_est + 2048 > context_limit:
                log(json.dumps(dict(session=name, step=step, stopped='context limit')))
                break
            x = _request(cl, body)
            u = x['usage'] or {}
            out = u.get('completion_tokens', 0)
            row = dict(session=name, step=step, prompt_tokens=u.get('prompt_tokens'), output_tokens=out,
                       ttft_s=x['ttft_s'], decode_s=x['decode_s'],
                       decode_tps=(out - 1) / x['decode_s'] if x['decode_s'] and out > 1 else None)
            if step == 0 and x['ttft_s']:
                row['prefill_tps'] = (u.get('prompt_tokens') or 0) / x['ttft_s']
            content, calls = split_tool_calls(x['text'])
            row['tools'] = [c['function']['name'] for c in calls]
            rows.append(row)
            log(json.dumps(row))
            msgs.append({'role': 'assistant', 'content': content, **({'tool_calls': calls} if calls else {})})
            if not calls:
                break
            for c in calls:
                try:
                    args = json.loads(c['function']['arguments'] or '{}')
                except ValueError:
                    args = None
                result = (sb.call(c['function']['name'], args) if isinstance(args, dict)
                          else 'error: the arguments are not a JSON object')
                msgs.append({'role': 'tool', 'tool_call_id': c['id'], 'content': result[:200_000]})
        return dict(session=name, target=target, requests=rows)
    finally:
        sb.close()


def table(results: list[dict]) -> dict:
    """Per session and overall: requests, output tokens, decode tok/s (output tokens / decode seconds), cold prefill
    TTFT and tok/s, median TTFT of the later requests."""
    def agg(rows):
        timed = [r for r in rows if r.get('decode_s') and r.get('decode_tps')]
        out = sum(r['output_tokens'] for r in timed)
        dec = sum(r['decode_s'] for r in timed)
        later = [r['ttft_s'] for r in rows if r['step'] > 0 and r.get('ttft_s')]
        first = next((r for r in rows if r['step'] == 0), None)
        return dict(requests=len(rows), output_tokens=sum(r['output_tokens'] for r in rows),
                    decode_tps=round(out / dec, 2) if dec else None,
                    cold_ttft_s=round(first['ttft_s'], 3) if first and first.get('ttft_s') else None,
                    cold_prefill_tps=round(first['prefill_tps'], 1) if first and first.get('prefill_tps') else None,
                    later_ttft_s=round(statistics.median(later), 3) if later else None)
    per = {}
    every = []
    for res in results:
        for s in res['sessions']:
            per.setdefault(s['session'], []).extend(s['requests'])
            every += s['requests']
    return dict(sessions={k: agg(v) for k, v in per.items()}, all=agg(every))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--url', default='http://127.0.0.1:18180')
    ap.add_argument('--tokenizer')
    ap.add_argument('--sessions', default='8k,32k,64k')
    ap.add_argument('--steps', type=int, default=12)
    ap.add_argument('--source', default=str(Path(__file__).resolve().parents[1]))
    ap.add_argument('--context-limit', type=int, default=None)
    ap.add_argument('--table', nargs='*')
    ap.add_argument('--out')
    a = ap.parse_args(argv)
    if a.table:
        print(json.dumps(table([json.load(open(p)) for p in a.table]), indent=1))
        return 0
    if not a.tokenizer:
        raise SystemExit('--tokenizer is needed to size the sessions')
    from transformers import AutoTokenizer
    tok = AutoTokenizer.from_pretrained(a.tokenizer)
    cl = Client(a.url)
    st, info = cl.request('GET', '/health')
    limit = a.context_limit or info.get('max_len', 1 << 20)
    run_id = f'{time.time_ns():x}'
    count = lambda s: len(tok.encode(s, add_special_tokens=False))   # noqa: E731
    res = dict(run=run_id, sessions=[run_session(cl, n, SESSIONS[n], Path(a.source), a.steps, count, run_id, limit,
                                                 log=lambda s: print(s, file=sys.stderr))
                                     for n in a.sessions.split(',')])
    res['table'] = table([res])
    print(json.dumps(res['table']))
    if a.out:
        with open(a.out, 'w') as f:
            json.dump(res, f, indent=1)
    return 0


if __name__ == '__main__':
    sys.exit(main())
