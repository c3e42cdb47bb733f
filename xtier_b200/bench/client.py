"""HTTP client of `xtier_b200.serve` (stdlib only): generation (streamed or not, with an optional early disconnect),
prompt scoring, cache flush, health and metrics. Times are taken on the client, as a user sees them."""
from __future__ import annotations

import http.client
import json
import time
from urllib.parse import urlparse


class ServerError(RuntimeError):
    def __init__(self, status: int, body):
        super().__init__(f'HTTP {status}: {body}')
        self.status, self.body = status, body


class Client:
    def __init__(self, url: str = 'http://127.0.0.1:18180', timeout: float = 1800.0):
        u = urlparse(url if '://' in url else f'http://{url}')
        self.host, self.port = u.hostname or '127.0.0.1', u.port or 80
        self.timeout = timeout

    def _conn(self):
        return http.client.HTTPConnection(self.host, self.port, timeout=self.timeout)

    def request(self, method: str, path: str, body=None, raw: bytes | None = None):
        """(status, decoded JSON or text) of one request."""
        c = self._conn()
        try:
            data = raw if raw is not None else (json.dumps(body).encode() if body is not None else None)
            c.request(method, path, body=data, headers={'Content-Type': 'application/json'} if data else {})
            r = c.getresponse()
            text = r.read().decode('utf-8', 'replace')
            try:
                return r.status, json.loads(text)
            except ValueError:
                return r.status, text
        finally:
            c.close()

    def _ok(self, method, path, body=None):
        st, out = self.request(method, path, body)
        if st != 200:
            raise ServerError(st, out)
        return out

    # ------------------------------------------------------------------ endpoints
    def health(self) -> bool:
        try:
            return bool(self._ok('GET', '/health').get('ready'))
        except OSError:
            return False

    def wait_ready(self, timeout: float = 900.0, every: float = 1.0) -> bool:
        t_end = time.monotonic() + timeout
        while time.monotonic() < t_end:
            if self.health():
                return True
            time.sleep(every)
        return False

    def metrics(self) -> dict:
        return self._ok('GET', '/metrics')

    def flush(self):
        return self._ok('POST', '/flush_cache', {})

    def logprobs(self, ids: list[int], top: int = 0) -> dict:
        return self._ok('POST', '/v1/logprobs', {'prompt_ids': list(ids), 'top': top})

    def generate(self, ids=None, max_new_tokens: int = 16, prompt: str | None = None, stop_ids=None) -> dict:
        body = {'max_new_tokens': max_new_tokens}
        body.update({'prompt': prompt} if prompt is not None else {'prompt_ids': list(ids)})
        if stop_ids:
            body['stop_ids'] = list(stop_ids)
        t0 = time.perf_counter()
        out = self._ok('POST', '/v1/generate', body)
        out['client_s'] = time.perf_counter() - t0
        return out

    def stream(self, ids=None, max_new_tokens: int = 16, prompt: str | None = None, abort_after: int | None = None,
               on_token=None) -> dict:
        """Streamed generation, timed on arrival: ttft_s (request sent -> first token), decode_s (first -> last token),
        decode_tok_s, the gaps between tokens, the server's summary (`server`). abort_after=k closes the connection
        after k tokens (`aborted`: True)."""
        body = {'max_new_tokens': max_new_tokens, 'stream': True}
        body.update({'prompt': prompt} if prompt is not None else {'prompt_ids': list(ids)})
        c = self._conn()
        ids_out, times, summary, aborted = [], [], None, False
        try:
            t0 = time.perf_counter()
            c.request('POST', '/v1/generate', body=json.dumps(body).encode(),
                      headers={'Content-Type': 'application/json'})
            r = c.getresponse()
            if r.status != 200:
                raise ServerError(r.status, r.read().decode('utf-8', 'replace'))
            for line in r:
                line = line.strip()
                if not line:
                    continue
                msg = json.loads(line)
                if msg.get('done'):
                    summary = msg
                    break
                ids_out.append(msg['id'])
                times.append(time.perf_counter())
                if on_token is not None:
                    on_token(msg)
                if abort_after is not None and len(ids_out) >= abort_after:
                    aborted = True
                    break
        finally:
            c.close()
        if summary is not None and summary.get('error'):
            raise ServerError(500, summary['error'])
        gaps = [b - a for a, b in zip(times, times[1:])]
        dec = times[-1] - times[0] if len(times) > 1 else 0.0
        return dict(ids=ids_out, ttft_s=(times[0] - t0) if times else None, decode_s=dec,
                    decode_tok_s=(len(times) - 1) / dec if dec > 0 else None, max_gap_s=max(gaps) if gaps else 0.0,
                    times=times, t0=t0, aborted=aborted, server=summary)
