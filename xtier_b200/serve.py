"""Minimal generation server over the framework's public API (the process the console launches).

    python -m xtier_b200.serve --model qwen3-moe [--layers 48] [--hot 0.4] [--max-len 8192] --port 18180

Endpoints: GET /health ({"ready": true} once the model is built and its decode step captured), GET /metrics (decode
counters, mailbox statistics, per-layer hit rates; /metrics/prometheus: the same in the Prometheus text format), POST /v1/generate {"prompt_ids": [...], "max_new_tokens": n} -> {"ids": [...],
"decode_tok_s": ...}. One request at a time (batch 1 decode, the CUDA graph of the tiered MoE model).
"""
from __future__ import annotations

import argparse
import json
import threading
import time
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import torch

MODELS = ('qwen3-moe',)


def build(args):
    from .engine.mailbox import Mailbox
    from .models.qwen3_moe import Qwen3MoeConfig, Qwen3MoeModel
    from .runtime.decode import Generator
    cfg = Qwen3MoeConfig(layers=args.layers)
    mailbox = Mailbox(cfg.hidden) if args.hot < 1.0 else None
    model = Qwen3MoeModel(cfg, device='cuda', seed=args.seed, hot_fraction=args.hot, mailbox=mailbox)
    if mailbox is not None:
        mailbox.start()
    return model, Generator(model, batch=1, max_len=args.max_len), mailbox


def make_handler(state):
    class Handler(BaseHTTPRequestHandler):
        server_version = 'xtier-b200'

        def log_message(self, fmt, *a):
            pass

        def _json(self, code, obj):
            data = json.dumps(obj).encode()
            self.send_response(code)
            self.send_header('Content-Type', 'application/json')
            self.send_header('Content-Length', str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            if self.path == '/health':
                return self._json(200, {'ready': state['ready']})
            if self.path in ('/metrics', '/metrics/prometheus'):
                from .utils.metrics import prometheus_text, snapshot
                snap = snapshot(state.get('model'), state.get('mailbox'), state)
                if self.path == '/metrics':
                    return self._json(200, snap)
                data = prometheus_text(snap).encode()
                self.send_response(200)
                self.send_header('Content-Type', 'text/plain; version=0.0.4')
                self.send_header('Content-Length', str(len(data)))
                self.end_headers()
                self.wfile.write(data)
                return
            self._json(404, {'error': 'not found'})

        def do_POST(self):
            if self.path != '/v1/generate':
                return self._json(404, {'error': 'not found'})
            if not state['ready']:
                return self._json(503, {'error': 'loading'})
            try:
                req = json.loads(self.rfile.read(int(self.headers.get('Content-Length', '0'))) or b'{}')
                ids = [int(t) for t in req['prompt_ids']]
                n = int(req.get('max_new_tokens', 16))
            except (KeyError, ValueError, TypeError) as e:
                return self._json(400, {'error': f'bad request: {e}'})
            with state['lock']:
                gen = state['gen']
                if len(ids) + n + 8 > gen.max_len:
                    return self._json(400, {'error': 'prompt + max_new_tokens exceed the server max length'})
                gen.prefill(torch.tensor([ids]))
                if gen.graph is None:
                    gen.capture()
                gen.host_tokens.copy_(gen.buf['tokens'].cpu())
                t0 = time.perf_counter()
                out = [int(gen.decode_one()[0]) for _ in range(n)]
                dt = time.perf_counter() - t0
                gen.check()
                state['requests'] += 1
                state['tokens'] += n
            self._json(200, {'ids': out, 'decode_tok_s': n / dt if dt > 0 else None})

    return Handler


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--model', default='qwen3-moe', choices=MODELS)
    ap.add_argument('--layers', type=int, default=48)
    ap.add_argument('--hot', type=float, default=0.4)
    ap.add_argument('--max-len', type=int, default=8192)
    ap.add_argument('--seed', type=int, default=0)
    ap.add_argument('--host', default='127.0.0.1')
    ap.add_argument('--port', type=int, default=18180)
    args = ap.parse_args(argv)
    state = {'ready': False, 'lock': threading.Lock(), 'requests': 0, 'tokens': 0}
    srv = ThreadingHTTPServer((args.host, args.port), make_handler(state))
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    print(f'[xtier_b200] loading {args.model} ...', flush=True)
    model, gen, mailbox = build(args)
    state.update(model=model, gen=gen, mailbox=mailbox, ready=True)
    print(f'[xtier_b200] ready on http://{args.host}:{args.port}', flush=True)
    try:
        threading.Event().wait()
    except KeyboardInterrupt:
        pass


if __name__ == '__main__':
    main()
