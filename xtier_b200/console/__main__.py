"""python -m xtier_b200.console [--host 127.0.0.1] [--port 8765] [--state-dir DIR]

Serves the console page and its JSON API: GET /api/status, GET /api/job, POST /api/start {model, values},
POST /api/stop. POSTs must carry JSON and the X-Xtier-Console header (a page of another origin cannot add that header
without a CORS preflight, which this server never answers), so another web page open in the browser cannot launch or
stop servers. Listens on 127.0.0.1 by default; reach it from another machine through an SSH tunnel.
(reference parity: xtier/console/__main__.py:89-123)
"""
import argparse
import json
import threading
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

from .. import config
from . import core, ui

API = {'start': 'api/start', 'stop': 'api/stop', 'status': 'api/status', 'job': 'api/job'}


class Jobs:
    """One launch at a time, in the background (stop the running server, start, wait until ready)."""

    def __init__(self, console):
        self.console = console
        self.lock = threading.Lock()
        self.job = {'id': 0, 'state': 'idle'}

    def launch(self, model, values):
        with self.lock:
            if self.job['state'] == 'running':
                return None, 'a launch is already in progress'
            core.validate(self.console.cards[model], values)
            self.job = {'id': self.job['id'] + 1, 'state': 'running', 'model': model, 'error': ''}
            job = self.job
        threading.Thread(target=self._run, args=(job, model, values), daemon=True).start()
        return job, ''

    def _run(self, job, model, values):
        try:
            self.console.start(model, values)
            ok, detail = self.console.wait_ready(self.console.cards[model].get('ready_timeout', 600))
            job.update(state='done' if ok else 'failed', error='' if ok else detail)
        except Exception as e:   # shown on the page
            job.update(state='failed', error=str(e))


def make_handler(console, jobs):
    class Handler(BaseHTTPRequestHandler):
        server_version = 'xtier-b200-console'

        def log_message(self, *a):
            pass

        def _send(self, code, body, ctype='application/json'):
            data = body.encode()
            self.send_response(code)
            self.send_header('Content-Type', ctype)
            self.send_header('Content-Length', str(len(data)))
            self.end_headers()
            self.wfile.write(data)

        def do_GET(self):
            path = self.path.split('?')[0].lstrip('/')
            if path == '':
                return self._send(200, ui.page_html(console.cards, API), 'text/html; charset=utf-8')
            if path == API['status']:
                return self._send(200, json.dumps(console.status()))
            if path == API['job']:
                return self._send(200, json.dumps({**jobs.job, 'log': console.log_tail()}))
            self._send(404, json.dumps({'error': 'not found'}))

        def do_POST(self):
            path = self.path.lstrip('/')
            if self.headers.get('X-Xtier-Console') != '1' or 'json' not in self.headers.get('Content-Type', ''):
                return self._send(403, json.dumps({'error': 'console POSTs need JSON and the X-Xtier-Console header'}))
            try:
                body = json.loads(self.rfile.read(int(self.headers.get('Content-Length', '0'))) or b'{}')
            except json.JSONDecodeError:
                return self._send(400, json.dumps({'error': 'bad JSON'}))
            if path == API['start']:
                model = body.get('model')
                if model not in console.cards:
                    return self._send(400, json.dumps({'error': f'unknown model {model!r}'}))
                try:
                    job, err = jobs.launch(model, body.get('values', {}))
                except ValueError as e:
                    return self._send(400, json.dumps({'error': str(e)}))
                return self._send(200 if job else 409, json.dumps(job or {'error': err}))
            if path == API['stop']:
                return self._send(200, json.dumps({'stopped': console.stop()}))
            self._send(404, json.dumps({'error': 'not found'}))

    return Handler


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--host', default='127.0.0.1')
    ap.add_argument('--port', type=int, default=config.get('XTIER_CONSOLE_PORT'))
    ap.add_argument('--state-dir', default=None)
    a = ap.parse_args(argv)
    console = core.Console(a.state_dir)
    srv = ThreadingHTTPServer((a.host, a.port), make_handler(console, Jobs(console)))
    print(f'xtier_b200 console on http://{a.host}:{a.port}', flush=True)
    try:
        srv.serve_forever()
    finally:
        console.stop()


if __name__ == '__main__':
    main()
