"""Console logic: model cards, option validation, launching and stopping the model server.

A card is configs/<dir>/console.py defining MODEL = {'id', 'name', 'port', 'options': [{'key', 'label', 'default',
'choices': [[value, label], ...]}], ...} and build(options, port) -> (argv, env). The server runs in its own process
group (stopped with the whole group), its output goes to a log file the page tails, and readiness is polled on its
/health endpoint. The last settings are kept in a small JSON file.

The page's status also carries the server's startup stage (its stage log lines), the last telemetry line (requests,
tokens, tok/s, queue, CPU tier calls) and, once it is down, why (its FATAL line or the last error). A card with
'oneshot': True runs a measuring tool instead of a server: it is done when the process exits 0, and its result is the
last JSON line it printed.

Reference parity: xtier/console/core.py:372-601 (Console: start, stop, status, wait_ready), :294-370 (the log read back:
loading progress, short log lines, why a server is down).
"""
from __future__ import annotations

import importlib.util
import json
import os
import re
import signal
import subprocess
import time
import urllib.request
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]

# ------------------------------------------------------------------ the server log, read back
# stage lines (serve.Stages), telemetry lines (serve.Server.telemetry), fatal lines
_STAGE = re.compile(r'\[xtier_b200\] stage (\w+) (\d+)/(\d+)')
_TELE = re.compile(r'\[xtier_b200\] decode (\d+) req (\d+) tok ([\d.]+) tok/s queue (\d+)'
                   r'(?: cpu (\d+) calls (\d+) us)?')
_FATAL = re.compile(r'\[xtier_b200\] FATAL: [^\n]*|CUDA error[^\n]*|[A-Za-z]*Error: [^\n]*')
_ANSI = re.compile(r'\x1b\[[0-9;]*m')
_LABELS = {'boot': ('starting the process', 3), 'weights': ('loading weights', 8),
           'pool': ('expert pools, CPU engines', 84), 'graphs': ('capturing the decode graph', 92), 'ready': ('ready', 100)}


def progress(text: str) -> dict:
    """The server's startup stage from its log: the last stage line wins; weights advance 8 -> 80 % by layer."""
    found = _STAGE.findall(text or '')
    if not found:
        return {'phase': 'boot', 'label': _LABELS['boot'][0], 'percent': _LABELS['boot'][1]}
    phase, done, total = found[-1][0], int(found[-1][1]), int(found[-1][2])
    label, pct = _LABELS.get(phase, (phase, 0))
    if phase == 'weights' and total:
        pct = 8 + int(72 * done / total)
        label = f'{label} ({done}/{total} layers)'
    return {'phase': phase, 'label': label, 'percent': pct}


def why_down(text: str) -> str:
    """Why a server stopped, from its log: its own FATAL line, else the last error line (an exception's last line,
    a CUDA error); '' when the log names none."""
    found = _FATAL.findall(text or '')
    if not found:
        return ''
    fatal = [f for f in found if f.startswith('[xtier_b200] FATAL')]
    return (fatal[-1] if fatal else found[-1]).strip()[:300]


def telemetry(text: str) -> dict | None:
    """The last telemetry line of the log as numbers (requests and tokens since the line before, tok/s, queue, CPU
    tier calls and their mean time)."""
    found = _TELE.findall(text or '')
    if not found:
        return None
    req, tok, tps, queue, calls, us = found[-1]
    out = {'requests': int(req), 'tokens': int(tok), 'tok_s': float(tps), 'queue': int(queue)}
    if calls:
        out.update(cpu_calls=int(calls), cpu_us=int(us))
    return out


def short(line: str) -> str:
    """A log line for the page: colour codes dropped, the server's stage and telemetry lines in short."""
    line = _ANSI.sub('', line).rstrip()
    m = _TELE.search(line)
    if m:
        req, tok, tps, queue, calls, us = m.groups()
        out = f'decode {req} req · {tok} tok · {float(tps):.1f} tok/s'
        if queue != '0':
            out += f' · queue {queue}'
        if calls:
            out += f' · CPU tier {calls} calls, {us} us'
        return out
    m = _STAGE.search(line)
    if m:
        return f'stage {m.group(1)}' + (f' {m.group(2)}/{m.group(3)}' if m.group(3) != '0' else '')
    return line[:240]


def last_json(text: str) -> dict | None:
    """The last line of `text` that is a JSON object (what a one-shot tool prints as its result)."""
    for ln in reversed(text.splitlines()):
        ln = ln.strip()
        if ln.startswith('{') and ln.endswith('}'):
            try:
                return json.loads(ln)
            except ValueError:
                continue
    return None


def load_cards(config_dir: Path | None = None) -> dict:
    cards = {}
    for f in sorted((config_dir or ROOT / 'configs').glob('*/console.py')):
        spec = importlib.util.spec_from_file_location(f'xtier_card_{f.parent.name}', f)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        m = dict(mod.MODEL)
        m['build'] = mod.build
        m['dir'] = str(f.parent)
        cards[m['id']] = m
    return dict(sorted(cards.items(), key=lambda kv: kv[1].get('order', 0)))


def validate(card: dict, values: dict) -> dict:
    """Defaults filled in; unknown keys or values outside the choices raise ValueError."""
    out = {}
    known = {o['key']: o for o in card['options']}
    for k in values:
        if k not in known:
            raise ValueError(f'unknown option {k!r}')
    for k, o in known.items():
        v = str(values.get(k, o['default']))
        if v not in [c[0] for c in o['choices']]:
            raise ValueError(f'{k}={v!r} is not one of {[c[0] for c in o["choices"]]}')
        out[k] = v
    return out


class Console:
    def __init__(self, state_dir: Path | None = None, config_dir: Path | None = None):
        self.cards = load_cards(config_dir)
        self.state_dir = Path(state_dir or Path.home() / '.xtier_b200_console')
        self.state_dir.mkdir(parents=True, exist_ok=True)
        self.proc = None
        self.current = None

    def command(self, model: str, values: dict):
        card = self.cards[model]
        opts = validate(card, values)
        argv, env = card['build'](opts, card['port'])
        return argv, {k: str(v) for k, v in env.items()}, opts

    def start(self, model: str, values: dict) -> dict:
        self.stop()
        argv, env, opts = self.command(model, values)
        log = open(self.state_dir / f'{model}.log', 'ab')
        self.proc = subprocess.Popen(argv, cwd=str(ROOT), env={**os.environ, **env}, stdout=log,
                                     stderr=subprocess.STDOUT, start_new_session=True)
        self.current = {'model': model, 'options': opts, 'pid': self.proc.pid, 'started': time.time()}
        (self.state_dir / 'settings.json').write_text(json.dumps({model: opts}))
        return self.current

    def stop(self, reason: str = 'stopped') -> bool:
        if self.proc is None or self.proc.poll() is not None:
            self.proc = None
            self.current = None
            return False
        try:
            os.killpg(self.proc.pid, signal.SIGTERM)   # the server's own process group only
            self.proc.wait(timeout=30)
        except (ProcessLookupError, subprocess.TimeoutExpired):
            try:
                os.killpg(self.proc.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
        self.proc = None
        self.current = None
        return True

    def health(self) -> dict | None:
        if not self.current:
            return None
        port = self.cards[self.current['model']]['port']
        try:
            with urllib.request.urlopen(f'http://127.0.0.1:{port}/health', timeout=1) as r:
                return json.loads(r.read())
        except Exception:
            return None

    def oneshot(self) -> bool:
        """The current card runs a tool that prints a result and exits (no server, no /health)."""
        return bool(self.current and self.cards[self.current['model']].get('oneshot'))

    def wait_ready(self, timeout_s: float) -> tuple[bool, str]:
        t0 = time.time()
        while time.time() - t0 < timeout_s:
            if self.proc is None or self.proc.poll() is not None:
                if self.oneshot() and self.proc is not None and self.proc.returncode == 0:
                    return True, 'finished'
                return False, 'the server exited'
            h = self.health()
            if h and h.get('ready'):
                return True, 'ready'
            time.sleep(1)
        return False, 'timed out'

    def log_tail(self, lines: int = 40) -> list[str]:
        if not self.current:
            return []
        f = self.state_dir / f'{self.current["model"]}.log'
        if not f.exists():
            return []
        return f.read_text(errors='replace').splitlines()[-lines:]

    def _log_text(self, model: str | None = None, size: int = 262144) -> str:
        model = model or (self.current or {}).get('model') or getattr(self, '_last_model', None)
        if not model:
            return ''
        try:
            with open(self.state_dir / f'{model}.log', 'rb') as fh:
                fh.seek(0, os.SEEK_END)
                fh.seek(max(0, fh.tell() - size))
                return fh.read().decode('utf-8', 'replace')
        except OSError:
            return ''

    def status(self) -> dict:
        running = self.proc is not None and self.proc.poll() is None
        if self.current:
            self._last_model = self.current['model']
        text = self._log_text()
        out = {'running': running, 'current': self.current, 'health': self.health() if running else None,
               'models': {k: {kk: v for kk, v in m.items() if kk != 'build'} for k, m in self.cards.items()}}
        if text:
            out['stage'] = progress(text)
            out['telemetry'] = telemetry(text)
            out['log'] = [short(ln) for ln in text.splitlines()[-8:] if ln.strip()]
            if not running and self.oneshot() and self.proc is not None and self.proc.returncode == 0:
                out['result'] = last_json(text)
            elif not running:
                out['down_reason'] = why_down(text)
        return out
