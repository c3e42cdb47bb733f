"""Console logic: model cards, option validation, launching and stopping the model server.

A card is configs/<dir>/console.py defining MODEL = {'id', 'name', 'port', 'options': [{'key', 'label', 'default',
'choices': [[value, label], ...]}], ...} and build(options, port) -> (argv, env). The server runs in its own process
group (stopped with the whole group), its output goes to a log file the page tails, and readiness is polled on its
/health endpoint. The last settings are kept in a small JSON file.

Reference parity: xtier/console/core.py:372-601 (Console: start, stop, status, wait_ready).
"""
from __future__ import annotations

import importlib.util
import json
import os
import signal
import subprocess
import time
import urllib.request
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


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

    def wait_ready(self, timeout_s: float) -> tuple[bool, str]:
        t0 = time.time()
        while time.time() - t0 < timeout_s:
            if self.proc is None or self.proc.poll() is not None:
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

    def status(self) -> dict:
        running = self.proc is not None and self.proc.poll() is None
        return {'running': running, 'current': self.current, 'health': self.health() if running else None,
                'models': {k: {kk: v for kk, v in m.items() if kk != 'build'} for k, m in self.cards.items()}}
