"""Console on the CPU: every option value of every card builds a command, the page renders, the API answers, POSTs
without the console header are refused, and a launch starts and stops a (stand-in) server process group."""
import json
import threading
import urllib.error
import urllib.request
from http.server import ThreadingHTTPServer

import pytest

from xtier_b200.console import __main__ as cmain
from xtier_b200.console import core


def test_every_option_builds_a_command():
    cards = core.load_cards()
    assert {'qwen3-moe', 'deepseek-v3'} <= set(cards)
    for card in cards.values():
        opts = card['options']
        for o in opts:
            for value, _ in o['choices']:
                argv, env, resolved = core.Console.command.__get__(type('C', (), {'cards': cards})())(
                    card['id'], {o['key']: value})
                assert argv and all(isinstance(a, str) for a in argv)
                assert resolved[o['key']] == value
                assert all(isinstance(v, str) for v in env.values())
        with pytest.raises(ValueError):
            core.validate(card, {'no_such_option': '1'})
        with pytest.raises(ValueError):
            core.validate(card, {opts[0]['key']: 'not-a-choice'})


def _serve(console):
    srv = ThreadingHTTPServer(('127.0.0.1', 0), cmain.make_handler(console, cmain.Jobs(console)))
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    return srv, f'http://127.0.0.1:{srv.server_address[1]}'


def test_page_api_and_post_guard(tmp_path):
    console = core.Console(tmp_path)
    srv, url = _serve(console)
    try:
        page = urllib.request.urlopen(url + '/').read().decode()
        assert 'xtier_b200 console' in page and 'qwen3-moe' in page
        st = json.loads(urllib.request.urlopen(url + '/api/status').read())
        assert st['running'] is False and 'qwen3-moe' in st['models']
        req = urllib.request.Request(url + '/api/stop', data=b'{}', method='POST',
                                     headers={'Content-Type': 'application/json'})
        with pytest.raises(urllib.error.HTTPError) as e:
            urllib.request.urlopen(req)
        assert e.value.code == 403
        req = urllib.request.Request(url + '/api/start', data=json.dumps({'model': 'nope'}).encode(), method='POST',
                                     headers={'Content-Type': 'application/json', 'X-Xtier-Console': '1'})
        with pytest.raises(urllib.error.HTTPError) as e:
            urllib.request.urlopen(req)
        assert e.value.code == 400
    finally:
        srv.shutdown()


def test_start_and_stop_a_server_process(tmp_path):
    cfg = tmp_path / 'cfg' / 'dummy'
    cfg.mkdir(parents=True)
    (cfg / 'console.py').write_text(
        "MODEL = {'id': 'dummy', 'name': 'dummy', 'port': 1, 'options': []}\n"
        "def build(options, port):\n"
        "    return ['python', '-c', 'import time; print(\"up\", flush=True); time.sleep(60)'], {}\n")
    console = core.Console(tmp_path / 'state', config_dir=tmp_path / 'cfg')
    cur = console.start('dummy', {})
    assert cur['pid'] > 0 and console.status()['running']
    assert console.stop() is True
    assert not console.status()['running']


def test_stages_and_telemetry_read_back():
    """The server's stage, telemetry and fatal lines, as the console reads them back from the log."""
    import io
    from xtier_b200.console import core
    from xtier_b200.serve import Server, Stages
    buf = io.StringIO()
    emit = lambda line, flush=True: buf.write(line + '\n')   # noqa: E731
    st = Stages(emit=emit)
    assert core.progress(buf.getvalue())['phase'] == 'boot'
    for li in range(4):
        st.set('weights', li, 4)
    p = core.progress(buf.getvalue())
    assert p['phase'] == 'weights' and p['percent'] == 8 + int(72 * 3 / 4)
    st.set('pool')
    st.set('graphs')
    st.set('ready')
    assert core.progress(buf.getvalue()) == {'phase': 'ready', 'label': 'ready', 'percent': 100}
    assert list(st.info()['times']) == ['boot', 'weights', 'pool', 'graphs', 'ready']
    with pytest.raises(ValueError):
        st.set('nonsense')
    # telemetry: rates since the last line
    srv = Server(None)
    srv.state.update(requests=3, tokens=250)
    line = srv.telemetry(force=True)
    t = core.telemetry(line)
    assert t['requests'] == 3 and t['tokens'] == 250 and t['queue'] == 0
    assert core.short(line).startswith('decode 3 req · 250 tok')
    assert srv.telemetry() is None                     # rate-limited
    # why a start died
    st.fail('RuntimeError: no CUDA device')
    text = buf.getvalue() + 'Traceback (most recent call last):\n  File "x"\nValueError: later noise\n'
    assert core.why_down(text) == '[xtier_b200] FATAL: RuntimeError: no CUDA device'
    assert core.why_down('ok\nnothing here\n') == ''
    assert core.why_down('x\nRuntimeError: CUDA error: out of memory\n') == 'RuntimeError: CUDA error: out of memory'


def test_oneshot_card_result(tmp_path):
    cfg = tmp_path / 'cfg' / 'tool'
    cfg.mkdir(parents=True)
    (cfg / 'console.py').write_text(
        "MODEL = {'id': 'tool', 'name': 'tool', 'port': 1, 'oneshot': True, 'options': []}\n"
        "def build(options, port):\n"
        "    return ['python', '-c', 'print(\"working\"); print(\\'{\"tok_s\": 22.2}\\')'], {}\n")
    console = core.Console(tmp_path / 'state', config_dir=tmp_path / 'cfg')
    console.start('tool', {})
    ok, why = console.wait_ready(60)
    assert ok and why == 'finished'
    st = console.status()
    assert not st['running'] and st['result'] == {'tok_s': 22.2} and 'down_reason' not in st
    assert core.last_json('a\n{"x": 1}\nnot json {\n') == {'x': 1} and core.last_json('none') is None
    cards = core.load_cards()
    assert cards['deepseek-v3-three-tier']['oneshot'] and not cards['deepseek-v3'].get('oneshot')
    argv, _ = cards['deepseek-v3']['build'](core.validate(cards['deepseek-v3'], {}), 18190)
    assert argv[:4] == ['python', '-m', 'xtier_b200.serve', '--model'] and argv[4] == 'deepseek-v3'
