"""The CPU expert engine and the cold store under ThreadSanitizer and under AddressSanitizer + UndefinedBehavior-
Sanitizer (csrc/engine/san_driver.cpp): two plans computing concurrently on the shared worker pool, a thread pinning
and unpinning slots meanwhile, and a cold-backed plan reading misses through the store's reader threads, each checked
bit-exactly against its single-threaded result. Needs g++ with the sanitizer runtimes; no GPU."""
import os
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
SRC = [ROOT / 'csrc/engine/san_driver.cpp', ROOT / 'csrc/engine/engine.cpp', ROOT / 'csrc/engine/kernels.cpp',
       ROOT / 'csrc/cold/store.cpp']


def _build(tmp: Path, mode: str) -> Path:
    exe = tmp / f'san_{mode.split(",")[0]}'
    cmd = ['g++', '-O1', '-g', '-std=c++17', '-pthread', f'-fsanitize={mode}', '-fno-omit-frame-pointer',
           f'-I{ROOT / "csrc/include"}', f'-I{ROOT / "csrc"}', *map(str, SRC), '-o', str(exe)]
    return exe, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)


@pytest.mark.skipif(shutil.which('g++') is None, reason='needs g++')
def test_engine_under_sanitizers(tmp_path):
    jobs = [_build(tmp_path, m) for m in ('thread', 'address,undefined')]
    for exe, proc in jobs:
        out, _ = proc.communicate(timeout=600)
        if proc.returncode != 0:
            if 'cannot find' in out and 'san' in out:
                pytest.skip('sanitizer runtime not installed')
            raise AssertionError(out[-3000:])
    env = dict(os.environ, TSAN_OPTIONS='halt_on_error=1', ASAN_OPTIONS='detect_leaks=0',
               UBSAN_OPTIONS='halt_on_error=1:print_stacktrace=1')
    for exe, _ in jobs:
        r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=900, env=env)
        assert r.returncode == 0 and 'ok' in r.stdout, (exe.name, r.stdout[-2000:], r.stderr[-4000:])
        assert 'WARNING: ThreadSanitizer' not in r.stderr and 'runtime error' not in r.stderr, r.stderr[-4000:]
