"""Host memory guard for a test server: kills the process group of PID when MemAvailable drops below MIN_GIB, so a
run that overcommits host memory cannot push the machine's other services into swap or the OOM killer.

    python -m xtier_b200.tools.mem_guard PID [--min-gib 20] [--interval 1]

Only the process group of the given PID is signalled (SIGKILL); the guard reports the lowest MemAvailable it saw when
PID exits on its own. Exit status 1 when it had to kill.
(Reference parity: tools/mem_guard.sh.)
"""
from __future__ import annotations

import argparse
import os
import signal
import sys
import time
from pathlib import Path


def mem_available_gib(meminfo='/proc/meminfo') -> float:
    for line in Path(meminfo).read_text().splitlines():
        if line.startswith('MemAvailable:'):
            return int(line.split()[1]) / (1 << 20)
    raise RuntimeError(f'{meminfo}: no MemAvailable line')


def _alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
    except ProcessLookupError:
        return False
    except PermissionError:
        return True
    try:   # a zombie child of this process counts as gone
        st = Path(f'/proc/{pid}/stat').read_text()
        return st[st.rindex(')') + 2] != 'Z'
    except (OSError, ValueError, IndexError):
        return True


def guard(pid: int, min_gib: float = 20.0, interval: float = 1.0, meminfo='/proc/meminfo', log=print) -> int:
    pgid = os.getpgid(pid)
    low = float('inf')
    while _alive(pid):
        avail = mem_available_gib(meminfo)
        low = min(low, avail)
        if avail < min_gib:
            log(f'{time.strftime("%F %T")} mem_guard: MemAvailable {avail:.1f} GiB < {min_gib} GiB, killing process '
                f'group {pgid} (pid {pid})')
            try:
                os.killpg(pgid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            return 1
        time.sleep(interval)
    log(f'{time.strftime("%F %T")} mem_guard: pid {pid} exited, lowest MemAvailable {low:.1f} GiB')
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('pid', type=int)
    ap.add_argument('--min-gib', type=float, default=20.0)
    ap.add_argument('--interval', type=float, default=1.0)
    a = ap.parse_args(argv)
    return guard(a.pid, a.min_gib, a.interval)


if __name__ == '__main__':
    sys.exit(main())
