"""Run a CPU-heavy command next to a model server without slowing its decode: in a transient user scope of CPU weight 1
(`systemd-run --user --scope -p CPUWeight=1`), optionally only on the given CPUs (those without engine workers).

    python -m xtier_b200.tools.low_cpu [--cpus 70,71,78] -- COMMAND [ARGS...]

Every MoE layer of a decode step waits for all engine workers, which take nearly every core, so a busy neighbour that
takes a slice of one worker's core stalls the whole step. Linux divides contended CPU time between control groups
before it looks at nice values, so only a low-weight cgroup protects the server; without a user systemd the command runs
at nice 19, which does not (a warning says so).
(Reference parity: tools/low_cpu.sh.)
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys


def have_user_systemd() -> bool:
    if shutil.which('systemd-run') is None:
        return False
    r = subprocess.run(['systemd-run', '--user', '--scope', '--quiet', '--collect', 'true'],
                       stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    return r.returncode == 0


def command(argv: list[str], cpus: str | None = None, systemd: bool | None = None) -> list[str]:
    """The argv that runs `argv` at low CPU priority."""
    if not argv:
        raise ValueError('no command')
    cmd = (['taskset', '-c', cpus] if cpus else []) + list(argv)
    if systemd is None:
        systemd = have_user_systemd()
    if systemd:
        return ['systemd-run', '--user', '--scope', '--quiet', '--collect', '-p', 'CPUWeight=1', '--'] + cmd
    return ['nice', '-n', '19'] + cmd


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--cpus', default=os.environ.get('LOW_CPU_CPUS'))
    ap.add_argument('cmd', nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    cmd = a.cmd[1:] if a.cmd[:1] == ['--'] else a.cmd
    full = command(cmd, a.cpus)
    if full[0] == 'nice':
        print('low_cpu: no user systemd here, running at nice 19 (that does not protect the server)', file=sys.stderr)
    os.execvp(full[0], full)


if __name__ == '__main__':
    main()
