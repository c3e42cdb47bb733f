"""CPU engine worker threads this process can use: the CPUs of its cgroup cpuset (a container's; else the affinity
mask), capped by the cgroup CPU quota (v2 `cpu.max`, v1 `cpu.cfs_quota_us` / `cpu.cfs_period_us`), less `--reserve`
per rank for the Python main thread and the mailbox dispatcher, rounded down to a multiple of the NUMA nodes that hold
those CPUs (the engine splits its workers evenly over the nodes of its shards). With --tp N the count is per rank: the
CPUs are split over N ranks first.

    python -m xtier_b200.tools.cpu_budget [--reserve 2] [--tp 1]      -> prints the number (for XTIER_THREADS)

Every file read takes a `root` (default "/"), so the tests run against a fake tree.
(Reference parity: tools/cpu_budget.py -- cpuset, quota, scheduler reserve, NUMA multiple, per-rank split.)
"""
from __future__ import annotations

import argparse
import math
import os
from pathlib import Path

from .. import config


def _read(root, rel: str) -> str | None:
    try:
        return (Path(root) / rel.lstrip('/')).read_text().strip()
    except OSError:
        return None


def cpuset(root='/') -> set[int]:
    """The cgroup's effective cpuset (v2, then v1), else this process's affinity mask."""
    for rel in ('sys/fs/cgroup/cpuset.cpus.effective', 'sys/fs/cgroup/cpuset/cpuset.effective_cpus',
                'sys/fs/cgroup/cpuset/cpuset.cpus'):
        txt = _read(root, rel)
        if txt:
            return set(config.cpulist(txt))
    return set(os.sched_getaffinity(0))


def quota_cpus(root='/') -> float | None:
    """CPUs worth of the cgroup CPU quota; None without one."""
    txt = _read(root, 'sys/fs/cgroup/cpu.max')
    if txt:
        q, _, p = txt.partition(' ')
        if q != 'max':
            return int(q) / int(p or 100000)
        return None
    q = _read(root, 'sys/fs/cgroup/cpu/cpu.cfs_quota_us') or _read(root, 'sys/fs/cgroup/cpu,cpuacct/cpu.cfs_quota_us')
    p = _read(root, 'sys/fs/cgroup/cpu/cpu.cfs_period_us') or _read(root, 'sys/fs/cgroup/cpu,cpuacct/cpu.cfs_period_us')
    if q and p and int(q) > 0:
        return int(q) / int(p)
    return None


def budget(reserve: int = 2, tp: int = 1, root='/') -> int:
    """Worker threads per rank (at least 1)."""
    from ..engine.placement import numa_nodes
    cpus = cpuset(root)
    nodes = numa_nodes(root, cpus)
    usable = len(cpus)
    q = quota_cpus(root)
    if q is not None:
        usable = min(usable, int(math.floor(q)))
    per_rank = usable // max(1, tp) - reserve
    nodes_per_rank = max(1, len(nodes) // max(1, tp))
    if per_rank >= nodes_per_rank:
        per_rank -= per_rank % nodes_per_rank
    return max(1, per_rank)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split('\n\n')[0])
    ap.add_argument('--reserve', type=int, default=2, help='CPUs kept per rank for the main thread and dispatcher')
    ap.add_argument('--tp', type=int, default=1, help='ranks sharing the CPUs')
    a = ap.parse_args(argv)
    print(budget(a.reserve, a.tp))
    return 0


if __name__ == '__main__':
    raise SystemExit(main())
