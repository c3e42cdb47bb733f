"""CPU placement of one rank's CPU tier: which CPUs run the engine workers, which one the mailbox dispatcher, which
the Python main thread, and on which NUMA nodes the rank's expert shards live.

`plan()` splits the CPUs this process may use among the ranks of the node: by NUMA node when there are at least as
many nodes with CPUs as ranks (a rank takes whole nodes, preferring the node its GPU hangs off, read from sysfs), else
by contiguous slices of the allowed CPUs. Within the rank's CPUs the dispatcher takes one core (its hyper-thread
siblings are kept off the workers when the rank has CPUs to spare), the main thread another, the workers the rest.
`apply()` pins the calling (main) thread, exports the dispatcher and worker choices to the engine (XTIER_DISPATCH_CPU,
XTIER_WORKER_CPUS) and moves every other thread of the process off the worker CPUs.

Every sysfs read takes a `root` (default "/") so the tests run against a fake tree.
(Reference parity: xtier/engine/placement.py:1-20 -- per-rank NUMA groups, GPU-local node, pinned workers and
dispatcher, other threads moved off (XTIER_MAIN_CPUS); the partition rule here is this project's own.)
"""
from __future__ import annotations

import dataclasses
import os
from pathlib import Path

from .. import config


@dataclasses.dataclass
class Placement:
    rank: int
    nodes: list[int]          # NUMA nodes whose memory holds this rank's shards
    workers: list[int]        # engine worker CPUs
    dispatcher: int           # mailbox dispatcher CPU
    main: int                 # Python main thread CPU


def _read(root, rel: str) -> str | None:
    try:
        return (Path(root) / rel.lstrip('/')).read_text().strip()
    except OSError:
        return None


def numa_nodes(root='/', allowed: set[int] | None = None) -> dict[int, list[int]]:
    """NUMA node -> its CPUs (only allowed ones; nodes without any are left out). One node 0 when sysfs says nothing."""
    allowed = set(os.sched_getaffinity(0)) if allowed is None else set(allowed)
    out = {}
    base = Path(root) / 'sys/devices/system/node'
    if base.is_dir():
        for d in sorted(base.glob('node[0-9]*'), key=lambda p: int(p.name[4:])):
            txt = _read(root, f'sys/devices/system/node/{d.name}/cpulist')
            cpus = [c for c in (config.cpulist(txt) if txt else []) if c in allowed]
            if cpus:
                out[int(d.name[4:])] = cpus
    return out or {0: sorted(allowed)}


def gpu_node(pci_bus: str, root='/') -> int | None:
    """NUMA node of the PCI device `pci_bus` ("0000:1b:00.0"), None when unknown."""
    txt = _read(root, f'sys/bus/pci/devices/{pci_bus.lower()}/numa_node')
    try:
        n = int(txt) if txt is not None else -1
    except ValueError:
        return None
    return n if n >= 0 else None


def torch_gpu_bus(device: int) -> str | None:
    try:
        import torch
        p = torch.cuda.get_device_properties(device)
        return f'{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0'
    except Exception:
        return None


def _siblings(cpu: int, root='/') -> set[int]:
    txt = _read(root, f'sys/devices/system/cpu/cpu{cpu}/topology/thread_siblings_list')
    return set(config.cpulist(txt)) if txt else {cpu}


def plan(rank: int, world: int, root='/', allowed: set[int] | None = None,
         gpu_nodes: list[int | None] | None = None, spare_siblings: bool = True) -> Placement:
    """This rank's CPUs. gpu_nodes: the NUMA node of every rank's GPU (None entries: unknown); spare_siblings: keep
    the dispatcher's hyper-thread siblings free of workers."""
    nodes = numa_nodes(root, allowed)
    ids = sorted(nodes)
    if len(ids) >= world:
        per = len(ids) // world
        groups = [ids[g * per:(g + 1) * per] for g in range(world)]
        order = list(range(world))
        if gpu_nodes and len(gpu_nodes) == world and None not in gpu_nodes:
            # give each rank the group holding its GPU's node when that is a one-to-one match
            owner = [next((g for g, grp in enumerate(groups) if n in grp), None) for n in gpu_nodes]
            if None not in owner and len(set(owner)) == world:
                order = owner
        mine_nodes = groups[order[rank]]
        cpus = [c for n in mine_nodes for c in nodes[n]]
    else:
        every = [c for n in ids for c in nodes[n]]
        per = max(1, len(every) // world)
        cpus = every[rank * per:(rank + 1) * per] or every[-1:]
        mine_nodes = sorted({n for n in ids for c in cpus if c in nodes[n]})
    cpus = sorted(cpus)
    if len(cpus) == 1:
        return Placement(rank, mine_nodes, cpus, cpus[0], cpus[0])
    dispatcher = cpus[-1]
    rest = [c for c in cpus if c != dispatcher]
    sib = _siblings(dispatcher, root) - {dispatcher}
    if spare_siblings and len(rest) - len(sib) >= 2:   # the dispatcher's siblings stay idle when CPUs allow
        rest = [c for c in rest if c not in sib]
    main = rest[-1] if len(rest) >= 2 else rest[0]
    workers = [c for c in rest if c != main] or rest
    return Placement(rank, mine_nodes, workers, dispatcher, main)


def apply(p: Placement, move_others: bool = True) -> Placement:
    """Pins the calling thread to p.main, tells the engine and the mailbox where to run, and moves the process's
    other threads (already running ones) off the worker CPUs."""
    os.environ['XTIER_DISPATCH_CPU'] = str(p.dispatcher)
    os.environ['XTIER_WORKER_CPUS'] = ','.join(map(str, p.workers))
    allowed = set(os.sched_getaffinity(0))
    os.sched_setaffinity(0, {p.main})
    if move_others:
        off = (allowed | {p.main, p.dispatcher}) - set(p.workers) or {p.main}
        me = os.getpid()
        try:
            tids = [int(t) for t in os.listdir(f'/proc/{me}/task')]
        except OSError:
            tids = []
        for tid in tids:
            if tid == me:
                continue
            try:
                os.sched_setaffinity(tid, off)
            except OSError:
                pass
    return p


def for_rank(rank: int, world: int, spare_siblings: bool = True) -> Placement:
    """plan() for this machine, with the NUMA node of every local rank's GPU (device index = local rank)."""
    try:
        import torch
        n = torch.cuda.device_count()
    except Exception:
        n = 0
    gpus = [gpu_node(b) if (b := torch_gpu_bus(r)) else None for r in range(world)] if n >= world else None
    return plan(rank, world, gpu_nodes=gpus, spare_siblings=spare_siblings)
