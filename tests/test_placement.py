"""CPU placement against a fake sysfs tree, and interleaved pinned host tables (host only)."""
import gc
import os

import torch

from xtier_b200.engine import memory, placement


def _fake_sysfs(root, nodes, siblings=None, gpu=None):
    for n, cpus in nodes.items():
        d = root / f'sys/devices/system/node/node{n}'
        d.mkdir(parents=True)
        (d / 'cpulist').write_text(cpus)
    for cpu, sib in (siblings or {}).items():
        d = root / f'sys/devices/system/cpu/cpu{cpu}/topology'
        d.mkdir(parents=True)
        (d / 'thread_siblings_list').write_text(sib)
    for bus, node in (gpu or {}).items():
        d = root / f'sys/bus/pci/devices/{bus}'
        d.mkdir(parents=True)
        (d / 'numa_node').write_text(str(node))


def test_plan_by_numa_node_with_gpu_affinity(tmp_path):
    _fake_sysfs(tmp_path, {0: '0-7', 1: '8-15'}, gpu={'0000:1b:00.0': 1, '0000:9c:00.0': 0})
    allowed = set(range(16))
    g = [placement.gpu_node('0000:1b:00.0', tmp_path), placement.gpu_node('0000:9c:00.0', tmp_path)]
    assert g == [1, 0]
    p0 = placement.plan(0, 2, tmp_path, allowed, g)
    p1 = placement.plan(1, 2, tmp_path, allowed, g)
    assert p0.nodes == [1] and p1.nodes == [0]           # each rank on its GPU's node
    assert p0.dispatcher == 15 and p0.main == 14 and p0.workers == list(range(8, 14))
    assert set(p1.workers) | {p1.main, p1.dispatcher} == set(range(8))


def test_plan_slices_and_siblings(tmp_path):
    _fake_sysfs(tmp_path, {0: '0-15'}, siblings={15: '7,15'})
    p = placement.plan(0, 1, tmp_path, set(range(16)))
    assert p.dispatcher == 15 and 7 not in p.workers and p.main == 14   # the dispatcher's sibling stays idle
    q = [placement.plan(r, 4, tmp_path, set(range(16))) for r in range(4)]
    cpus = [set(x.workers) | {x.main, x.dispatcher} for x in q]
    assert all(len(c) == 4 for c in cpus) and len(set().union(*cpus)) == 16


def test_apply_pins_main_thread(monkeypatch):
    monkeypatch.setenv('XTIER_DISPATCH_CPU', '')
    monkeypatch.setenv('XTIER_WORKER_CPUS', '')
    before = os.sched_getaffinity(0)
    cpus = sorted(before)
    p = placement.Placement(0, [0], cpus[:-1] or cpus, cpus[-1], cpus[-1])
    try:
        placement.apply(p, move_others=False)
        assert os.sched_getaffinity(0) == {cpus[-1]}
        assert os.environ['XTIER_DISPATCH_CPU'] == str(cpus[-1])
    finally:
        os.sched_setaffinity(0, before)


def test_pinned_interleaved_table():
    t, info = memory.pinned_interleaved(5 * 1024 * 1024 + 123, register=False)
    assert t.numel() == 5 * 1024 * 1024 + 123 and info['bytes'] % 4096 == 0
    t[:] = 7
    t[-1] = 3
    assert int(t[:-1].float().mean()) == 7 and int(t[-1]) == 3
    view = t[:4096].view(torch.int32)
    view[0] = 123456
    assert int(t[:4].view(torch.int32)[0]) == 123456
    del t, view
    gc.collect()
