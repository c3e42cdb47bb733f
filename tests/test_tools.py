"""Operations tools: CPU budget from a fake cgroup / sysfs tree, the host memory guard against a stand-in process
group, the low-priority launcher's command line, the VRAM hold size, the engine library's ISA check, and the
repository checks."""
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

from xtier_b200.tools import cpu_budget, isa_check, low_cpu, mem_guard, repo_check, vram_limit

ROOT = Path(__file__).resolve().parents[1]


def _tree(tmp_path, cpuset='0-15', cpu_max=None, v1_quota=None, nodes=('0-7', '8-15')):
    r = tmp_path / 'root'
    cg = r / 'sys/fs/cgroup'
    cg.mkdir(parents=True)
    (cg / 'cpuset.cpus.effective').write_text(cpuset + '\n')
    if cpu_max:
        (cg / 'cpu.max').write_text(cpu_max + '\n')
    if v1_quota:
        (cg / 'cpu').mkdir()
        (cg / 'cpu' / 'cpu.cfs_quota_us').write_text(f'{v1_quota[0]}\n')
        (cg / 'cpu' / 'cpu.cfs_period_us').write_text(f'{v1_quota[1]}\n')
    for i, cl in enumerate(nodes):
        d = r / f'sys/devices/system/node/node{i}'
        d.mkdir(parents=True)
        (d / 'cpulist').write_text(cl + '\n')
    return r


def test_cpu_budget(tmp_path):
    r = _tree(tmp_path / 'a')
    assert cpu_budget.cpuset(r) == set(range(16))
    assert cpu_budget.budget(reserve=2, root=r) == 14                    # 16 - 2, a multiple of the 2 nodes
    assert cpu_budget.budget(reserve=1, root=r) == 14                    # 15 rounded down to 2 nodes
    assert cpu_budget.budget(reserve=2, tp=2, root=r) == 6               # 8 per rank - 2
    r = _tree(tmp_path / 'b', cpu_max='800000 100000')
    assert cpu_budget.quota_cpus(r) == 8.0 and cpu_budget.budget(reserve=2, root=r) == 6
    r = _tree(tmp_path / 'c', cpu_max='max 100000', v1_quota=(300000, 100000))
    assert cpu_budget.quota_cpus(r) is None                              # v2 says no quota
    r = _tree(tmp_path / 'd', v1_quota=(300000, 100000))
    assert cpu_budget.quota_cpus(r) == 3.0 and cpu_budget.budget(reserve=2, root=r) == 1
    r = _tree(tmp_path / 'e', cpuset='0-3', nodes=('0-3', '4-7'))
    assert cpu_budget.budget(reserve=1, root=r) == 3                     # one node holds the CPUs


def test_mem_guard_kills_only_its_process_group(tmp_path):
    low = tmp_path / 'meminfo_low'
    low.write_text('MemTotal: 100000000 kB\nMemAvailable: 1048576 kB\n')
    high = tmp_path / 'meminfo_high'
    high.write_text('MemTotal: 100000000 kB\nMemAvailable: 104857600 kB\n')
    assert mem_guard.mem_available_gib(low) == 1.0
    p = subprocess.Popen([sys.executable, '-c', 'import time; time.sleep(60)'], start_new_session=True)
    try:
        logs = []
        assert mem_guard.guard(p.pid, min_gib=2.0, interval=0.05, meminfo=low, log=logs.append) == 1
        assert p.wait(timeout=10) != 0 and 'killing process group' in logs[0]
    finally:
        if p.poll() is None:
            p.kill()
    q = subprocess.Popen([sys.executable, '-c', 'import time; time.sleep(0.3)'], start_new_session=True)
    logs = []
    assert mem_guard.guard(q.pid, min_gib=2.0, interval=0.05, meminfo=high, log=logs.append) == 0
    q.wait(timeout=10)
    assert 'exited' in logs[-1]


def test_low_cpu_and_vram_limit():
    assert low_cpu.command(['make', '-j'], systemd=False) == ['nice', '-n', '19', 'make', '-j']
    assert low_cpu.command(['make'], cpus='70,71', systemd=True) == [
        'systemd-run', '--user', '--scope', '--quiet', '--collect', '-p', 'CPUWeight=1', '--',
        'taskset', '-c', '70,71', 'make']
    with pytest.raises(ValueError):
        low_cpu.command([], systemd=False)
    assert vram_limit.hold_bytes(10 << 30, 4096) == 6 << 30 and vram_limit.hold_bytes(1 << 30, 2048) < 0


def test_isa_check_on_the_built_engine():
    lib = ROOT / 'xtier_b200' / '_lib' / 'libxt_engine.so'
    if shutil.which('objdump') is None or not lib.exists():
        pytest.skip('objdump or the engine library missing')
    src = (ROOT / 'csrc' / 'engine' / 'kernels.cpp').read_text()
    assert isa_check.marked(src)['dot_avx512_n'] == 'avx512' and isa_check.marked(src)['dot_avx2'] == 'avx2'
    assert isa_check.check(str(lib), src) == []
    # the same library against a source that no longer marks one AVX-512 kernel: the check must notice
    unmarked = src.replace('XT_AVX512 static void prep_x_avx512', 'static void prep_x_avx512')
    found = isa_check.check(str(lib), unmarked)
    assert any('prep_x_avx512' in f for f in found)


def test_repo_check_is_clean():
    assert repo_check.run() == []
