"""CPU expert engine vs the FP32 dequant reference (the single-layer CPU config: H 2048, 64 routed experts of I 768 plus one
shared expert, NVFP4, softmax top-8 with renormalized weights, 16 bf16 tokens ~ N(0,1), seed 0)."""
import pytest
import torch

from xtier_b200 import formats
from xtier_b200.engine import CpuEngine, isa


def _routes(x, gate_w, k):
    logits = x.float() @ gate_w.T
    p = torch.softmax(logits, -1)
    w, ids = torch.topk(p, k, dim=-1)
    return ids.int(), (w / w.sum(-1, keepdim=True)).float()


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.fixture(scope='module')
def config1():
    torch.manual_seed(0)
    H, I, E = 2048, 768, 64
    experts = formats.random_experts(E, H, I, formats.NVFP4, seed=0)
    shared = formats.random_experts(1, H, I, formats.NVFP4, seed=1)
    gate_w = torch.randn(E, H, generator=torch.Generator().manual_seed(2)) * 0.02
    x = torch.randn(16, H, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    ids, w = _routes(x, gate_w, 8)
    ref = formats.reference_moe(x, ids, w, experts, shared=shared)
    return dict(experts=experts, shared=shared, x=x, ids=ids, w=w, ref=ref)


def test_config1_vs_fp32_reference(config1):
    eng = CpuEngine(config1['experts'], shared=config1['shared'], threads=4)
    y = eng.forward(config1['x'], config1['ids'], config1['w'])
    assert _rel(y, config1['ref']) < 2e-5, _rel(y, config1['ref'])


_DIGEST = """
import hashlib, torch
from xtier_b200 import formats
from xtier_b200.engine import CpuEngine
ex = formats.random_experts(16, 512, 256, formats.NVFP4, seed=0)
sh = formats.random_experts(1, 512, 256, formats.NVFP4, seed=1)
g = torch.Generator().manual_seed(3)
x = torch.randn(11, 512, generator=g).to(torch.bfloat16)
ids = torch.randint(0, 16, (11, 4), generator=g, dtype=torch.int32)
w = torch.rand(11, 4, generator=g)
y = CpuEngine(ex, shared=sh).forward(x, ids, w)
print(hashlib.sha1(y.numpy().tobytes()).hexdigest())
"""


def test_thread_count_does_not_change_bits():
    """The worker pool is per process, so each thread count runs in its own process."""
    import os
    import subprocess
    import sys
    digests = set()
    for t in (1, 3, 7):
        env = dict(os.environ, XTIER_THREADS=str(t))
        out = subprocess.run([sys.executable, '-c', _DIGEST], env=env, capture_output=True, text=True, check=True,
                             cwd=str(__import__('pathlib').Path(__file__).resolve().parent.parent))
        digests.add(out.stdout.strip().splitlines()[-1])
    assert len(digests) == 1, digests


@pytest.mark.parametrize('isa_name', ['scalar', 'avx2', 'avx512'])
def test_isas_agree(config1, isa_name, monkeypatch):
    monkeypatch.setenv('XTIER_ISA', isa_name)
    if isa_name == 'avx512' and isa() != 'avx512':
        pytest.skip('CPU lacks AVX-512 BF16')
    eng = CpuEngine(config1['experts'], shared=config1['shared'], threads=4)
    x, ids, w = config1['x'][:4], config1['ids'][:4], config1['w'][:4]
    y = eng.forward(x, ids, w)
    assert _rel(y, config1['ref'][:4]) < 2e-5


def test_skip_routes_and_decode(config1):
    eng = CpuEngine(config1['experts'], threads=4)
    ids = config1['ids'][:2].clone()
    ids[:, ::2] = -1   # routes served elsewhere
    ref = formats.reference_moe(config1['x'][:2], ids, config1['w'][:2], config1['experts'])
    y = eng.forward(config1['x'][:2], ids, config1['w'][:2], decode=True)
    assert _rel(y, ref) < 2e-5


def test_mxfp4_with_limit():
    H, I, E = 512, 256, 8
    ex = formats.random_experts(E, H, I, formats.MXFP4, seed=5, std=0.2)
    x = torch.randn(5, H).to(torch.bfloat16)
    ids = torch.randint(0, E, (5, 3), dtype=torch.int32)
    w = torch.rand(5, 3)
    ref = formats.reference_moe(x, ids, w, ex, limit=0.5)
    eng = CpuEngine(ex, threads=2, limit=0.5)
    y = eng.forward(x, ids, w)
    assert _rel(y, ref) < 2e-5


def test_gptoss_swiglu():
    H, I, E = 256, 128, 4
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=6, std=0.1)
    x = torch.randn(3, H).to(torch.bfloat16)
    ids = torch.tensor([[0, 1], [2, 3], [1, 2]], dtype=torch.int32)
    w = torch.rand(3, 2)
    ref = formats.reference_moe(x, ids, w, ex, alpha=1.702, beta=1.0)
    eng = CpuEngine(ex, threads=2)
    eng.set_swiglu(1.702, 1.0)
    assert _rel(eng.forward(x, ids, w), ref) < 2e-5


def test_tail_skip(monkeypatch):
    monkeypatch.setenv('XTIER_TAIL_SKIP', '1/2')
    H, I, E = 256, 128, 6
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=7)
    x = torch.randn(2, H).to(torch.bfloat16)
    ids = torch.tensor([[0, 1], [2, 1]], dtype=torch.int32)
    w = torch.tensor([[0.7, 0.3], [0.4, 0.6]])
    eng = CpuEngine(ex, threads=2)
    y = eng.forward(x, ids, w, decode=True)
    # token 0 keeps expert 0, token 1 keeps expert 1: expert 2 is left out everywhere, expert 1 stays for both
    ref = formats.reference_moe(x, torch.tensor([[0, 1], [-1, 1]], dtype=torch.int32), w, ex)
    assert _rel(y, ref) < 2e-5
    calls, distinct, dropped = eng.tail_stats()
    assert (calls, distinct, dropped) == (1, 3, 1)


def test_ram_slots_reject_missing_expert():
    H, I, E = 256, 128, 6
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=8)
    eng = CpuEngine(ex, threads=2, slots=3, resident=[0, 2, 4])
    x = torch.randn(1, H).to(torch.bfloat16)
    ok = eng.forward(x, torch.tensor([[0, 4]], dtype=torch.int32), torch.tensor([[0.5, 0.5]]))
    ref = formats.reference_moe(x, torch.tensor([[0, 4]], dtype=torch.int32), torch.tensor([[0.5, 0.5]]), ex)
    assert _rel(ok, ref) < 2e-5
    with pytest.raises(RuntimeError, match='not in RAM'):
        eng.forward(x, torch.tensor([[1, 4]], dtype=torch.int32), torch.tensor([[0.5, 0.5]]))
    tab = eng.slot_table()
    assert list(tab) == [0, -1, 1, -1, 2, -1]
    assert eng.place(1, 0) == 0
    assert list(eng.slot_table())[:2] == [-1, 0]
