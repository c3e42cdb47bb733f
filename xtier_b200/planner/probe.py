"""Planner probes: measure the cost-model coefficients on this machine.

GPU side: CUDA-event timings of the decode MoE kernels of a synthetic layer for growing numbers of hot routes
(-> g0, g1). CPU side: the engine's decode call for growing numbers of cold experts (-> c1), plus the mailbox round
trip of a call whose work is one tiny expert (-> c0). Results are written as {"coeffs": {...}, "samples": {...}}.

Reference parity: xtier/planner/probe.py:102-227 (graph timings of real mailbox/pool decode calls).
"""
from __future__ import annotations

import time

import torch

from .. import formats
from .cost import Coeffs, fit


def probe_cpu(H: int, I: int, fmt: str = formats.NVFP4, threads: int | None = None, reps: int = 30) -> list:
    from ..engine import CpuEngine
    E = 32
    ew = formats.synthetic_experts(E, H, I, fmt, 'cpu', seed=7)
    eng = CpuEngine(ew, threads=threads)
    x = torch.randn(1, H).bfloat16()
    samples = []
    for n in (1, 2, 4, 8):
        ids = torch.full((1, 8), -1, dtype=torch.int32)
        w = torch.rand(1, 8)
        for _ in range(5):
            ids[0, :n] = torch.randperm(E)[:n].int()
            eng.forward(x, ids, w, decode=True)
        t0 = time.perf_counter()
        for _ in range(reps):
            ids[0, :n] = torch.randperm(E)[:n].int()
            eng.forward(x, ids, w, decode=True)
        samples.append((n, (time.perf_counter() - t0) / reps * 1e6))
    eng.close()
    return samples


def probe_gpu(H: int, I: int, fmt: str = formats.NVFP4, reps: int = 50) -> list:
    from ..cache.pool import TieredMoE
    E = 64
    ew = formats.synthetic_experts(E, H, I, fmt, 'cuda', seed=8)
    samples = []
    x = torch.randn(1, H, device='cuda').bfloat16()
    for k in (1, 2, 4, 8):
        layer = TieredMoE(0, torch.randn(E, H) * 0.02, ew, k, device='cuda')
        out = torch.empty_like(x)
        for _ in range(5):
            layer.forward(x, out=out)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            layer.forward(x, out=out)
        e.record()
        torch.cuda.synchronize()
        samples.append((k, s.elapsed_time(e) / reps * 1e3))
    return samples


def measure(H: int, I: int, fmt: str = formats.NVFP4, threads: int | None = None, gpu: bool = True) -> dict:
    cpu = probe_cpu(H, I, fmt, threads)
    c0, c1 = fit(cpu)
    out = {'samples': {'cpu': cpu}}
    co = Coeffs(c0=max(c0, 1.0) + 8.0, c1=max(c1, 0.1))   # + the PCIe handshake both ways
    if gpu and torch.cuda.is_available():
        g = probe_gpu(H, I, fmt)
        g0, g1 = fit(g)
        co.g0, co.g1 = max(g0, 0.5), max(g1, 0.01)
        out['samples']['gpu'] = g
    out['coeffs'] = co.to_dict()
    out['shape'] = {'hidden': H, 'inter': I, 'fmt': fmt}
    return out
