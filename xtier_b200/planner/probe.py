"""Planner probes: measure the cost-model coefficients on this machine.

GPU side: the decode MoE call of a synthetic layer (route, gate/up, down) for growing numbers of hot routes, timed as
CUDA-graph replays (no launch cost) -> g0, g1. CPU side: the engine's decode call for growing numbers of cold
experts -> c1. Mailbox: the round trip of a captured decode call of a layer without GPU slots whose single route goes
to a tiny expert on the CPU engine, minus that expert's engine time -> c0 (GPU publish, dispatcher wake-up, engine
hand-off and the GPU's poll, both PCIe directions). NVLink: with a second GPU, the time to read one expert's weights
from the peer's memory (device-to-device copy over the NVLink path, events on the reader) -> p1, the cost of a route
to an expert another GPU's slot pool holds. PCIe: the staging copy kernel (`ep_stage`) of 1-8 experts from a CPU
engine's registered host memory, as graph replays -> h1 per staged expert. Results are written as {"coeffs": {...},
"samples": {...}}.

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


def _graph_time_us(fn, reps: int) -> float:
    """Device time of one fn() call: `reps` calls captured in a CUDA graph, replayed after warm-up."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    g.replay()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    g.replay()
    b.record()
    torch.cuda.synchronize()
    del g
    return a.elapsed_time(b) / reps * 1e3


def probe_gpu(H: int, I: int, fmt: str = formats.NVFP4, reps: int = 50) -> list:
    from ..cache.pool import TieredMoE
    E = 64
    ew = formats.synthetic_experts(E, H, I, fmt, 'cuda', seed=8)
    samples = []
    x = torch.randn(1, H, device='cuda').bfloat16()
    for k in (1, 2, 4, 8):
        layer = TieredMoE(0, torch.randn(E, H) * 0.02, ew, k, device='cuda')
        out = torch.empty_like(x)
        samples.append((k, _graph_time_us(lambda: layer.forward(x, out=out), reps)))
    return samples


def probe_mailbox(H: int, fmt: str = formats.NVFP4, threads: int | None = None, reps: int = 30) -> dict:
    """Captured decode call of a layer without GPU slots (one route per call, a tiny expert of 128 intermediate
    units on the CPU engine) and that expert's engine time alone: their difference is the mailbox round trip."""
    from ..cache.pool import TieredMoE
    from ..engine import CpuEngine
    from ..engine.mailbox import Mailbox
    E, I = 4, 128
    ew = formats.synthetic_experts(E, H, I, fmt, 'cpu', seed=9)
    eng = CpuEngine(ew, threads=threads)
    mb = Mailbox(H, timeout_s=10.0)
    layer = TieredMoE(0, torch.randn(E, H) * 0.02, ew, 1, hot=[], mailbox=mb, engine=eng, device='cuda')
    mb.start()
    try:
        x = torch.randn(1, H, device='cuda').bfloat16()
        out = torch.empty_like(x)
        call = _graph_time_us(lambda: layer.forward(x, out=out), reps)
        mb.check()
        xc, ids, w = x.cpu(), torch.zeros(1, 1, dtype=torch.int32), torch.ones(1, 1)
        for _ in range(5):
            eng.forward(xc, ids, w, decode=True)
        t0 = time.perf_counter()
        for _ in range(reps):
            eng.forward(xc, ids, w, decode=True)
        engine = (time.perf_counter() - t0) / reps * 1e6
    finally:
        mb.stop()
        mb.close()
        eng.close()
    return {'call_us': call, 'engine_us': engine}


def probe_peer(H: int, I: int, fmt: str = formats.NVFP4, reps: int = 20) -> dict | None:
    """Time for GPU 0 to read one expert's weights from GPU 1's memory (device-to-device copy, events on GPU 0):
    the NVLink term of a route to an expert another GPU's pool holds. None with fewer than two GPUs. The decode
    kernels read peer slots with 16-byte loads, so this DMA rate is the upper bound they approach."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        return None
    one = formats.synthetic_experts(1, H, I, fmt, 'cpu', seed=10)
    nbytes = one.nbytes_per_expert()
    src = torch.empty(nbytes, dtype=torch.uint8, device='cuda:1')
    dst = torch.empty(nbytes, dtype=torch.uint8, device='cuda:0')
    with torch.cuda.device(0):
        for _ in range(3):
            dst.copy_(src)
        torch.cuda.synchronize(0)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            dst.copy_(src)
        b.record()
        torch.cuda.synchronize(0)
        us = a.elapsed_time(b) / reps * 1e3
    return {'bytes': nbytes, 'us': us, 'gbs': nbytes / us / 1e3, 'peer_access': torch.cuda.can_device_access_peer(0, 1)}


def probe_pcie(H: int, I: int, fmt: str = formats.NVFP4, reps: int = 10) -> list:
    """The PCIe staging copy (`ep_stage`) of n = 1, 2, 4, 8 experts from a CPU engine's registered host memory into
    GPU staging slots, timed as CUDA-graph replays -> h1 (us per staged expert)."""
    from ..engine import CpuEngine
    from ..parallel.ep import map_engine, unmap_engine
    E, S = 8, 8
    ew = formats.synthetic_experts(E, H, I, fmt, 'cpu', seed=11)
    eng = CpuEngine(ew, threads=1)
    g13 = ew.g13.float().cuda()
    g2 = ew.g2.float().cuda()
    stage, regs = map_engine(eng, list(range(E)), E, g13, g2)
    if stage is None:
        eng.close()
        return []
    try:
        bs = formats.BLOCK[fmt]
        u8 = lambda *shape: torch.zeros(*shape, dtype=torch.uint8, device='cuda')   # noqa: E731
        st = (u8(S, 2 * I, H // 2), u8(S, 2 * I, H // bs), u8(S, H, I // 2), u8(S, H, I // bs),
              torch.ones(S, 2, device='cuda'), torch.ones(S, device='cuda'))
        idx = stage['cold_index'].cuda()
        claim_list = torch.arange(E, dtype=torch.int32, device='cuda')
        claim = torch.full((E,), -1, dtype=torch.int32, device='cuda')
        count = torch.zeros(1, dtype=torch.int32, device='cuda')
        done = torch.zeros(1, dtype=torch.int32, device='cuda')
        fmt_code = 0 if fmt == formats.NVFP4 else 1
        samples = []
        for n in (1, 2, 4, 8):
            def call(n=n):
                count.fill_(n)
                torch.ops.xtier.ep_stage(claim_list, claim, count, done, idx, stage['bases'], stage['stride'],
                                         stage['piece_off'], stage['piece_bytes'], *st, g13, g2, I, H, fmt_code,
                                         max(4, 148 * 8 // S))
            samples.append((n, _graph_time_us(call, reps)))
        ok = all(bool(torch.equal(st[0][i].cpu(), ew.w13[i])) for i in range(S))   # the last call staged every expert
        if not ok:
            raise RuntimeError('PCIe staging probe: the staged expert bytes differ from the engine\'s')
        return samples
    finally:
        torch.cuda.synchronize()
        unmap_engine(regs)
        eng.close()


def measure(H: int, I: int, fmt: str = formats.NVFP4, threads: int | None = None, gpu: bool = True) -> dict:
    cpu = probe_cpu(H, I, fmt, threads)
    c0, c1 = fit(cpu)
    out = {'samples': {'cpu': cpu}}
    co = Coeffs(c1=max(c1, 0.1))
    if gpu and torch.cuda.is_available():
        g = probe_gpu(H, I, fmt)
        g0, g1 = fit(g)
        co.g0, co.g1 = max(g0, 0.5), max(g1, 0.01)
        out['samples']['gpu'] = g
        mbx = probe_mailbox(H, fmt, threads)
        co.c0 = max(mbx['call_us'] - mbx['engine_us'], 1.0)
        out['samples']['mailbox'] = mbx
        peer = probe_peer(H, I, fmt)
        if peer is not None:
            co.p1 = peer['us']
            out['samples']['peer'] = peer
        pcie = probe_pcie(H, I, fmt)
        if pcie:
            co.h1 = max(fit(pcie)[1], 0.1)
            out['samples']['pcie'] = pcie
    else:   # no GPU to measure the round trip on: the engine's fixed cost plus a nominal 8 us for PCIe both ways
        co.c0 = max(c0, 1.0) + 8.0
        out['c0_measured'] = False
    out['coeffs'] = co.to_dict()
    out['shape'] = {'hidden': H, 'inter': I, 'fmt': fmt}
    return out
