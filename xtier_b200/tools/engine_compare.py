"""Same-host comparison of this framework's CPU expert engine with the reference's own C++ engine (benchmark config
1: hidden 2048, 64 NVFP4 experts of intermediate 768, softmax top-8 with renormalized weights, 8 threads).

Both engines receive the same expert bytes (the shared checkpoint layout), the same activations and routes, and are
driven through their C functions directly (no Python wrapper work inside the timed loop); each result is checked
against the fp32 dequantized reference. The reference's engine is built from its own sources and CMake (out of
source) and loaded from --ref-lib (the directory of its libxtier_engine.so).

    cmake -S <reference>/csrc -B <build> -DCMAKE_BUILD_TYPE=Release && cmake --build <build> --target xtier_engine
    python -m xtier_b200.tools.engine_compare --ref-lib <build> [--threads 8] [--tokens 1,2,4,8,16]
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import time

import torch


def _ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def _ref_lib(path: str):
    lib = C.CDLL(os.path.join(path, 'libxtier_engine.so'))
    P, I = C.c_void_p, C.c_int
    lib.xtier_create3.argtypes = [I, I, I, I, C.c_float, I] + [P] * 6
    lib.xtier_create3.restype = P
    lib.xtier_forward_decode.argtypes = [P, I, I] + [P] * 4
    lib.xtier_forward_decode.restype = I
    lib.xtier_forward.argtypes = [P, I, I] + [P] * 4
    lib.xtier_forward.restype = I
    lib.xtier_destroy.argtypes = [P]
    lib.xtier_last_error.restype = C.c_char_p
    lib.xtier_isa.restype = C.c_char_p
    return lib


def _time_us(fn, reps: int) -> float:
    for _ in range(10):
        fn()
    best = float('inf')
    for _ in range(3):   # best of three rounds (the host is shared)
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        best = min(best, (time.perf_counter() - t0) / reps * 1e6)
    return best


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument('--ref-lib', required=True, help="directory of the reference's libxtier_engine.so")
    ap.add_argument('--threads', type=int, default=8)
    ap.add_argument('--tokens', default='1,2,4,8,16')
    ap.add_argument('--reps', type=int, default=200)
    a = ap.parse_args(argv)
    from .. import formats
    from ..engine import CpuEngine, lib as our_lib
    H, I, E, k = 2048, 768, 64, 8
    g = torch.Generator().manual_seed(0)
    ex = formats.random_experts(E, H, I, formats.NVFP4, seed=0, std=0.02)
    gate = torch.randn(E, H, generator=g) * 0.02
    w13, w2, s13, s2 = (getattr(ex, f).contiguous() for f in ('w13', 'w2', 's13', 's2'))
    g13, g2 = ex.g13.float().contiguous(), ex.g2.float().contiguous()
    cases = []
    for m in [int(t) for t in a.tokens.split(',')]:
        x = torch.randn(m, H, generator=g).bfloat16().contiguous()
        p = torch.softmax(x.float() @ gate.t(), -1)
        w, ids = torch.topk(p, k, -1)
        w = (w / w.sum(-1, keepdim=True)).float().contiguous()
        cases.append((m, x, ids.int().contiguous(), w, formats.reference_moe(x, ids.int(), w, ex)))
    rel = lambda y, want: float((y - want).norm() / want.norm())
    # one engine alive at a time: the other's worker pool must not compete for the cores
    results = {}
    ours = CpuEngine(ex, threads=a.threads)
    lib = our_lib()
    try:
        for m, x, ids, w, want in cases:
            y = torch.zeros(m, H)
            args = (ours.plan, m, k, _ptr(x), _ptr(ids), _ptr(w), _ptr(y))
            results[m] = dict(ours_us=round(_time_us(lambda: lib.xt_engine_forward_decode(*args), a.reps), 1),
                              ours_rel_err=rel(y, want))
    finally:
        ours.close()
    ref = _ref_lib(a.ref_lib)
    plan = ref.xtier_create3(H, I, E, a.threads, 0.0, 0, _ptr(w13), _ptr(w2), _ptr(s13), _ptr(s2), _ptr(g13),
                             _ptr(g2))
    if not plan:
        raise SystemExit(f'reference engine: {ref.xtier_last_error().decode()}')
    try:
        for m, x, ids, w, want in cases:
            y = torch.zeros(m, H)
            args = (plan, m, k, _ptr(x), _ptr(ids), _ptr(w), _ptr(y))
            r = results[m]
            r['reference_us'] = round(_time_us(lambda: ref.xtier_forward_decode(*args), a.reps), 1)
            r['reference_rel_err'] = rel(y, want)
            print(json.dumps(dict(tool='engine_compare', tokens=m, threads=a.threads, ours_us=r['ours_us'],
                                  reference_us=r['reference_us'], ratio=round(r['reference_us'] / r['ours_us'], 3),
                                  ours_rel_err=float('%.3g' % r['ours_rel_err']),
                                  reference_rel_err=float('%.3g' % r['reference_rel_err']),
                                  reference_isa=ref.xtier_isa().decode())), flush=True)
    finally:
        ref.xtier_destroy(plan)


if __name__ == '__main__':
    main()
