"""Prefill of the GPU-resident experts with the grouped FP4 tensor-core GEMM (csrc/cuda/moe_prefill.cu).

Routes whose expert has a GPU slot are sorted by slot (stable, so each slot's tokens keep their order), their token
rows gathered into X [R, H] with every slot's run padded to 128 rows, and two grouped GEMMs run over per-slot tile
lists: gate/up with the SwiGLU in the epilogue (mid [R, I] BF16), then down with the route weight and g2 applied
(Y [R, H] FP32). Each token's GPU part is the sum of its routes' Y rows in route order (deterministic; no atomics).
The expert weights are read once per 128 routed tokens instead of once per route, which is what makes prefill-sized
calls compute-bound instead of weight-bound.
(Reference parity: xtier/backend/prefill.py:64-140 grouped gate/up and down over sorted route tiles, :1511 the
FlashInfer CUTLASS fused MoE it calls on SM100.)
"""
from __future__ import annotations

import torch

from .. import ops
from ..formats import NVFP4, ExpertWeights

TILE = 128


def plan(slots: torch.Tensor):
    """slots [m, k] int32 (-1: not on the GPU) -> (order: route ids sorted by slot, rows: destination row of each
    sorted route in X, R: padded row count, runs: list of (slot, first row, count))."""
    flat = slots.flatten().long()
    gpu = torch.nonzero(flat >= 0).flatten()
    if gpu.numel() == 0:
        return gpu, gpu, 0, []
    key = flat[gpu]
    perm = torch.sort(key, stable=True).indices
    order = gpu[perm]
    sorted_slots = key[perm]
    uniq, counts = torch.unique_consecutive(sorted_slots, return_counts=True)
    uniq, counts = uniq.tolist(), counts.tolist()
    runs, rows, r0 = [], [], 0
    for s, c in zip(uniq, counts):
        runs.append((s, r0, c))
        rows.append(torch.arange(r0, r0 + c))
        r0 += (c + TILE - 1) // TILE * TILE
    return order, torch.cat(rows).to(slots.device), r0, runs


def _tiles(runs, n_tiles: int, device) -> torch.Tensor:
    t = []
    for s, r0, c in runs:
        for mt in range(0, c, TILE):
            for nt in range(n_tiles):
                t.append((s, r0 + mt, nt, min(TILE, c - mt)))
    return torch.tensor(t, dtype=torch.int32, device=device).reshape(-1, 4)


def grouped_experts(x: torch.Tensor, slots: torch.Tensor, w: torch.Tensor, pool: ExpertWeights,
                    err: torch.Tensor | None = None) -> torch.Tensor:
    """x [m, H] BF16, slots [m, k] GPU slot per route (-1 skips), w [m, k] route weights -> FP32 [m, H]: the sum over
    each token's GPU routes of w * MoE_expert(x), in route order."""
    m, k = slots.shape
    H, I = pool.hidden, pool.inter
    dev = x.device
    out = torch.zeros(m, H, dtype=torch.float32, device=dev)
    order, rows, R, runs = plan(slots)
    if not runs:
        return out
    if H % 128 or I % 64:
        raise ValueError('grouped prefill needs H % 128 == 0 and I % 64 == 0')
    tok = order // k
    X = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
    X[rows] = x[tok]
    rw = torch.zeros(R, dtype=torch.float32, device=dev)
    rw[rows] = w.flatten().float()[order]
    err = torch.zeros(1, dtype=torch.int32, device=dev) if err is None else err
    fmt = 0 if pool.fmt == NVFP4 else 1
    ops.load()
    mid = torch.empty(R, I, dtype=torch.bfloat16, device=dev)
    torch.ops.xtier.moe_grouped(X, pool.w13, pool.s13, pool.g13.float().contiguous(), _tiles(runs, I // 64, dev), True,
                                I, fmt, None, mid, err)
    Y = torch.empty(R, H, dtype=torch.float32, device=dev)
    torch.ops.xtier.moe_grouped(mid, pool.w2, pool.s2, pool.g2.float().contiguous(), _tiles(runs, H // 128, dev),
                                False, I, fmt, rw, Y, err)
    # route-ordered sum per token: Y row of route (t, j) or zero
    dest = torch.full((m * k,), -1, dtype=torch.long, device=dev)
    dest[order] = rows.long()
    per_route = torch.where(dest[:, None] >= 0, Y[dest.clamp_min(0)], torch.zeros((), device=dev)).view(m, k, H)
    for j in range(k):
        out += per_route[:, j]
    return out
