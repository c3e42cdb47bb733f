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

from .. import config, ops
from ..formats import NVFP4, ExpertWeights

TILE = 128


def plan(slots: torch.Tensor):
    """slots [m, k] int32 (-1: not on the GPU) -> (order: route ids sorted by slot, rows: destination row of each
    sorted route in X, R: padded row count, runs: CPU int64 [n, 3] of (slot, first row, count)). One device->host
    copy (the per-slot counts)."""
    flat = slots.flatten().long()
    gpu = torch.nonzero(flat >= 0).flatten()
    if gpu.numel() == 0:
        return gpu, gpu, 0, torch.zeros(0, 3, dtype=torch.long)
    key = flat[gpu]
    perm = torch.sort(key, stable=True).indices
    order = gpu[perm]
    uniq, counts = torch.unique_consecutive(key[perm], return_counts=True)
    padded = (counts + TILE - 1) // TILE * TILE
    starts = torch.cumsum(padded, 0) - padded                      # first row of each run in X
    run_of = torch.repeat_interleave(torch.arange(counts.numel(), device=slots.device), counts)
    first = torch.cumsum(counts, 0) - counts                         # first sorted route of each run
    rows = starts[run_of] + (torch.arange(order.numel(), device=slots.device) - first[run_of])
    runs = torch.stack([uniq, starts, counts], 1).cpu()
    R = int(runs[-1, 1] + (runs[-1, 2] + TILE - 1) // TILE * TILE)
    return order, rows, R, runs


WORK_ROWS = 2 * TILE   # rows of one work item of the kernel: two 128-row m-tiles share each dequantized weight tile


def _tiles(runs: torch.Tensor, n_tiles: int, device, work_rows: int = WORK_ROWS) -> torch.Tensor:
    """[T, 4] int32 (slot, first row, n-tile, valid rows <= work_rows) for every work_rows-row block of every run x
    every n-tile (rows past a run's end in its last block are computed and dropped by the kernel's epilogue)."""
    WORK_ROWS = work_rows
    mt = (runs[:, 2] + WORK_ROWS - 1) // WORK_ROWS
    run = torch.repeat_interleave(torch.arange(runs.shape[0]), mt)
    first_block = torch.cumsum(mt, 0) - mt
    blk = torch.arange(run.numel()) - first_block[run]
    row0 = runs[run, 1] + blk * WORK_ROWS
    valid = torch.clamp(runs[run, 2] - blk * WORK_ROWS, max=WORK_ROWS)
    slot = runs[run, 0]
    T = run.numel()
    t = torch.stack([slot.repeat_interleave(n_tiles), row0.repeat_interleave(n_tiles),
                     torch.arange(n_tiles).repeat(T), valid.repeat_interleave(n_tiles)], 1)
    return t.to(torch.int32).to(device, non_blocking=True)


def _grouped_routes_mx(x, src, w, pool, order, rows, R, runs, m, k, err, route_rows, out):
    """grouped_routes with MXFP8 activations and the block-scaled MXFP4 kernel (csrc/cuda/moe_prefill_mx.cu): the
    gathered token rows and the SwiGLU output are quantized to E4M3 with UE8M0 scales per 32 values."""
    H, I = pool.hidden, pool.inter
    dev = x.device
    X8 = torch.empty(R, H, dtype=torch.uint8, device=dev)
    SFX = torch.empty(R * H // 32, dtype=torch.uint8, device=dev)
    torch.ops.xtier.mx_quant_rows(x.contiguous(), src, X8, SFX)
    rw = torch.zeros(R, dtype=torch.float32, device=dev)
    rw[rows] = w.flatten().float()[order]
    err = torch.zeros(1, dtype=torch.int32, device=dev) if err is None else err
    mid = torch.empty(R, I, dtype=torch.bfloat16, device=dev)
    torch.ops.xtier.moe_grouped_mx(X8, SFX, pool.w13, pool.s13, pool.g13.float().contiguous(),
                                   _tiles(runs, I // 64, dev, TILE), True, I, None, mid, err)
    del X8, SFX
    M8 = torch.empty(R, I, dtype=torch.uint8, device=dev)
    SFM = torch.empty(R * I // 32, dtype=torch.uint8, device=dev)
    torch.ops.xtier.mx_quant_rows(mid, None, M8, SFM)
    del mid
    dest = torch.full((m * k,), -1, dtype=torch.int32, device=dev)
    if route_rows:
        Y = torch.empty(m * k, H, dtype=torch.float32, device=dev) if out is None else out
        dst = torch.full((R,), -1, dtype=torch.int32, device=dev)
        dst[rows] = order.int()
        dest[order] = order.int()
    else:
        Y = torch.empty(R, H, dtype=torch.float32, device=dev)
        dst = None
        dest[order] = rows.int()
    torch.ops.xtier.moe_grouped_mx(M8, SFM, pool.w2, pool.s2, pool.g2.float().contiguous(),
                                   _tiles(runs, H // 128, dev, TILE), False, I, rw, Y, err, dst)
    return Y, dest


def grouped_routes(x: torch.Tensor, slots: torch.Tensor, w: torch.Tensor, pool: ExpertWeights,
                   err: torch.Tensor | None = None, route_rows: bool = False, out: torch.Tensor | None = None,
                   mx: bool | None = None):
    """x [m, H] BF16, slots [m, k] GPU slot per route (-1 skips), w [m, k] route weights -> (Y [R, H] FP32: every
    computed route's w * MoE_expert(x) row, dest [m * k] int32: the Y row of each route or -1); (None, None) when no
    route has a slot. Token rows are gathered into the padded per-expert runs by a kernel (csrc/cuda/moe_prefill.cu
    gather_rows); the down GEMM's epilogue applies the route weight. route_rows=True: Y [m * k, H] indexed by route
    (t * k + j), written there directly by the down GEMM's epilogue (into `out` when given). mx (default
    XTIER_PREFILL_MX): MXFP4 pools run with MXFP8 activations on the block-scaled kernel (the reference's prefill
    numerics) instead of the exact W4A16 one."""
    m, k = slots.shape
    H, I = pool.hidden, pool.inter
    dev = x.device
    order, rows, R, runs = plan(slots)
    if runs.shape[0] == 0:
        return None, None
    if H % 128 or I % 64:
        raise ValueError('grouped prefill needs H % 128 == 0 and I % 64 == 0')
    ops.load()
    src = torch.full((R,), -1, dtype=torch.int32, device=dev)
    src[rows] = (order // k).int()
    if mx is None:
        mx = bool(config.get('XTIER_PREFILL_MX'))
    if mx and pool.fmt != NVFP4 and H % 128 == 0 and I % 128 == 0:
        return _grouped_routes_mx(x, src, w, pool, order, rows, R, runs, m, k, err, route_rows, out)
    X = torch.empty(R, H, dtype=torch.bfloat16, device=dev)
    torch.ops.xtier.gather_rows(x.contiguous(), src, X)
    rw = torch.zeros(R, dtype=torch.float32, device=dev)
    rw[rows] = w.flatten().float()[order]
    err = torch.zeros(1, dtype=torch.int32, device=dev) if err is None else err
    fmt = 0 if pool.fmt == NVFP4 else 1
    mid = torch.empty(R, I, dtype=torch.bfloat16, device=dev)
    torch.ops.xtier.moe_grouped(X, pool.w13, pool.s13, pool.g13.float().contiguous(), _tiles(runs, I // 64, dev), True,
                                I, fmt, None, mid, err)
    dest = torch.full((m * k,), -1, dtype=torch.int32, device=dev)
    if route_rows:
        Y = torch.empty(m * k, H, dtype=torch.float32, device=dev) if out is None else out
        dst = torch.full((R,), -1, dtype=torch.int32, device=dev)
        dst[rows] = order.int()
        dest[order] = order.int()
    else:
        Y = torch.empty(R, H, dtype=torch.float32, device=dev)
        dst = None
        dest[order] = rows.int()
    torch.ops.xtier.moe_grouped(mid, pool.w2, pool.s2, pool.g2.float().contiguous(), _tiles(runs, H // 128, dev),
                                False, I, fmt, rw, Y, err, dst)
    return Y, dest


def combine(parts, out: torch.Tensor, add: torch.Tensor | None = None) -> torch.Tensor:
    """out [m, H] (BF16 or FP32) = per token, the sum of its routes' rows in route order over the (Y, dest) parts
    (a route appears in at most one part) + add; one kernel pass."""
    parts = [p for p in parts if p[0] is not None]
    if not parts:
        if add is None:
            out.zero_()
        else:
            out.copy_(add)
        return out
    (Ya, da), (Yb, db) = parts[0], (parts[1] if len(parts) > 1 else (None, None))
    torch.ops.xtier.route_combine(Ya, da, Yb, db, add, out)
    return out


def grouped_experts(x: torch.Tensor, slots: torch.Tensor, w: torch.Tensor, pool: ExpertWeights,
                    err: torch.Tensor | None = None) -> torch.Tensor:
    """x [m, H] BF16, slots [m, k] GPU slot per route (-1 skips), w [m, k] route weights -> FP32 [m, H]: the sum over
    each token's GPU routes of w * MoE_expert(x), in route order."""
    out = torch.empty(slots.shape[0], pool.hidden, dtype=torch.float32, device=x.device)
    return combine([grouped_routes(x, slots, w, pool, err)], out)
