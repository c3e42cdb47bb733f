"""Tensor parallelism with the collective fused into the GEMM (tcgen05 + NVLink peer memory), and the NCCL baselines.

Two ops (`torch.ops.xtier.gemm_rs`, `torch.ops.xtier.ag_gemm`, csrc/cuda/gemm_tp.cu):

* `TPComm.gemm_rs(a, b)`  -- a row-parallel linear followed by a reduce-scatter of its rows. Every rank holds a K
  shard of the activations `a [M, K/W]` and of the weight `b [N, K/W]`; rank r gets rows [r M/W, (r+1) M/W) of
  sum_ranks a b^T. The GEMM's epilogue stores each finished 128 x BN tile into its owner's receive slot over NVLink
  and releases a per-tile flag, so the transfer overlaps the next tiles' MMAs; the owner sums the W partials in rank
  order (FP32) and adds the residual.
* `TPComm.ag_gemm(a_shard, b)` -- an all-gather of the row-sharded activations followed by a column-parallel linear.
  A push kernel stores this rank's rows into every rank's gather buffer (128-row blocks, one flag each); the GEMM's
  TMA producer waits per block and reads only this rank's own memory. The walk starts with the local rows, so the MMAs
  begin before the peers' rows land.

Together they are the sequence-parallel MLP (`TPMLP`): AG-GEMM (gate/up, column shards) -> activation -> GEMM-RS
(down, row shards). The flags carry a per-call epoch kept in device memory and the data regions are double buffered by
call parity, so both ops replay from CUDA graphs with no host work. Every wait in the kernels is bounded; a timeout
sets the error word (`check()` raises).

`nccl_gemm_rs` / `nccl_ag_gemm` are the baselines: the same GEMM (cuBLAS) then `reduce_scatter_tensor`, or
`all_gather_into_tensor` then the GEMM.

(The reference has no tensor parallelism of its own: it runs inside SGLang's TP groups, xtier/backend/method.py:60-110.)
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from . import dist as xdist
from .symm import SymmetricBuffer

TILE_M = 128


class TPComm:
    """Symmetric buffer, epoch state and error word shared by every fused TP op of a process group.

    `max_elems`: the largest M x N (gemm_rs) or M x K (ag_gemm) of any call, in elements. Calls on one stream, in the
    same order on every rank."""

    def __init__(self, max_elems: int, max_rows: int, device=None, timeout_s: float = 10.0):
        env = xdist.get()
        self.W, self.rank = env.world, env.rank
        self.device = device or env.device
        self.max_elems = int(max_elems)
        self.max_rows = int(max_rows)
        # flags: RS needs W x (M/W/128) x ceil(N/128) <= M/128 x ceil(N/128) words; AG needs M/128
        data = (self.max_elems * 2 + 4095) // 4096 * 4096
        self.max_flags = max(self.max_elems // (TILE_M * 128) + self.max_rows // TILE_M + 64, 1024)
        flags = (self.max_flags * 4 + 4095) // 4096 * 4096
        self.offsets = [0, data, 2 * data, 2 * data + flags]
        self.buf = SymmetricBuffer(2 * data + 2 * flags, self.device)
        self.local_base = self.buf.ptrs[self.rank]
        self.state = torch.zeros(4, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_s = timeout_s

    def _check_shape(self, M, cols):
        if M % (TILE_M * self.W):
            raise ValueError(f'fused TP ops need M % {TILE_M * self.W} == 0, got M={M}')
        if M * cols > self.max_elems or M > self.max_rows:
            raise ValueError(f'TPComm sized for {self.max_elems} elements / {self.max_rows} rows; got {M} x {cols}')

    def gemm_rs(self, a: torch.Tensor, b: torch.Tensor, residual: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """Rows [r M/W, (r+1) M/W) of sum_ranks a b^T (+ residual). a [M, Kr], b [N, Kr] BF16, contiguous."""
        M, N = a.shape[0], b.shape[0]
        self._check_shape(M, N)
        tiles = (M // TILE_M) * ((N + 127) // 128)
        if tiles > self.max_flags:
            raise ValueError('TPComm: too many output tiles for the flag region')
        out = torch.empty(M // self.W, N, dtype=a.dtype, device=a.device) if out is None else out
        ops.load()
        torch.ops.xtier.gemm_rs(a, b, self.buf.peer_table, self.state, residual, out, self.err, self.W, self.rank,
                                self.offsets, self.timeout_s)
        return out

    def ag_gemm(self, a_shard: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """all_gather(a_shard) b^T. a_shard [M/W, K] (this rank's rows), b [N, K] BF16, contiguous -> [M, N]."""
        M, N, K = a_shard.shape[0] * self.W, b.shape[0], a_shard.shape[1]
        self._check_shape(M, K)
        out = torch.empty(M, N, dtype=a_shard.dtype, device=a_shard.device) if out is None else out
        ops.load()
        torch.ops.xtier.ag_gemm(a_shard, b, self.buf.peer_table, self.local_base, self.state, out, self.err, self.W,
                                self.rank, self.offsets, self.timeout_s)
        return out

    def check(self):
        if int(self.err.item()):
            self.err.zero_()
            raise RuntimeError('xtier_b200 TP: a wait for a peer rank timed out')

    def close(self):
        self.buf.close()


def nccl_gemm_rs(a, b, residual=None, group=None):
    """Baseline: cuBLAS GEMM of the K shard, then NCCL reduce_scatter_tensor of the rows (+ residual)."""
    W = dist.get_world_size(group)
    part = torch.matmul(a, b.t())
    out = torch.empty(a.shape[0] // W, b.shape[0], dtype=a.dtype, device=a.device)
    dist.reduce_scatter_tensor(out, part, group=group)
    return out if residual is None else out + residual


def nccl_ag_gemm(a_shard, b, group=None):
    """Baseline: NCCL all_gather_into_tensor of the row shards, then the cuBLAS GEMM."""
    W = dist.get_world_size(group)
    full = torch.empty(a_shard.shape[0] * W, a_shard.shape[1], dtype=a_shard.dtype, device=a_shard.device)
    dist.all_gather_into_tensor(full, a_shard, group=group)
    return torch.matmul(full, b.t())


class TPMLP:
    """Sequence-parallel SwiGLU MLP over W ranks: x [M/W, H] (this rank's rows) -> [M/W, H].

    w13 [2 I/W, H]: this rank's column shard of gate and up (gate rows first); w2 [H, I/W]: its row shard of down.
    AG-GEMM (gate/up) -> SiLU(gate) * up -> GEMM-RS (down) + residual."""

    def __init__(self, comm: TPComm, w13: torch.Tensor, w2: torch.Tensor):
        self.comm, self.w13, self.w2 = comm, w13.contiguous(), w2.contiguous()
        self.Il = w2.shape[1]

    def __call__(self, x_shard: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        gu = self.comm.ag_gemm(x_shard, self.w13)
        h = (torch.nn.functional.silu(gu[:, :self.Il].float()) * gu[:, self.Il:].float()).to(x_shard.dtype)
        return self.comm.gemm_rs(h, self.w2, residual=residual)
