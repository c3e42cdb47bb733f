"""DSA-style sparse attention selection: the lightning indexer over an FP8 key cache and a top-k per query.

Per cached token the indexer keeps one 128-dim key (FP8 E4M3, one FP32 scale per token: 132 bytes). A query t with 64
indexer heads q[t, h] and head weights w[t, h] scores every cached key s of its sequence as
I(t, s) = sum_h w[t, h] * relu(q[t, h] . k[s]); attention then runs over the top `k` (2048 in the DeepSeek shape)
keys only (`xtier_b200.attention.mla.mla_decode` takes the resulting slot lists). Kernels: csrc/cuda/dsa.cu.
`reference_scores` / `reference_topk` are the fp32 PyTorch oracles.
(Reference parity: xtier/packs/deepseek_v4/paged_indexer.py:1-13, xtier/packs/qwen4_exp/qsa_prefill.py:1-12.)
"""
from __future__ import annotations

import torch

from .. import ops

HEADS, DIM = 64, 128


class IndexCache:
    """slots = rows * max_len; slot of (row, pos) = row * max_len + pos."""

    def __init__(self, rows: int, max_len: int, device='cuda'):
        self.rows, self.max_len = rows, max_len
        self.codes = torch.zeros(rows * max_len, DIM, dtype=torch.uint8, device=device)
        self.scale = torch.ones(rows * max_len, dtype=torch.float32, device=device)

    def write(self, k: torch.Tensor, slots: torch.Tensor):
        ops.load()
        torch.ops.xtier.dsa_key_write(k.contiguous(), slots.long().contiguous(), self.codes, self.scale)

    def dequant(self, slots: torch.Tensor) -> torch.Tensor:
        s = slots.long()
        return self.codes[s].view(torch.float8_e4m3fn).float() * self.scale[s, None]


def quantize_queries(q: torch.Tensor, w: torch.Tensor):
    """q [Q, 64, 128] -> FP8 E4M3 bytes with one scale per (query, head), folded into the head weights (relu commutes
    with a positive scale): returns (q8 uint8 [Q, 64, 128], w' fp32 [Q, 64])."""
    qf = q.float()
    s = (qf.abs().amax(-1) / 448.0).clamp_min(1e-12)
    q8 = (qf / s[..., None]).to(torch.float8_e4m3fn).view(torch.uint8)
    return q8.contiguous(), (w.float() * s).contiguous()


def index_scores(q: torch.Tensor, w: torch.Tensor, cache: IndexCache, rows: torch.Tensor, lengths: torch.Tensor,
                 out: torch.Tensor | None = None, tensor_cores: bool = True, err: torch.Tensor | None = None,
                 per_cta: int = 1) -> torch.Tensor:
    """q [Q, 64, 128] BF16, w [Q, 64] fp32, rows / lengths [Q] (each query's cache row and key count) -> scores
    [Q, max_len] fp32 (-inf past the length). The tensor-core path quantizes the queries to FP8 (E4M3 x E4M3 MMA);
    per_cta = 2 lets two consecutive queries of one cache row share each key tile (prefill)."""
    Q = q.shape[0]
    out = torch.empty(Q, cache.max_len, dtype=torch.float32, device=q.device) if out is None else out
    base = rows.long() * cache.max_len
    ops.load()
    if tensor_cores:
        q8, w8 = quantize_queries(q, w)
        err = torch.zeros(1, dtype=torch.int32, device=q.device) if err is None else err
        torch.ops.xtier.dsa_index_tc(q8, w8, cache.codes, cache.scale, base, lengths.int().contiguous(), out,
                                     per_cta, err)
    else:
        torch.ops.xtier.dsa_index_decode(q.contiguous(), w.float().contiguous(), cache.codes, cache.scale, base,
                                         lengths.int().contiguous(), out)
    return out


def index_scores_prefill(q: torch.Tensor, w: torch.Tensor, cache: IndexCache, row: int, lengths: torch.Tensor,
                         out: torch.Tensor | None = None, err: torch.Tensor | None = None,
                         splits: int = 0, w_scale: float = 1.0) -> torch.Tensor:
    """Indexer scores of queries that share cache row `row` (a prefill chunk of one sequence): q [Q, 64, 128] BF16,
    head weights w_scale * w [Q, 64] (BF16: quantized with the queries by one kernel, or fp32), lengths [Q] -> scores
    [Q, max_len] fp32, valid in [0, lengths[i]) of row i (then -inf up to the end of the last 128-key tile, unwritten
    beyond: pass the same lengths to topk). FP8 queries (E4M3 x E4M3 MMA), 4 queries per CTA over a pipelined key
    stream; `splits` key ranges per query group (0: chosen by the launcher)."""
    Q = q.shape[0]
    out = torch.empty(Q, cache.max_len, dtype=torch.float32, device=q.device) if out is None else out
    ops.load()
    if w.dtype == torch.bfloat16 and q.is_contiguous():   # one kernel: FP8 queries, scales into the head weights
        q8 = torch.empty(q.shape, dtype=torch.uint8, device=q.device)
        w8 = torch.empty(w.shape, dtype=torch.float32, device=q.device)
        torch.ops.xtier.dsa_quant_q(q, w.contiguous(), float(w_scale), q8, w8)
    else:
        q8, w8 = quantize_queries(q, w.float() * w_scale)
    err = torch.zeros(1, dtype=torch.int32, device=q.device) if err is None else err
    torch.ops.xtier.dsa_index_pf(q8, w8, cache.codes, cache.scale, int(row) * cache.max_len,
                                 lengths.int().contiguous(), out, int(splits), err)
    return out


def topk(scores: torch.Tensor, k: int, out: torch.Tensor | None = None,
         lengths: torch.Tensor | None = None) -> torch.Tensor:
    """Indices of the k largest finite scores per row, ascending; -1 padding. int32 [rows, k]. With lengths, row i
    is read only in [0, lengths[i])."""
    out = torch.empty(scores.shape[0], k, dtype=torch.int32, device=scores.device) if out is None else out
    ops.load()
    torch.ops.xtier.topk_rows(scores.contiguous(), k, out,
                              None if lengths is None else lengths.to(torch.int32).contiguous())
    return out


def select_slots(scores: torch.Tensor, rows: torch.Tensor, k: int, max_len: int) -> torch.Tensor:
    """Top-k positions of each query turned into cache slots of its row (-1 stays -1)."""
    pos = topk(scores, k)
    return torch.where(pos >= 0, pos + (rows.long() * max_len)[:, None].int(), pos)


def reference_scores(q, w, cache: IndexCache, rows, lengths, fp8_queries: bool = False) -> torch.Tensor:
    """fp32 oracle; fp8_queries=True scores the FP8-rounded queries the tensor-core path uses."""
    Q = q.shape[0]
    if fp8_queries:
        q8, w = quantize_queries(q, w)
        q = q8.view(torch.float8_e4m3fn).float()
    out = torch.full((Q, cache.max_len), float('-inf'), device=q.device)
    for i in range(Q):
        n = int(lengths[i])
        slots = int(rows[i]) * cache.max_len + torch.arange(n, device=q.device)
        k = cache.dequant(slots)                                       # [n, 128]
        s = torch.relu(q[i].float() @ k.t())                           # [64, n]
        out[i, :n] = (w[i].float()[:, None] * s).sum(0)
    return out


def reference_topk(scores: torch.Tensor, k: int) -> list[set]:
    res = []
    for row in scores:
        fin = torch.isfinite(row)
        n = int(fin.sum())
        idx = torch.topk(row, min(k, n)).indices if n else torch.empty(0, dtype=torch.long)
        res.append(set(idx.tolist()))
    return res
