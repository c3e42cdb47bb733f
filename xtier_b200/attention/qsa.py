"""Sparse GQA attention over an NVFP4 KV cache: the attention of the Qwen4-exp QSA layers and of MiniMax's sparse
decode -- few KV heads (2-8), head dim up to 256, each decode query attending only to the cache slots its indexer
selected (top-k), keys and values kept as NVFP4 (E2M1 codes, one E4M3 scale per 16 values).

`KvCacheFP4(rows, max_len, kv_heads, head_dim)` holds K and V of `rows` sequences; `write(k, v, slots)` quantizes new
rows into it (csrc/cuda/qsa.cu `qsa_kv_write`), `dequant(slots)` returns the FP32 values the kernels compute with.
`qsa_decode(q, idx, cache, scale)` is the attention: q [B, Hq, D] BF16, idx [B, nsel] int32 cache slots (-1 = none),
-> [B, Hq, D] BF16. The G = Hq / Hkv query heads of a KV head share one CTA per 32 selected keys, which stages their
NVFP4 rows in shared memory and dequantizes each key and value once in registers for all of them; the splits meet in a
log-sum-exp merge. The selection comes from an indexer: the DSA lightning indexer of attention/dsa.py (FP8 index
keys, ReLU head-sum scores, length-aware radix top-k) has the same form as QSA's.

Reference parity: xtier/packs/qwen4_exp/qsa_fp4.py:82-147 (top-k KV rows gathered from an NVFP4 pool and dequantized
in registers), qsa_decode.py:26-64 (split-key decode with a merge, 24 query / 2 KV heads of dim 256),
xtier/packs/minimax_m3/kv_fp4.py:53-149 (sparse decode over an NVFP4 KV cache). The kernels, cache layout and split
size here are this project's own.
"""
from __future__ import annotations

import torch

from .. import formats, ops

KEYS_PER_SPLIT = 32


class KvCacheFP4:
    """slots = rows * max_len token slots; slot of (row, pos) = row * max_len + pos."""

    def __init__(self, rows: int, max_len: int, kv_heads: int, head_dim: int, device='cuda'):
        if head_dim % 32 or not 32 <= head_dim <= 256:
            raise ValueError('head_dim must be a multiple of 32 in [32, 256]')
        n = rows * max_len
        self.rows, self.max_len, self.H, self.D = rows, max_len, kv_heads, head_dim
        u8 = lambda d: torch.zeros(n, kv_heads, d, dtype=torch.uint8, device=device)   # noqa: E731
        self.kc, self.ks = u8(head_dim // 2), u8(head_dim // 16)
        self.vc, self.vs = u8(head_dim // 2), u8(head_dim // 16)

    def slots(self, rows: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        return rows.long() * self.max_len + pos.long()

    def write(self, k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor):
        """k, v [T, Hkv, D] BF16 into the given slots (int64 [T])."""
        ops.load()
        s = slots.long().contiguous()
        torch.ops.xtier.qsa_kv_write(k.contiguous(), s, self.kc, self.ks)
        torch.ops.xtier.qsa_kv_write(v.contiguous(), s, self.vc, self.vs)

    def dequant(self, slots: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 K and V [n, Hkv, D] of the given slots (the values the kernels compute with)."""
        s = slots.long()
        k = formats.dequant(self.kc[s], self.ks[s], formats.NVFP4)
        v = formats.dequant(self.vc[s], self.vs[s], formats.NVFP4)
        return k, v


class QsaWorkspace:
    """Split partials of up to `batch` queries of `heads` query heads, head dim D, over up to `nsel` keys."""

    def __init__(self, batch: int, heads: int, head_dim: int, nsel: int, device='cuda'):
        splits = (nsel + KEYS_PER_SPLIT - 1) // KEYS_PER_SPLIT
        self.part_o = torch.empty(batch * heads * splits * head_dim, dtype=torch.float32, device=device)
        self.part_ml = torch.empty(batch * heads * splits * 2, dtype=torch.float32, device=device)


def qsa_decode(q: torch.Tensor, idx: torch.Tensor, cache: KvCacheFP4, scale: float,
               ws: QsaWorkspace | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(scale * q.k) . v over the selected slots of each query; q [B, Hq, D] BF16, idx [B, nsel] int32."""
    ops.load()
    B, Hq, D = q.shape
    ws = ws or QsaWorkspace(B, Hq, D, idx.shape[1], q.device)
    out = torch.empty_like(q) if out is None else out
    torch.ops.xtier.qsa_decode(q.contiguous(), idx.int().contiguous(), cache.kc, cache.ks, cache.vc, cache.vs,
                               ws.part_o, ws.part_ml, out, float(scale))
    return out


def reference(q: torch.Tensor, idx: torch.Tensor, cache: KvCacheFP4, scale: float) -> torch.Tensor:
    """The same attention in FP32 PyTorch over the dequantized cache (tests)."""
    B, Hq, D = q.shape
    G = Hq // cache.H
    out = torch.zeros(B, Hq, D, dtype=torch.float32, device=q.device)
    for b in range(B):
        sel = idx[b][idx[b] >= 0]
        if sel.numel() == 0:
            continue
        k, v = cache.dequant(sel)                                   # [n, Hkv, D]
        k = k.repeat_interleave(G, dim=1).transpose(0, 1)           # [Hq, n, D]
        v = v.repeat_interleave(G, dim=1).transpose(0, 1)
        p = torch.softmax(torch.einsum('hd,hnd->hn', q[b].float(), k) * scale, -1)
        out[b] = torch.einsum('hn,hnd->hd', p, v)
    return out
