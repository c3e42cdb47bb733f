"""MLA attention over an NVFP4 latent KV cache (DeepSeek-V3-shaped models), decode side.

`LatentCache` holds, per layer, every cached token's 512 latent values as NVFP4 (E2M1 codes + an E4M3 scale per 16
values, global scale 1) and its 64 rotary key values in BF16: 416 bytes per token instead of 1152 for BF16.
`mla_decode` attends each query's 128 heads over a list of cache slots -- the DSA indexer's top-k for sparse
attention, or every slot of the sequence for dense attention -- on the tensor cores (csrc/cuda/mla_sparse.cu):
gather + dequantize the selected rows, S = Q.K^T into TMEM, one softmax pass per 128-key block in BF16, O = P.V into
TMEM, and a merge of the blocks. Queries arrive in the absorbed form (the nope part already multiplied by W_uk, so the
query lives in the 512-dim latent space, followed by its 64 rotary dims); the caller applies W_uv to the latent
output.

`reference_decode` is the fp32 PyTorch oracle of the same computation on the dequantized cache.
(Reference parity: xtier/packs/deepseek_v4/sparse_mla.py:1-20 -- sparse MLA over a quantized KV cache.)
"""
from __future__ import annotations

import math

import torch

from .. import formats, ops

LATENT, ROPE, BLOCK = 512, 64, 128


class LatentCache:
    """slots = rows * max_len token slots; slot of (row, pos) = row * max_len + pos."""

    def __init__(self, rows: int, max_len: int, device='cuda'):
        n = rows * max_len
        self.rows, self.max_len = rows, max_len
        self.codes = torch.zeros(n, LATENT // 2, dtype=torch.uint8, device=device)
        self.scales = torch.zeros(n, LATENT // 16, dtype=torch.uint8, device=device)
        self.rope = torch.zeros(n, ROPE, dtype=torch.bfloat16, device=device)

    def slots(self, rows: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        return rows.long() * self.max_len + pos.long()

    def write(self, lat: torch.Tensor, slots: torch.Tensor):
        """lat [T, 576] BF16 (latent then rotary) into the given slots."""
        ops.load()
        torch.ops.xtier.mla_kv_write(lat.contiguous(), slots.long().contiguous(), self.codes, self.scales, self.rope)

    def dequant(self, slots: torch.Tensor) -> torch.Tensor:
        """fp32 [n, 576] rows of the given slots (the values the kernels compute with)."""
        s = slots.long()
        lat = formats.dequant(self.codes[s], self.scales[s], formats.NVFP4)
        return torch.cat([lat, self.rope[s].float()], -1)


class MlaWorkspace:
    """Scratch of mla_decode for up to `queries` queries of `nsel` selected slots (nsel % 128 == 0)."""

    def __init__(self, queries: int, nsel: int, device='cuda'):
        if nsel % BLOCK:
            raise ValueError(f'nsel must be a multiple of {BLOCK}')
        self.Q, self.nsel = queries, nsel
        self.kg = torch.empty(queries * nsel * (LATENT + ROPE), dtype=torch.bfloat16, device=device)
        self.vt = torch.empty(queries * LATENT * nsel, dtype=torch.bfloat16, device=device)
        blocks = nsel // BLOCK
        self.part_o = torch.empty(queries * blocks * 128 * LATENT, dtype=torch.float32, device=device)
        self.part_ml = torch.empty(queries * blocks * 128 * 2, dtype=torch.float32, device=device)
        self.err = torch.zeros(1, dtype=torch.int32, device=device)


def mla_decode(q: torch.Tensor, idx: torch.Tensor, cache: LatentCache, ws: MlaWorkspace, scale: float,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """q [Q, 128, 576] BF16 (absorbed), idx [Q, nsel] int32 cache slots (-1: none) -> latent output [Q, 128, 512]."""
    Q, nsel = idx.shape
    if Q > ws.Q or nsel != ws.nsel:
        raise ValueError('workspace too small for this call')
    out = torch.empty(Q, 128, LATENT, dtype=torch.bfloat16, device=q.device) if out is None else out
    ops.load()
    torch.ops.xtier.mla_decode(q.contiguous(), idx.to(torch.int32).contiguous(), cache.codes, cache.scales,
                               cache.rope, ws.kg, ws.vt, ws.part_o, ws.part_ml, out, float(scale), ws.err)
    return out


class FlashWorkspace:
    """Split partials of mla_flash for up to `queries` queries and `splits` key splits (none needed at one split)."""

    def __init__(self, queries: int, splits: int, device='cuda'):
        self.Q, self.splits = queries, splits
        n = queries * splits * 128 if splits > 1 else 0
        self.part_o = torch.empty(n * LATENT, dtype=torch.float32, device=device) if n else None
        self.part_ml = torch.empty(n * 2, dtype=torch.float32, device=device) if n else None
        self.err = torch.zeros(1, dtype=torch.int32, device=device)


FLASH_BLOCK = 64


def flash_splits(queries: int, nsel: int, sms: int = 148) -> int:
    """Key splits of mla_flash: enough CTAs (2 value halves x splits x queries) to cover the SMs, at least four 64-key
    blocks per split."""
    nblk = max(1, nsel // FLASH_BLOCK)
    want = max(1, -(-sms // (2 * queries)))
    return max(1, min(want, nblk // 4 if nblk >= 8 else 1))


def mla_flash(q: torch.Tensor, idx: torch.Tensor, cache: LatentCache, scale: float, splits: int = 1,
              ws: FlashWorkspace | None = None, out: torch.Tensor | None = None,
              q_rope: torch.Tensor | None = None) -> torch.Tensor:
    """mla_decode in one pass (csrc/cuda/mla_sparse.cu mla_flash): q [Q, 128, 576] BF16 (absorbed), idx [Q, nsel]
    int32 cache slots (-1: none; nsel % 64 == 0) -> latent output [Q, 128, 512]. With q_rope, q is the latent part
    [Q, 128, 512] and q_rope the rotary part [Q, 128, 64]; q, q_rope and out may be strided views with unit stride
    along the last dim (e.g. head-major buffers seen through transpose(0, 1)). splits > 1 splits every query's keys
    over that many CTAs (short query batches) and merges their partials from `ws` (out contiguous then)."""
    Q = q.shape[0]
    out = torch.empty(Q, 128, LATENT, dtype=torch.bfloat16, device=q.device) if out is None else out
    if ws is None:
        ws = FlashWorkspace(Q, splits, q.device)
    ops.load()
    if q.stride(-1) != 1:
        q = q.contiguous()
    torch.ops.xtier.mla_flash(q, idx.to(torch.int32).contiguous(), cache.codes, cache.scales,
                              cache.rope, ws.part_o, ws.part_ml, out, float(scale), int(splits), ws.err, q_rope)
    return out


def reference_decode(q: torch.Tensor, idx: torch.Tensor, cache: LatentCache, scale: float) -> torch.Tensor:
    """fp32 oracle: per query, softmax(scale * q . k) over its valid slots, times the latent values."""
    outs = []
    for i in range(q.shape[0]):
        sel = idx[i][idx[i] >= 0]
        kv = cache.dequant(sel)                              # [n, 576]
        s = (q[i].float() @ kv.t()) * scale                  # [128, n]
        p = torch.softmax(s, -1)
        outs.append(p @ kv[:, :LATENT])
    return torch.stack(outs)


def default_scale(qk_nope: int = 128, qk_rope: int = 64) -> float:
    return 1.0 / math.sqrt(qk_nope + qk_rope)
