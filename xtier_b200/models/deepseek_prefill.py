"""Long-prompt prefill of the DeepSeek-V3-shaped model with DSA sparse attention over the ranks of a node (the 64K
time-to-first-token of benchmark config 4).

Layout: the prompt's tokens are split over the W ranks in contiguous slices (sequence parallel); every rank runs the
dense parts of every layer on its own slice. Per layer:

  * projections of the slice on the tcgen05 GEMM: fused [q_a | kv_a], q_b, the indexer's key / query / head-weight
    projections; `mla_prep` writes each token's NVFP4 latent row and `dsa_key_write` its FP8 index key at the token's
    position. The two caches of the layer (416 + 132 bytes per token) are then all-gathered, so every rank holds the
    keys of the whole prompt (27 MB + 8.6 MB per layer at 64K tokens: small next to the weights).
  * attention, per chunk of queries: the lightning indexer scores every earlier key on the tensor cores (FP8,
    `attention/dsa.py`), a radix select keeps each query's top `index_topk` positions, and the one-pass tcgen05 MLA
    kernel (`attention/mla.py` mla_flash) attends over exactly those latent rows; the queries enter absorbed
    (q_nope . W_uk) and the latent output leaves through W_uv.
  * the MoE, expert parallel: each token's routes (top-8 + the shared expert) are sorted by owner rank, the token rows
    and route weights cross with one all-to-all, the owner runs its pool's experts as grouped FP4 tcgen05 GEMMs
    (`cache/prefill.py`, weights read once per 128 routed tokens), the weighted rows come back with a second
    all-to-all and every token sums its routes in route order.

Every rank ends the layer with its slice's residual stream; the rank holding the last token produces the first
generated token. The exchanges are NCCL collectives (plumbing of a prefill that is compute-bound); the decode step's
exchange is the in-kernel one (`parallel/ep.py`).

Reference parity: the reference prefills through SGLang with its own chunked sparse attention (DeepSeek V4 pack:
xtier/packs/deepseek_v4/sparse_mla.py) and the grouped expert GEMMs of xtier/backend/prefill.py:64-140.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .. import ops
from ..attention import dsa
from ..attention.mla import BLOCK, FlashWorkspace, LatentCache
from ..cache.prefill import grouped_routes
from ..parallel import dist as xdist
from .deepseek_v3 import DeepSeekV3Model, _rope


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int]):
    if xdist.get().world == 1:
        out.copy_(inp)
    else:
        dist.all_to_all_single(out, inp, out_splits, in_splits)


class EPPrefillMoE:
    """Prefill-sized calls of an EPMoE layer (every expert in some rank's HBM): route, all-to-all to the owners,
    grouped GEMMs on the owner's pool, all-to-all back, route-ordered combine."""

    def __init__(self, chunk: int = 16384, mx: bool = True):
        self.chunk = chunk
        self.mx = mx   # MXFP8 activations on the block-scaled FP4 kernel (the reference's prefill numerics)
        self.err = None
        self.count = None

    def forward(self, moe, x: torch.Tensor, out: torch.Tensor, add: torch.Tensor | None = None):
        c = moe.comm
        W, kk, spr = c.W, c.k, c.spr
        dev = x.device
        H = x.shape[1]
        if self.err is None:
            self.err = torch.zeros(1, dtype=torch.int32, device=dev)
            self.count = torch.zeros(self.chunk, dtype=torch.int32, device=dev)
        r = moe.router
        for s in range(0, x.shape[0], self.chunk):
            e = min(x.shape[0], s + self.chunk)
            xc = x[s:e].contiguous()
            m = e - s
            logits = ops.gemm_f32(xc, r.w)
            ids = torch.empty(m, kk, dtype=torch.int32, device=dev)
            wt = torch.empty(m, kk, dtype=torch.float32, device=dev)
            slots = torch.empty(m, kk, dtype=torch.int32, device=dev)
            ops.moe_route(xc, r.w, r.bias, r.corr, r.table, r.shared_slots, ids, wt, slots, logits,
                          self.count, r.k, r.mode, r.n_group, r.topk_group, r.renorm, r.scale, moe.layer, 0, None,
                          logits)
            flat = slots.flatten().long()
            if bool((flat < 0).any()):
                raise RuntimeError('EP prefill: a route has no GPU slot (the CPU tier is a decode path)')
            add_c = None if add is None else add[s:e].contiguous()
            if W == 1:   # every route is local: grouped GEMMs straight from the chunk, rows written in route order
                Y, dest = grouped_routes(xc, slots, wt, moe.local, self.err, route_rows=True, mx=self.mx)
                torch.ops.xtier.route_combine(Y, dest, None, None, add_c, out[s:e])
                self.last = (ids, wt)
                continue
            owner = flat // spr
            n = flat.numel()
            order = torch.sort(owner, stable=True).indices   # by owner, route order inside
            send = torch.bincount(owner, minlength=W)
            recv = torch.empty_like(send)
            _a2a(recv, send, [1] * W, [1] * W)
            sc, rc = send.tolist(), recv.tolist()
            rows = xc.index_select(0, order // kk)
            meta = torch.stack([(flat % spr)[order].int(), wt.flatten()[order].view(torch.int32)], 1).contiguous()
            nr = sum(rc)
            r_rows = torch.empty(nr, H, dtype=xc.dtype, device=dev)
            r_meta = torch.empty(nr, 2, dtype=torch.int32, device=dev)
            _a2a(r_rows, rows, rc, sc)
            _a2a(r_meta, meta, rc, sc)
            del rows
            y = torch.empty(nr, H, dtype=torch.float32, device=dev)
            if nr:   # the received routes' rows, written in received order by the down GEMM
                r_w = r_meta[:, 1:].contiguous().view(torch.float32)
                grouped_routes(r_rows, r_meta[:, :1].contiguous(), r_w, moe.local, self.err, route_rows=True, out=y,
                               mx=self.mx)
            del r_rows
            back = torch.empty(n, H, dtype=torch.float32, device=dev)
            _a2a(back, y, sc, rc)
            del y
            inv = torch.empty(n, dtype=torch.int32, device=dev)   # route -> its row of `back`
            inv[order] = torch.arange(n, dtype=torch.int32, device=dev)
            torch.ops.xtier.route_combine(back, inv, None, None, add_c, out[s:e])
            self.last = (ids, wt)   # the last chunk's routes (tests)
        return out


class SparsePrefill:
    """Prefill of one prompt of `total` tokens split over the process group (see the module docstring).

    `model` is a DeepSeekV3Model built with ep=True (world = the group) and `indexer=True`, every expert in HBM.
    dense=True replaces the indexer + sparse attention by causal attention over every earlier key (the expanded form
    of `DeepSeekV3Model._mla_prefill`), the oracle of the tests. mx=False runs the experts on the exact W4A16 kernel
    instead of the block-scaled MXFP4 x MXFP8 one."""

    def __init__(self, model: DeepSeekV3Model, total: int, q_chunk: int = 1024, moe_chunk: int = 16384,
                 dense: bool = False, mx: bool = True):
        cfg = model.cfg
        env = xdist.get()
        self.model, self.cfg = model, cfg
        self.W, self.rank = env.world, env.rank
        if total % self.W:
            raise ValueError(f'{total} tokens do not split over {self.W} ranks')
        self.total, self.Tl = total, total // self.W
        self.q_chunk = q_chunk
        self.dense = dense
        self.topk = min(cfg.index_topk, (total + BLOCK - 1) // BLOCK * BLOCK)
        dev = model.device
        self.latent = [LatentCache(1, total, dev) for _ in model.layers]
        self.index = [dsa.IndexCache(1, total, dev) for _ in model.layers]
        self.ws = FlashWorkspace(q_chunk, 1, dev)
        self.moe = EPPrefillMoE(moe_chunk, mx)
        self.scores = torch.empty(q_chunk, total, dtype=torch.float32, device=dev)
        self.idx_err = torch.zeros(1, dtype=torch.int32, device=dev)

    def _gather_caches(self, li: int):
        if self.W == 1:
            return
        s0, s1 = self.rank * self.Tl, (self.rank + 1) * self.Tl
        for t in (self.latent[li].codes, self.latent[li].scales, self.latent[li].rope, self.index[li].codes,
                  self.index[li].scale):
            mine = t[s0:s1].clone()
            dist.all_gather_into_tensor(t, mine)

    def _attention(self, L, li, q, q_a, h, pos) -> torch.Tensor:
        """q [Tl, heads, nope+rope] (before RoPE), q_a [Tl, q_lora], h [Tl, H] -> [Tl, heads * v]."""
        cfg = self.cfg
        T = q.shape[0]
        out = torch.empty(T, cfg.heads * cfg.v_head, dtype=torch.bfloat16, device=q.device)
        scale = 1.0 / math.sqrt(cfg.qk_nope + cfg.qk_rope)
        lc = self.latent[li]
        if self.dense:
            lat = lc.dequant(torch.arange(self.total, device=q.device)).to(torch.bfloat16)
        for c0 in range(0, T, self.q_chunk):
            c1 = min(T, c0 + self.q_chunk)
            C = c1 - c0
            qc = q[c0:c1]
            pc = pos[c0:c1]
            if self.dense:
                q_pe = _rope(qc[..., cfg.qk_nope:].transpose(0, 1), pc, cfg.rope_theta).transpose(0, 1)
                qq = torch.cat([qc[..., :cfg.qk_nope], q_pe], -1)
                for i in range(C):   # causal, one query at a time (test sizes)
                    p = int(pc[i])
                    out[c0 + i] = self.model._mla_prefill(L, qq[i:i + 1], lat[:p + 1], p)[0]
                continue
            # absorbed queries, head-major: latent part [heads, C, kv_lora] by one batched GEMM, rotary part
            # [heads, C, rope] by the RoPE kernel; flash MLA reads both through strided views, no [C, heads, 576] copy
            q_lat = torch.bmm(qc[..., :cfg.qk_nope].transpose(0, 1), L['w_uk'])
            q_pe = torch.empty(cfg.heads, C, cfg.qk_rope, dtype=torch.bfloat16, device=q.device)
            ops.rope_heads(qc[..., cfg.qk_nope:], pc, cfg.rope_theta, q_pe.transpose(0, 1))
            # indexer: top-k earlier positions of every query (slot = position: one sequence)
            qi = ops.linear(q_a[c0:c1], L['idx_q']).view(C, cfg.index_heads, cfg.index_dim)
            wi = ops.linear(h[c0:c1], L['idx_w'])
            lens = pc + 1
            sc = dsa.index_scores_prefill(qi, wi, self.index[li], 0, lens, out=self.scores[:C], err=self.idx_err,
                                          w_scale=cfg.index_heads ** -0.5)
            idx = dsa.topk(sc, self.topk, lengths=lens)
            o_lat = torch.empty(cfg.heads, C, cfg.kv_lora, dtype=torch.bfloat16, device=q.device)
            torch.ops.xtier.mla_flash(q_lat.transpose(0, 1), idx, lc.codes, lc.scales, lc.rope, None, None,
                                      o_lat.transpose(0, 1), float(scale), 1, self.ws.err, q_pe.transpose(0, 1))
            out[c0:c1] = torch.bmm(o_lat, L['w_uvT']).transpose(0, 1).reshape(C, -1)
        return out

    @torch.no_grad()
    def run(self, ids: torch.Tensor, return_logits: bool = False) -> torch.Tensor:
        """ids: this rank's slice of the prompt [Tl] (device). Returns the next token (on the rank holding the last
        prompt token; other ranks return -1), or that token's logits with return_logits."""
        cfg, model = self.cfg, self.model
        dev = model.device
        T = self.Tl
        pos = torch.arange(self.rank * T, (self.rank + 1) * T, dtype=torch.int32, device=dev)
        slot = pos.long()
        residual = model.embed.index_select(0, ids).contiguous()
        h = torch.empty_like(residual)
        blk = torch.empty_like(residual)
        q_a = torch.empty(T, cfg.q_lora, dtype=torch.bfloat16, device=dev)
        for li, L in enumerate(model.layers):
            if li == 0:
                ops.add_rmsnorm(residual, None, L['in_norm'], h, cfg.eps)
            else:
                ops.add_rmsnorm(blk, residual, L['in_norm'], h, cfg.eps)
            qkv = ops.linear(h, L['qkv_a'])
            lc = self.latent[li]
            ops.mla_prep(qkv, cfg.q_lora, L['q_a_norm'], L['kv_a_norm'], pos, slot, cfg.eps, cfg.rope_theta, q_a,
                         lc.codes, lc.scales, lc.rope)
            del qkv
            self.index[li].write(ops.linear(h, L['idx_k']), slot)
            self._gather_caches(li)
            q = ops.linear(q_a, L['q_b']).view(T, cfg.heads, cfg.qk_nope + cfg.qk_rope)
            a = self._attention(L, li, q, q_a, h, pos)
            del q
            o = ops.linear(a, L['o'])
            del a
            ops.add_rmsnorm(o, residual, L['post_norm'], h, cfg.eps)
            if 'moe' in L:
                self.moe.forward(L['moe'], h, blk)
            else:
                model._mlp(L, h, blk)
        ops.add_rmsnorm(blk, residual, model.final_norm, h, cfg.eps)
        if self.rank == self.W - 1:
            logits = ops.linear(h[-1:].contiguous(), model.lm_head)
            return logits[0] if return_logits else logits.argmax(-1)
        return torch.full((1,), -1, dtype=torch.int64, device=dev)

    def check(self):
        for name, e in (('indexer', self.idx_err), ('MLA', self.ws.err), ('expert GEMM', self.moe.err)):
            code = 0 if e is None else int(e.item())
            if code == 2:
                raise RuntimeError(f'sparse prefill: the {name} kernel met a cache slot out of range')
            if code:
                raise RuntimeError(f'sparse prefill: a bounded wait of the {name} kernel ran out')
