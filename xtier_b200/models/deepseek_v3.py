"""DeepSeek-V3-shaped MoE language model (the EP decode, long-prefill and three-tier benchmark shapes).

Shape by default: hidden 7168, 61 layers (the first 3 dense, intermediate 18432), MLA attention with 128 heads,
q_lora 1536, kv_lora 512, qk_nope 128, qk_rope 64, v_head 128; 256 routed MXFP4 experts (intermediate 2048) plus one
shared expert, grouped top-8 routing (8 groups, top-4 groups, sigmoid scores with a selection bias, renormalized,
routed scale 2.5); vocab 129280; random-init N(0, 0.02) weights.

MLA keeps a latent cache: per token the normalized 512-dim compressed KV and the 64-dim rotary key, 576 BF16 values
shared by all heads. Decode uses the absorbed form (queries projected into the latent space, attention over the
latent rows, values projected back per head); prefill expands keys and values per head and runs causal attention.
The MoE layers are `TieredMoE` (one GPU, hot slots + CPU engine) or `EPMoE` (experts split over the ranks, NVLink
peer exchange) — attention is data parallel across ranks (each rank serves its own requests).

Reference parity: the reference runs DeepSeek V4.1 through SGLang with its MoE method (xtier/backend/method.py) and
the DeepSeek pack (xtier/packs/deepseek_v4); this model is the framework's own runner of the named shape.
"""
from __future__ import annotations

import dataclasses
import math

import torch

from .. import formats, ops


@dataclasses.dataclass
class DeepSeekV3Config:
    hidden: int = 7168
    layers: int = 61
    dense_layers: int = 3
    dense_inter: int = 18432
    heads: int = 128
    q_lora: int = 1536
    kv_lora: int = 512
    qk_nope: int = 128
    qk_rope: int = 64
    v_head: int = 128
    experts: int = 256
    shared: int = 1
    top_k: int = 8
    inter: int = 2048
    n_group: int = 8
    topk_group: int = 4
    routed_scale: float = 2.5
    vocab: int = 129280
    rope_theta: float = 10000.0
    eps: float = 1e-6
    fmt: str = formats.MXFP4
    std: float = 0.02
    attn: str = 'auto'        # decode attention: 'torch' (BF16 latent cache), 'mla' (NVFP4 latent cache, tcgen05),
                              # 'dsa' (indexer top-k + 'mla'); 'auto' = 'mla' when the MLA kernels' shape fits
    index_heads: int = 64     # DSA lightning indexer
    index_dim: int = 128
    index_topk: int = 2048

    @staticmethod
    def tiny(**kw):
        base = dict(hidden=512, layers=3, dense_layers=1, dense_inter=1024, heads=4, q_lora=256, kv_lora=128,
                    qk_nope=64, qk_rope=64, v_head=64, experts=16, top_k=4, inter=256, n_group=4, topk_group=2,
                    vocab=1000)
        base.update(kw)
        return DeepSeekV3Config(**base)


def _rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """NeoX-style rotation of the last dim of x [..., T, d] at positions pos [T] (FP32 math)."""
    d = x.shape[-1]
    inv = theta ** (-torch.arange(0, d // 2, device=x.device, dtype=torch.float64) * 2 / d)
    ang = pos.double()[:, None] * inv[None]
    cos, sin = ang.cos().float(), ang.sin().float()
    a, b = x.float()[..., : d // 2], x.float()[..., d // 2:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1).to(x.dtype)


class DeepSeekV3Model:
    def __init__(self, cfg: DeepSeekV3Config, device='cuda', seed: int = 0, moe_factory=None, max_tokens: int = 64):
        """moe_factory(layer, router_w, corr_bias, experts_fn, shared_experts) -> an MoE layer with .forward(x, out);
        experts_fn(rank_slice) generates the quantized experts (synthetic MXFP4 bytes) of the given expert ids.
        Default: every expert on this GPU (TieredMoE, all hot)."""
        self.cfg = cfg
        dev = self.device = torch.device(device)
        g = torch.Generator(device='cpu').manual_seed(seed)
        H = cfg.hidden

        def randn(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=dev)
            return t.normal_(0.0, cfg.std, generator=torch.Generator(device=dev).manual_seed(
                int(torch.randint(0, 2 ** 31 - 1, (1,), generator=g))))

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)
        self.embed = randn(cfg.vocab, H)
        self.lm_head = randn(cfg.vocab, H)
        self.final_norm = ones(H)
        qk = cfg.qk_nope + cfg.qk_rope
        self.layers = []
        for li in range(cfg.layers):
            L = dict(in_norm=ones(H), post_norm=ones(H),
                     q_a=randn(cfg.q_lora, H), q_a_norm=ones(cfg.q_lora), q_b=randn(cfg.heads * qk, cfg.q_lora),
                     kv_a=randn(cfg.kv_lora + cfg.qk_rope, H), kv_a_norm=ones(cfg.kv_lora),
                     kv_b=randn(cfg.heads * (cfg.qk_nope + cfg.v_head), cfg.kv_lora),
                     o=randn(H, cfg.heads * cfg.v_head))
            if cfg.attn == 'dsa':   # own seeds: the other weights are the same with and without the indexer
                gi = torch.Generator(device=dev).manual_seed(seed * 7919 + li)
                L['idx_q'] = (torch.randn(cfg.index_heads * cfg.index_dim, cfg.q_lora, device=dev, generator=gi)
                              * cfg.std).bfloat16()
                L['idx_k'] = (torch.randn(cfg.index_dim, H, device=dev, generator=gi) * cfg.std).bfloat16()
                L['idx_w'] = (torch.randn(cfg.index_heads, H, device=dev, generator=gi) * cfg.std).bfloat16()
            kvb = L['kv_b'].view(cfg.heads, cfg.qk_nope + cfg.v_head, cfg.kv_lora)
            L['w_uk'] = kvb[:, :cfg.qk_nope].contiguous()          # [h, nope, lora]
            L['w_uv'] = kvb[:, cfg.qk_nope:].contiguous()          # [h, v, lora]
            if li < cfg.dense_layers:
                L['gate_up'] = randn(2 * cfg.dense_inter, H)
                L['down'] = randn(H, cfg.dense_inter)
            else:
                router = randn(cfg.experts, H)
                corr = torch.randn(cfg.experts, generator=g) * 0.01
                seed_l = seed * 1000 + li

                def experts_fn(ids, seed_l=seed_l):
                    full = formats.synthetic_experts(len(ids), H, cfg.inter, cfg.fmt, dev, seed=seed_l, std=cfg.std)
                    return full

                shared = formats.synthetic_experts(cfg.shared, H, cfg.inter, cfg.fmt, dev, seed=seed_l + 500,
                                                   std=cfg.std) if cfg.shared else None
                if moe_factory is None:
                    from ..cache.pool import TieredMoE
                    L['moe'] = TieredMoE(li, router, experts_fn(list(range(cfg.experts))), cfg.top_k, shared=shared,
                                         mode=1, n_group=cfg.n_group, topk_group=cfg.topk_group, renorm=True,
                                         scale=cfg.routed_scale, corr_bias=corr, device=dev, max_tokens=16)
                else:
                    L['moe'] = moe_factory(li, router, corr, experts_fn, shared)
            self.layers.append(L)

    # ------------------------------------------------------------------ state
    def kernel_attention(self) -> bool:
        """True when decode attention runs on the MLA kernels (NVFP4 latent cache, tcgen05)."""
        cfg = self.cfg
        fits = cfg.heads == 128 and cfg.kv_lora == 512 and cfg.qk_rope == 64 and self.device.type == 'cuda'
        if cfg.attn in ('mla', 'dsa') and not fits:
            raise ValueError('the MLA kernels need 128 heads, kv_lora 512 and qk_rope 64')
        return cfg.attn in ('mla', 'dsa') or (cfg.attn == 'auto' and fits)

    def alloc_state(self, batch: int, max_len: int) -> dict:
        cfg = self.cfg
        st = dict(batch=batch, max_len=max_len,
                  cache=[torch.zeros(batch, max_len, cfg.kv_lora + cfg.qk_rope, dtype=torch.bfloat16,
                                     device=self.device) for _ in self.layers],
                  lengths=torch.zeros(batch, dtype=torch.int32, device=self.device))
        if self.kernel_attention():
            from ..attention.mla import BLOCK, LatentCache, MlaWorkspace
            st['latent'] = [LatentCache(batch, max_len, self.device) for _ in self.layers]
            nsel = cfg.index_topk if cfg.attn == 'dsa' else (max_len + BLOCK - 1) // BLOCK * BLOCK
            st['mla_ws'] = MlaWorkspace(batch, nsel, self.device)
            if cfg.attn == 'dsa':
                from ..attention.dsa import IndexCache
                st['index'] = [IndexCache(batch, max_len, self.device) for _ in self.layers]
        return st

    # ------------------------------------------------------------------ blocks
    def _mla_project(self, L, h, pos):
        """Queries [T, heads, nope+rope] and the latent cache rows [T, kv_lora + rope] of h [T, H]."""
        cfg = self.cfg
        T = h.shape[0]
        q_a = ops.linear(h, L['q_a'])
        q_a = ops.rmsnorm(q_a.contiguous(), L['q_a_norm'], cfg.eps)
        self._q_a = q_a
        q = ops.linear(q_a, L['q_b']).view(T, cfg.heads, cfg.qk_nope + cfg.qk_rope)
        q_pe = _rope(q[..., cfg.qk_nope:].transpose(0, 1), pos, cfg.rope_theta).transpose(0, 1)
        q = torch.cat([q[..., :cfg.qk_nope], q_pe], -1)
        kv = ops.linear(h, L['kv_a'])
        c = ops.rmsnorm(kv[:, :cfg.kv_lora].contiguous(), L['kv_a_norm'], cfg.eps)
        k_pe = _rope(kv[:, cfg.kv_lora:], pos, cfg.rope_theta)
        return q, torch.cat([c, k_pe], -1)

    def _mla_decode(self, L, q, cache, lengths):
        """Absorbed MLA over the latent cache: q [B, heads, nope+rope] -> [B, heads * v]."""
        cfg = self.cfg
        B = q.shape[0]
        q_lat = torch.einsum('bhn,hnl->bhl', q[..., :cfg.qk_nope].float(), L['w_uk'].float())   # [B, h, lora]
        qf = torch.cat([q_lat, q[..., cfg.qk_nope:].float()], -1)                                # [B, h, lora+rope]
        scale = 1.0 / math.sqrt(cfg.qk_nope + cfg.qk_rope)
        out = torch.empty(B, cfg.heads, cfg.v_head, dtype=torch.float32, device=q.device)
        for b in range(B):
            n = int(lengths[b])
            kv = cache[b, :n].float()                       # [n, lora+rope]
            s = (qf[b] @ kv.t()) * scale                    # [h, n]
            p = torch.softmax(s, -1)
            o_lat = p @ kv[:, :cfg.kv_lora]                 # [h, lora]
            out[b] = torch.einsum('hl,hvl->hv', o_lat, L['w_uv'].float())
        return out.to(torch.bfloat16).view(B, -1)

    def _mla_decode_kernel(self, li, L, st, q, h, q_a, rows, lens):
        """Absorbed MLA decode on the tensor cores over the NVFP4 latent cache: every cached position (dense) or the
        DSA indexer's top-k (sparse). q [B, heads, nope+rope] -> [B, heads * v]."""
        from ..attention import dsa
        from ..attention.mla import mla_decode
        cfg = self.cfg
        B = q.shape[0]
        q_lat = torch.einsum('bhn,hnl->bhl', q[..., :cfg.qk_nope].float(), L['w_uk'].float())
        qf = torch.cat([q_lat, q[..., cfg.qk_nope:].float()], -1).to(torch.bfloat16).contiguous()
        lc = st['latent'][li]
        if cfg.attn == 'dsa':
            qi = ops.linear(q_a, L['idx_q']).view(B, cfg.index_heads, cfg.index_dim)
            w = ops.linear(h, L['idx_w']).float() * cfg.index_heads ** -0.5
            scores = dsa.index_scores(qi, w, st['index'][li], rows, lens)
            idx = dsa.select_slots(scores, rows, cfg.index_topk, st['max_len'])
        else:
            nsel = st['mla_ws'].nsel
            pos = torch.arange(nsel, device=q.device, dtype=torch.int32)[None]
            idx = torch.where(pos < lens[:, None], pos + rows[:, None] * st['max_len'], -1).int()
        o_lat = mla_decode(qf, idx, lc, st['mla_ws'], 1.0 / math.sqrt(cfg.qk_nope + cfg.qk_rope))
        out = torch.einsum('bhl,hvl->bhv', o_lat.float(), L['w_uv'].float())
        return out.to(torch.bfloat16).reshape(B, -1)

    def _mla_prefill(self, L, q, lat, start):
        """Expanded MLA (causal) for one sequence: q [T, h, nope+rope], lat [start+T, lora+rope] -> [T, h*v]."""
        cfg = self.cfg
        T = q.shape[0]
        c, k_pe = lat[:, :cfg.kv_lora], lat[:, cfg.kv_lora:]
        k_nope = torch.einsum('nl,hdl->hnd', c.float(), L['w_uk'].float()).to(torch.bfloat16)   # [h, n, nope]
        v = torch.einsum('nl,hdl->hnd', c.float(), L['w_uv'].float()).to(torch.bfloat16)        # [h, n, v]
        k = torch.cat([k_nope, k_pe.unsqueeze(0).expand(cfg.heads, -1, -1)], -1)
        qq = q.transpose(0, 1)
        mask = None
        if start:
            mask = torch.ones(T, start + T, dtype=torch.bool, device=q.device).tril(start)
        o = torch.nn.functional.scaled_dot_product_attention(qq.unsqueeze(0), k.unsqueeze(0), v.unsqueeze(0),
                                                             attn_mask=mask, is_causal=(start == 0),
                                                             scale=1.0 / math.sqrt(cfg.qk_nope + cfg.qk_rope))
        return o[0].transpose(0, 1).reshape(T, -1)

    def _mlp(self, L, h, out):
        g = ops.linear(h, L['gate_up'])
        I = g.shape[-1] // 2
        a = (torch.nn.functional.silu(g[..., :I].float()) * g[..., I:].float()).to(torch.bfloat16)
        out.copy_(ops.linear(a.contiguous(), L['down']))

    # ------------------------------------------------------------------ forward
    def forward(self, st: dict, tokens: torch.Tensor, rows: torch.Tensor, pos: torch.Tensor, decode: bool):
        """tokens [T] (decode: one per row), rows [T] cache row, pos [T] position. Returns logits of the last token
        (prefill) or of every token (decode)."""
        cfg = self.cfg
        residual = self.embed.index_select(0, tokens).contiguous()
        h = torch.empty_like(residual)
        blk = torch.empty_like(residual)
        T = tokens.shape[0]
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.add_rmsnorm(residual, None, L['in_norm'], h, cfg.eps)
            else:
                ops.add_rmsnorm(blk, residual, L['in_norm'], h, cfg.eps)
            q, lat = self._mla_project(L, h, pos)
            cache = st['cache'][li]
            cache[rows.long(), pos.long()] = lat
            if 'latent' in st:
                slots = rows.long() * st['max_len'] + pos.long()
                st['latent'][li].write(lat, slots)
                if 'index' in st:
                    st['index'][li].write(ops.linear(h, L['idx_k']), slots)
            if decode:
                lens = pos + 1
                if 'latent' in st:
                    a = self._mla_decode_kernel(li, L, st, q, h, self._q_a, rows, lens)
                else:
                    a = self._mla_decode(L, q, cache[rows.long()], lens)
            else:
                start = int(pos[0])
                a = self._mla_prefill(L, q, cache[int(rows[0]), :start + T], start)
            o = ops.linear(a.contiguous(), L['o'])
            ops.add_rmsnorm(o, residual, L['post_norm'], h, cfg.eps)
            if 'moe' in L:
                L['moe'].forward(h, out=blk)
            else:
                self._mlp(L, h, blk)
        ops.add_rmsnorm(blk, residual, self.final_norm, h, cfg.eps)
        x = h if decode else h[-1:]
        return ops.linear(x.contiguous(), self.lm_head)

    def prefill(self, st, tokens, row: int = 0):
        T = tokens.shape[0]
        pos = torch.arange(T, dtype=torch.int32, device=self.device)
        rows = torch.full((T,), row, dtype=torch.int32, device=self.device)
        logits = self.forward(st, tokens.to(self.device), rows, pos, decode=False)
        st['lengths'][row] = T
        return logits.argmax(-1)

    def decode_step(self, st, tokens, rows):
        pos = st['lengths'][rows.long()].clone()
        logits = self.forward(st, tokens, rows, pos, decode=True)
        st['lengths'][rows.long()] += 1
        return logits.argmax(-1)
