"""Qwen3-style MoE language model (GQA attention with per-head Q/K RMSNorm, RoPE, routed SwiGLU experts).

BASELINE config 2 shape by default: hidden 2048, 48 layers, 32 query / 4 KV heads of dim 128, RoPE theta 1e6,
128 experts top-8 of intermediate 768 (NVFP4), vocab 151936, random-init N(0, 0.02) weights, and a per-layer router
bias that follows a Zipf(1.1) expert popularity so that hot experts exist.

The dense parts are BF16; the projections are plain GEMMs (cuBLAS through torch), the norms, RoPE, KV append and
decode attention are this package's kernels, the MoE is `TieredMoE` (GPU hot slots + CPU engine).
"""
from __future__ import annotations

import dataclasses
import math

import torch

from .. import formats, ops
from ..cache.pool import TieredMoE


@dataclasses.dataclass
class Qwen3MoeConfig:
    hidden: int = 2048
    layers: int = 48
    heads: int = 32
    kv_heads: int = 4
    head_dim: int = 128
    experts: int = 128
    top_k: int = 8
    inter: int = 768
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6
    fmt: str = formats.NVFP4
    zipf_s: float = 1.1
    std: float = 0.02

    @staticmethod
    def tiny(**kw):
        base = dict(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, experts=8, top_k=2, inter=128,
                    vocab=512)
        base.update(kw)
        return Qwen3MoeConfig(**base)


def zipf_bias(E: int, s: float, gen: torch.Generator) -> torch.Tensor:
    """log of a Zipf(s) popularity over a random permutation of the experts: added to the router logits, it makes the
    softmax route probabilities proportional to the popularity (times the data-dependent part)."""
    ranks = torch.randperm(E, generator=gen).float() + 1.0
    p = ranks.pow(-s)
    p = p / p.sum()
    return p.log()


class Qwen3MoeModel:
    def __init__(self, cfg: Qwen3MoeConfig, device='cuda', seed: int = 0, hot_fraction: float = 1.0,
                 engine_threads: int | None = None, mailbox=None, synthetic_experts: bool = True,
                 hot_sets: list[list[int]] | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        g = torch.Generator(device='cpu').manual_seed(seed)
        H, D = cfg.hidden, cfg.head_dim
        dev = self.device

        def randn(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=dev)
            return t.normal_(0.0, cfg.std, generator=torch.Generator(device=dev).manual_seed(
                int(torch.randint(0, 2 ** 31 - 1, (1,), generator=g))))

        self.embed = randn(cfg.vocab, H)
        self.lm_head = randn(cfg.vocab, H)
        self.final_norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.layers = []
        n_hot = cfg.experts if hot_fraction >= 1.0 else max(1, int(round(hot_fraction * cfg.experts)))
        self.mailbox = mailbox
        self.engines = []
        for li in range(cfg.layers):
            L = dict(
                in_norm=torch.ones(H, dtype=torch.bfloat16, device=dev),
                post_norm=torch.ones(H, dtype=torch.bfloat16, device=dev),
                qkv=randn((cfg.heads + 2 * cfg.kv_heads) * D, H),
                q_norm=torch.ones(D, dtype=torch.bfloat16, device=dev),
                k_norm=torch.ones(D, dtype=torch.bfloat16, device=dev),
                o=randn(H, cfg.heads * D),
            )
            router = randn(cfg.experts, H)
            bias = zipf_bias(cfg.experts, cfg.zipf_s, g)
            seed_l = seed * 1000 + li
            if synthetic_experts:   # random codes generated on the GPU (fast), copied to the host for the CPU tier
                ew = formats.synthetic_experts(cfg.experts, H, cfg.inter, cfg.fmt, dev, seed=seed_l, std=cfg.std)
            else:
                ew = formats.random_experts(cfg.experts, H, cfg.inter, cfg.fmt, std=cfg.std, seed=seed_l)
            if hot_sets is not None:
                hot = hot_sets[li]
            elif n_hot < cfg.experts:
                hot = torch.argsort(bias, descending=True)[:n_hot].tolist()   # most popular first (a profile)
            else:
                hot = None
            engine = None
            host = None
            if hot is not None and len(hot) < cfg.experts:
                from ..engine import CpuEngine
                host = ew.to('cpu')
                engine = CpuEngine(host, threads=engine_threads)
                self.engines.append(engine)
            L['moe'] = TieredMoE(li, router, ew, cfg.top_k, hot=hot, router_bias=bias, mailbox=mailbox,
                                 engine=engine, device=dev, host_experts=host)
            del ew
            self.layers.append(L)

    # ------------------------------------------------------------------ state
    def alloc_state(self, batch: int, max_len: int) -> dict:
        cfg = self.cfg
        dev = self.device
        Hkv, D = cfg.kv_heads, cfg.head_dim
        splits = ops.attn_decode_splits(batch, Hkv, max_len)
        G = cfg.heads // cfg.kv_heads
        st = dict(
            batch=batch, max_len=max_len, splits=splits,
            k=[torch.zeros(batch, Hkv, max_len, D, dtype=torch.bfloat16, device=dev) for _ in self.layers],
            v=[torch.zeros(batch, Hkv, max_len, D, dtype=torch.bfloat16, device=dev) for _ in self.layers],
            ws_o=torch.empty(batch * Hkv * splits * G * D, dtype=torch.float32, device=dev),
            ws_ml=torch.empty(batch * Hkv * splits * G * 2, dtype=torch.float32, device=dev),
            counters=torch.zeros(batch * Hkv, dtype=torch.int32, device=dev),
            lengths=torch.zeros(batch, dtype=torch.int32, device=dev),
        )
        return st

    # ------------------------------------------------------------------ decode step (graph capturable)
    def decode_buffers(self, batch: int) -> dict:
        cfg = self.cfg
        dev = self.device
        H = cfg.hidden
        return dict(
            tokens=torch.zeros(batch, dtype=torch.int64, device=dev),
            pos=torch.zeros(batch, dtype=torch.int32, device=dev),
            seqlens=torch.zeros(batch, dtype=torch.int32, device=dev),
            rows=torch.arange(batch, dtype=torch.int32, device=dev),
            x=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            h=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            residual=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            q=torch.empty(batch, cfg.heads, cfg.head_dim, dtype=torch.bfloat16, device=dev),
            attn=torch.empty(batch, cfg.heads, cfg.head_dim, dtype=torch.bfloat16, device=dev),
            moe_out=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            next=torch.zeros(batch, dtype=torch.int64, device=dev),
        )

    def decode_step(self, st: dict, buf: dict):
        """One token per sequence: reads buf['tokens'], buf['pos'] (device), writes buf['next'] (greedy)."""
        cfg = self.cfg
        B = buf['tokens'].shape[0]
        torch.add(buf['pos'], 1, out=buf['seqlens'])
        torch.index_select(self.embed, 0, buf['tokens'], out=buf['residual'])
        scale = 1.0 / math.sqrt(cfg.head_dim)
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.add_rmsnorm(buf['residual'], None, L['in_norm'], buf['h'], cfg.eps)
            else:
                ops.add_rmsnorm(buf['moe_out'], buf['residual'], L['in_norm'], buf['h'], cfg.eps)
            qkv = torch.matmul(buf['h'], L['qkv'].t())
            ops.qk_norm_rope_kv(qkv, L['q_norm'], L['k_norm'], buf['pos'], buf['rows'], buf['q'], st['k'][li],
                                st['v'][li], cfg.heads, cfg.kv_heads, cfg.rope_theta, cfg.eps)
            ops.attn_decode(buf['q'], st['k'][li], st['v'][li], buf['seqlens'], buf['attn'], st['ws_o'], st['ws_ml'],
                            st['counters'], st['splits'], scale)
            o = torch.matmul(buf['attn'].view(B, -1), L['o'].t())
            ops.add_rmsnorm(o, buf['residual'], L['post_norm'], buf['h'], cfg.eps)
            L['moe'].forward(buf['h'], out=buf['moe_out'])
        ops.add_rmsnorm(buf['moe_out'], buf['residual'], self.final_norm, buf['h'], cfg.eps)
        logits = torch.matmul(buf['h'], self.lm_head.t())
        torch.argmax(logits, dim=-1, out=buf['next'])
        return buf['next']

    # ------------------------------------------------------------------ prefill (one sequence)
    def prefill(self, st: dict, tokens: torch.Tensor, row: int = 0, start: int = 0) -> torch.Tensor:
        """Runs `tokens` [T] of sequence `row` from position `start`; fills the KV cache; returns the next token."""
        cfg = self.cfg
        dev = self.device
        T = tokens.shape[0]
        H, D = cfg.hidden, cfg.head_dim
        pos = torch.arange(start, start + T, dtype=torch.int32, device=dev)
        rows = torch.full((T,), row, dtype=torch.int32, device=dev)
        residual = self.embed.index_select(0, tokens.to(dev)).contiguous()
        h = torch.empty_like(residual)
        moe_out = torch.empty_like(residual)
        q = torch.empty(T, cfg.heads, D, dtype=torch.bfloat16, device=dev)
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.add_rmsnorm(residual, None, L['in_norm'], h, cfg.eps)
            else:
                ops.add_rmsnorm(moe_out, residual, L['in_norm'], h, cfg.eps)
            qkv = torch.matmul(h, L['qkv'].t())
            ops.qk_norm_rope_kv(qkv, L['q_norm'], L['k_norm'], pos, rows, q, st['k'][li], st['v'][li], cfg.heads,
                                cfg.kv_heads, cfg.rope_theta, cfg.eps)
            kk = st['k'][li][row:row + 1, :, :start + T]
            vv = st['v'][li][row:row + 1, :, :start + T]
            qq = q.transpose(0, 1).unsqueeze(0)
            attn = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, is_causal=(start == 0),
                                                                    enable_gqa=True)
            o = torch.matmul(attn[0].transpose(0, 1).reshape(T, -1), L['o'].t())
            ops.add_rmsnorm(o, residual, L['post_norm'], h, cfg.eps)
            L['moe'].forward(h, out=moe_out)
        ops.add_rmsnorm(moe_out, residual, self.final_norm, h, cfg.eps)
        logits = torch.matmul(h[-1:], self.lm_head.t())
        st['lengths'][row] = start + T
        return torch.argmax(logits, dim=-1)
