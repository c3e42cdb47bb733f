"""Qwen3-style MoE language model (GQA attention with per-head Q/K RMSNorm, RoPE, routed SwiGLU experts).

The flagship decode shape by default: hidden 2048, 48 layers, 32 query / 4 KV heads of dim 128, RoPE theta 1e6,
128 experts top-8 of intermediate 768 (NVFP4), vocab 151936, random-init N(0, 0.02) weights, and a per-layer router
bias that follows a Zipf(1.1) expert popularity so that hot experts exist.

The dense parts are BF16; the projections are plain GEMMs (cuBLAS through torch), the norms, RoPE, KV append and
decode attention are this package's kernels, the MoE is `TieredMoE` (GPU hot slots + CPU engine).
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import torch

from .. import config, formats, ops
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
    norm_topk: bool = True     # renormalize the top-k routing weights to sum to 1 (Qwen3's norm_topk_prob)

    @staticmethod
    def tiny(**kw):
        base = dict(hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128, experts=8, top_k=2, inter=128,
                    vocab=512)
        base.update(kw)
        return Qwen3MoeConfig(**base)


def _sdpa(q, k, v, mask, causal: bool):
    """Prefill attention (GQA). Long sequences are restricted to the fused kernels (flash / cuDNN / memory-efficient),
    so a shape they cannot take fails instead of falling back to the math path, which materializes T x T scores; when
    GQA itself is what they cannot take, the KV heads are expanded first."""
    F = torch.nn.functional
    if q.shape[2] * k.shape[2] < (1 << 26) or not q.is_cuda:
        return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal, enable_gqa=True)
    from torch.nn.attention import SDPBackend, sdpa_kernel
    fused = [SDPBackend.FLASH_ATTENTION, SDPBackend.CUDNN_ATTENTION, SDPBackend.EFFICIENT_ATTENTION]
    try:
        with sdpa_kernel(fused):
            return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, is_causal=causal, enable_gqa=True)
    except RuntimeError:
        rep = q.shape[1] // k.shape[1]
        with sdpa_kernel(fused):
            return F.scaled_dot_product_attention(q, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1),
                                                  attn_mask=mask, is_causal=causal)


def zipf_temperature(E: int, k: int, s: float, logit_std: float, hot_fraction: float = 0.4, seed: int = 0) -> float:
    """Strength tau of the router bias tau * log(p_zipf) for which the experts' measured route shares follow the
    Zipf(s) popularity: the hot_fraction most popular experts receive the Zipf head mass of the routes after top-k
    selection on logits ~ N(0, logit_std^2) + bias. (tau = 1 would concentrate far more than Zipf: the top-k of a
    peaked softmax takes almost only the head.) Found by bisection on a fixed Monte-Carlo sample."""
    g = torch.Generator().manual_seed(seed)
    r = torch.arange(1, E + 1, dtype=torch.float64)
    p = r.pow(-s)
    p = p / p.sum()
    n_hot = max(1, int(round(hot_fraction * E)))
    target = float(p[:n_hot].sum())
    noise = torch.randn(4096, E, generator=g, dtype=torch.float64) * logit_std
    lo, hi = 0.0, 4.0
    for _ in range(30):
        tau = (lo + hi) / 2
        ids = (noise + tau * p.log()).topk(k, -1).indices
        share = float((ids < n_hot).double().mean())
        lo, hi = (tau, hi) if share < target else (lo, tau)
    return (lo + hi) / 2


def zipf_bias(E: int, s: float, gen: torch.Generator, tau: float = 1.0) -> torch.Tensor:
    """tau * log of a Zipf(s) popularity over a random permutation of the experts, added to the router logits."""
    ranks = torch.randperm(E, generator=gen).float() + 1.0
    p = ranks.pow(-s)
    p = p / p.sum()
    return tau * p.log()


class Qwen3MoeModel:
    def __init__(self, cfg: Qwen3MoeConfig, device='cuda', seed: int = 0, hot_fraction: float = 1.0,
                 engine_threads: int | None = None, mailbox=None, synthetic_experts: bool = True,
                 hot_sets: list[list[int]] | None = None, peer: bool | None = None, weights=None,
                 popularity: torch.Tensor | None = None, progress=None):
        """peer: spread the hot slots over the ranks of the process group (cache/peer.py): every rank holds the same
        model (same seed), its slot pool in symmetric memory, and reads the experts other GPUs hold over NVLink
        (None: XTIER_GPU2_SLOTS=auto / on turns it on).
        weights: a weight source (models/hf.py HFWeights: embed(), lm_head(), final_norm(), layer(li)) instead of
        random init; such a model has no router bias. popularity [layers, experts]: measured route shares (a planner
        profile) that choose the hot and RAM-resident experts when hot_sets is not given; without it the random
        model's Zipf bias does, and a loaded model takes the lowest expert ids. progress(layer, layers): called as
        each layer starts building."""
        if peer is None:
            peer = str(config.get('XTIER_GPU2_SLOTS')).strip().lower() in ('auto', '1', 'on', 'true', 'yes')
        self.cfg = cfg
        self.device = torch.device(device)
        g = torch.Generator(device='cpu').manual_seed(seed)
        H, D = cfg.hidden, cfg.head_dim
        dev = self.device

        def randn(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=dev)
            return t.normal_(0.0, cfg.std, generator=torch.Generator(device=dev).manual_seed(
                int(torch.randint(0, 2 ** 31 - 1, (1,), generator=g))))

        if weights is not None:
            self.embed = weights.embed().to(dev).contiguous()
            self.lm_head = weights.lm_head().to(dev).contiguous()
            self.final_norm = weights.final_norm().to(dev).contiguous()
        else:
            self.embed = randn(cfg.vocab, H)
            self.lm_head = randn(cfg.vocab, H)
            self.final_norm = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.layers = []
        from .. import planner
        if planner.configured():   # per-layer slots from the planner's switches (plan file, fraction, slots, ...)
            hot_counts = [planner.layer_slots(li, cfg.experts, cfg.layers) for li in range(cfg.layers)]
        else:
            n = cfg.experts if hot_fraction >= 1.0 else max(1, int(round(hot_fraction * cfg.experts)))
            hot_counts = [n] * cfg.layers
        partial = any(h < cfg.experts for h in hot_counts)
        if popularity is None and config.get('XTIER_CACHE_PROFILE'):   # a measured route profile fills the slots
            popularity = planner.profile_popularity(config.get('XTIER_CACHE_PROFILE'), cfg.layers, cfg.experts)
        self.mailbox = mailbox
        self.engines = []
        self.cold = None
        self.peers = None
        self.bigram = None   # tables.engram.BigramTable (attach_bigram)
        self.lm_head_fp8 = None   # (E4M3 [V, H], scales [V, H / 128], MXFP8 copy or None): quantize_lm_head
        prank, pworld = 0, 1
        if peer and partial:
            from ..parallel import dist as xdist
            env = xdist.init()
            prank, pworld = env.rank, env.world
            if pworld > 1:
                from ..cache.peer import PeerPools
                bs = 16 if cfg.fmt == formats.NVFP4 else 32
                self.peers = PeerPools([(h, H, cfg.inter, bs) for h in hot_counts], dev)
        if config.get('XTIER_COLD') and partial:
            from ..cache.cold import ColdPool
            if not config.get('XTIER_COLD_DIR'):
                raise ValueError('XTIER_COLD=1 needs XTIER_COLD_DIR (one directory per drive, comma separated)')
            self.cold = ColdPool(config.get('XTIER_COLD_DIR'), parts=config.get('XTIER_COLD_PARTS') or None,
                                 threads=config.get('XTIER_COLD_THREADS'))
        # router logits are N(0, (std * sqrt(H))^2) for RMS-normalized hidden states
        self.zipf_tau = (zipf_temperature(cfg.experts, cfg.top_k, cfg.zipf_s, cfg.std * H ** 0.5)
                         if weights is None else 0.0)
        for li in range(cfg.layers):
            if progress is not None:   # e.g. the server's startup stages (layer li of cfg.layers)
                progress(li, cfg.layers)
            n_hot = hot_counts[li]
            if weights is not None:
                src = weights.layer(li)
                L = {k: src[k].to(dev).contiguous() for k in ('in_norm', 'post_norm', 'qkv', 'q_norm', 'k_norm', 'o')}
                router = src['router'].to(dev).contiguous()
                bias = None
                ew = src['experts']
                del src
            else:
                L = dict(
                    in_norm=torch.ones(H, dtype=torch.bfloat16, device=dev),
                    post_norm=torch.ones(H, dtype=torch.bfloat16, device=dev),
                    qkv=randn((cfg.heads + 2 * cfg.kv_heads) * D, H),
                    q_norm=torch.ones(D, dtype=torch.bfloat16, device=dev),
                    k_norm=torch.ones(D, dtype=torch.bfloat16, device=dev),
                    o=randn(H, cfg.heads * D),
                )
                router = randn(cfg.experts, H)
                bias = zipf_bias(cfg.experts, cfg.zipf_s, g, self.zipf_tau)
                seed_l = seed * 1000 + li
                if synthetic_experts:   # random codes generated on the GPU (fast), copied to the host for the CPU tier
                    ew = formats.synthetic_experts(cfg.experts, H, cfg.inter, cfg.fmt, dev, seed=seed_l, std=cfg.std)
                else:
                    ew = formats.random_experts(cfg.experts, H, cfg.inter, cfg.fmt, std=cfg.std, seed=seed_l)
            # expert popularity of this layer: a measured profile, the random model's bias, or none (id order)
            pop = (popularity[li].float().cpu() if popularity is not None else
                   bias.float().cpu() if bias is not None else torch.zeros(cfg.experts))
            sets = None
            if hot_sets is not None:
                hot = hot_sets[li]
            elif self.peers is not None:
                from ..cache.peer import plan_sets
                sets = plan_sets(cfg.experts, n_hot, pworld, pop)
                hot = sets[prank]
            elif n_hot < cfg.experts:
                hot = sorted(range(cfg.experts), key=lambda e: (-float(pop[e]), e))[:n_hot]   # most popular first
            else:
                hot = None
            engine = None
            host = None
            if hot is not None and len(hot) < cfg.experts:
                from ..engine import CpuEngine
                host = ew.to('cpu')
                if self.cold is not None:   # RAM slots for part of the experts, the rest read from the drives
                    from ..cache.cold import cold_engine
                    engine = cold_engine(li, host, self.cold, config.get('XTIER_COLD_FRACTION'), pop, hot,
                                         threads=engine_threads)
                elif sets is not None:   # peer mode: the CPU tier holds only the experts no GPU's slots hold
                    covered = set().union(*map(set, sets))
                    uncovered = [e for e in range(cfg.experts) if e not in covered]
                    engine = (CpuEngine(host, threads=engine_threads, slots=len(uncovered), resident=uncovered)
                              if uncovered else None)
                else:
                    engine = CpuEngine(host, threads=engine_threads)
                if engine is not None:
                    self.engines.append(engine)
            L['moe'] = TieredMoE(li, router, ew, cfg.top_k, hot=hot, router_bias=bias, renorm=cfg.norm_topk,
                                 mailbox=mailbox,
                                 engine=engine, device=dev, host_experts=host,
                                 pool_storage=self.peers.storage(li) if self.peers is not None else None)
            if sets is not None:
                L['moe'].use_peers(self.peers.table(li), n_hot, prank, sets)
            if self.cold is not None and engine is not None:
                # prefill stages the CPU tier's experts from the engine's RAM slots and the drives; no host copy
                from ..cache.cold import ColdPrefill
                moe = L['moe']
                moe.attach_cold_prefill(ColdPrefill(self.cold, li, engine,
                                                    [e for e in range(cfg.experts) if int(moe.table_host[e]) < 0]))
            L['moe'].prepare_prefill()
            if sets is not None or L['moe'].cold_prefill is not None:
                # peer mode: no swaps, the pinned staging copy is all the host copy is kept for; cold mode: swaps
                # and prefill read the engine and the drives
                L['moe'].host = None
                host = None
            del ew
            self.layers.append(L)
        if self.peers is not None:   # every rank's pool is filled before any rank reads a peer's
            torch.cuda.synchronize()
            from ..parallel import dist as xdist
            xdist.barrier()
        # adaptive hot-slot swaps (AdaptivePolicy) and elastic extra slots (Governor), stepped between decode steps by
        # the runtime (runtime/decode.py Generator)
        self.policy = None
        self.governor = None
        if mailbox is not None and partial:
            from ..cache.policy import AdaptivePolicy
            self.policy = AdaptivePolicy([L['moe'] for L in self.layers], mailbox)
            if config.get('XTIER_CACHE_ELASTIC'):
                from ..cache.elastic import Governor, install
                self.governor = Governor(install(self))
        # swap ring: swaps copy on a side stream; the decode step's first kernel maps the ones that have landed.
        # Layers whose decode kernels read the pinned host pool (XTIER_DECODE_MISS_GPU) keep stream-ordered swaps
        self.ring = None
        if self.policy is not None and dev.type == 'cuda' and config.get('XTIER_CACHE_RING'):
            ring_layers = [L['moe'] for L in self.layers
                           if L['moe'].can_refill and not L['moe'].all_hot and L['moe'].host_table is None]
            if ring_layers:
                from ..cache.ring import SwapRing
                self.ring = SwapRing(ring_layers, dev)

    @classmethod
    def from_pretrained(cls, path, device='cuda', hot_fraction: float = 1.0, fmt: str | None = None, **kw):
        """A model built from a Hugging Face qwen3_moe checkpoint directory (models/hf.py: BF16, ModelOpt NVFP4,
        compressed-tensors NVFP4 or MXFP4 experts; `fmt` (default XTIER_CKPT_FORMAT) for unquantized experts)."""
        from .hf import HFWeights
        dev = torch.device(device)
        w = HFWeights(path, fmt=fmt, quant_device=dev if dev.type == 'cuda' else 'cpu')
        try:
            return cls(w.cfg, device=device, hot_fraction=hot_fraction, weights=w, **kw)
        finally:
            w.close()

    def attach_bigram(self, table):
        """Adds a hashed-bigram NVMe embedding table (tables/engram.py) to the token embeddings, in prefill and inside
        the decode graph. Attach before capturing the decode step."""
        self.bigram = table

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
        if config.get('XTIER_L2_PREFETCH'):
            st['prefetch'] = [self._prefetch_list(li, st) for li in range(len(self.layers))]
            st['side'] = torch.cuda.Stream(device=dev) if dev.type == 'cuda' else None
        return st

    def _prefetch_list(self, li: int, st: dict):
        """Device arrays (addresses, bytes) of what layer li's dense part streams: QKV and output projections,
        router, KV cache. A side branch of the decode graph pulls them into L2 while layer li-1 waits on its CPU
        experts."""
        L = self.layers[li]
        ts = [L['qkv'], L['o'], L['moe'].router_w, st['k'][li], st['v'][li]]
        ptrs = torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device=self.device)
        sizes = torch.tensor([t.numel() * t.element_size() for t in ts], dtype=torch.int64, device=self.device)
        return ptrs, sizes

    # ------------------------------------------------------------------ decode step (graph capturable)
    def decode_buffers(self, batch: int) -> dict:
        cfg = self.cfg
        dev = self.device
        H = cfg.hidden
        return dict(
            tokens=torch.zeros(batch, dtype=torch.int64, device=dev),
            prev=torch.zeros(batch, dtype=torch.int64, device=dev),   # the previous input (hashed n-gram rows)
            pos=torch.zeros(batch, dtype=torch.int32, device=dev),
            seqlens=torch.zeros(batch, dtype=torch.int32, device=dev),
            rows=torch.arange(batch, dtype=torch.int32, device=dev),
            x=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            h=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            residual=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            q=torch.empty(batch, cfg.heads, cfg.head_dim, dtype=torch.bfloat16, device=dev),
            attn=torch.empty(batch, cfg.heads, cfg.head_dim, dtype=torch.bfloat16, device=dev),
            moe_out=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            qkv=torch.empty(batch, (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim, dtype=torch.bfloat16, device=dev),
            o=torch.empty(batch, H, dtype=torch.bfloat16, device=dev),
            logits=torch.empty(batch, cfg.vocab, dtype=torch.bfloat16, device=dev),
            next=torch.zeros(batch, dtype=torch.int64, device=dev),
            temp=torch.zeros(batch, dtype=torch.float32, device=dev),     # per row; 0: greedy (runtime/sampling.py)
            top_p=torch.ones(batch, dtype=torch.float32, device=dev),
        )

    def decode_step(self, st: dict, buf: dict):
        """One token per sequence: reads buf['tokens'], buf['pos'] (device), writes buf['next'] (greedy)."""
        cfg = self.cfg
        B = buf['tokens'].shape[0]
        side = st.get('side') if B <= 16 else None
        main = torch.cuda.current_stream(self.device) if side is not None else None
        forked = False
        if getattr(self, 'ring', None) is not None:   # hot-slot swaps whose copies have landed take effect
            self.ring.commit()
        torch.add(buf['pos'], 1, out=buf['seqlens'])
        torch.index_select(self.embed, 0, buf['tokens'], out=buf['residual'])
        if self.bigram is not None:   # NVMe hashed-bigram rows, looked up inside the graph
            self.bigram.add_decode(buf['residual'], buf['prev'], buf['tokens'])
        scale = 1.0 / math.sqrt(cfg.head_dim)
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.add_rmsnorm(buf['residual'], None, L['in_norm'], buf['h'], cfg.eps)
            else:
                ops.add_rmsnorm(buf['moe_out'], buf['residual'], L['in_norm'], buf['h'], cfg.eps)
            ops.linear(buf['h'], L['qkv'], out=buf['qkv'])
            ops.qk_norm_rope_kv(buf['qkv'], L['q_norm'], L['k_norm'], buf['pos'], buf['rows'], buf['q'], st['k'][li],
                                st['v'][li], cfg.heads, cfg.kv_heads, cfg.rope_theta, cfg.eps)
            ops.attn_decode(buf['q'], st['k'][li], st['v'][li], buf['seqlens'], buf['attn'], st['ws_o'], st['ws_ml'],
                            st['counters'], st['splits'], scale)
            ops.linear(buf['attn'].view(B, -1), L['o'], out=buf['o'])
            ops.add_rmsnorm(buf['o'], buf['residual'], L['post_norm'], buf['h'], cfg.eps)
            if side is not None and li + 1 < len(self.layers):   # next layer's weights into L2 meanwhile
                forked = True
                side.wait_stream(main)
                with torch.cuda.stream(side):
                    ops.l2_prefetch(*st['prefetch'][li + 1])
            L['moe'].forward(buf['h'], out=buf['moe_out'])
        ops.add_rmsnorm(buf['moe_out'], buf['residual'], self.final_norm, buf['h'], cfg.eps)
        if self.lm_head_fp8 is not None:   # W8A16: half the bytes of the largest read of the step
            ops.gemv_fp8(buf['h'], self.lm_head_fp8[0], self.lm_head_fp8[1], buf['logits'])
        else:
            ops.gemv(buf['h'], self.lm_head, buf['logits'])
        if getattr(self, 'sampling', False):   # temperature / top-p per row, decided on the device
            from ..runtime.sampling import sample
            sample(buf['logits'], buf['temp'], buf['top_p'], out=buf['next'])
        else:
            torch.argmax(buf['logits'], dim=-1, out=buf['next'])
        buf['prev'].copy_(buf['tokens'])
        if side is not None and forked:   # a one-layer model never forks the prefetch branch
            main.wait_stream(side)
        return buf['next']

    # ------------------------------------------------------------------ prefill (one sequence)
    def prefill_chunked(self, st: dict, tokens: torch.Tensor, row: int = 0, start: int = 0, chunk: int = 0,
                        return_logits: bool = False):
        """`prefill` of a long prompt in chunks of `chunk` tokens (0: XTIER_LONG_PREFILL_CHUNK, whose default 0 means
        one piece), each continuing after the KV of the ones before, so activations stay bounded by the chunk;
        with a hashed n-gram table the next chunk's rows are read from the drive on a thread while this chunk
        computes. Returns what the last chunk's prefill returns."""
        chunk = chunk or config.get('XTIER_LONG_PREFILL_CHUNK')
        T = tokens.shape[0]
        if chunk <= 0 or T <= chunk:
            return self.prefill(st, tokens, row=row, start=start, return_logits=return_logits)
        bounds = list(range(0, T, chunk)) + [T]
        ahead = None
        res = None
        for i, (a, b) in enumerate(zip(bounds, bounds[1:])):
            if self.bigram is not None:
                ahead_rows = ahead.result() if ahead is not None else None
                if b < T:      # the next chunk's rows, read while this one computes
                    ahead = self.bigram.prefetch_rows(tokens[b:bounds[i + 2]], int(tokens[b - 1]))
                st.setdefault('bigram_rows', {})[row] = ahead_rows
            res = self.prefill(st, tokens[a:b], row=row, start=start + a,
                               return_logits=return_logits and b == T)
        return res

    def prefill(self, st: dict, tokens: torch.Tensor, row: int = 0, start: int = 0, return_logits: bool = False,
                all_logits: bool = False, active: torch.Tensor | None = None, tree=None):
        """Runs `tokens` [T] of sequence `row` from position `start`; fills the KV cache; returns the next token
        (and the last position's logits with return_logits; every position's with all_logits, e.g. a speculative
        verify). `active` (int32 [T] token flags, calls of <= 16 tokens): flag-0 tokens skip their routed experts.
        `tree` (runtime/tree.py Tree, T <= 64 nodes, GPU only): the tokens are a draft tree in breadth-first order;
        node i goes to cache slot start + i at RoPE position start + depth(i) and attends to the cache before `start`
        and to its ancestors (call with all_logits; `compact_tree` keeps the accepted path)."""
        cfg = self.cfg
        dev = self.device
        T = tokens.shape[0]
        H, D = cfg.hidden, cfg.head_dim
        slots = tree_mask = None
        if tree is not None:
            if dev.type != 'cuda' or D != 128 or T != tree.n or T > 64 or self.bigram is not None:
                raise ValueError('tree verification needs the GPU attention kernel (head dim 128), at most 64 nodes '
                                 'and no bigram table')
            pos = torch.as_tensor(start + tree.depth.astype(np.int64), dtype=torch.int32).to(dev)
            slots = torch.arange(start, start + T, dtype=torch.int32, device=dev)
            tree_mask = torch.as_tensor(tree.ancestor_words()).to(dev)
        else:
            pos = torch.arange(start, start + T, dtype=torch.int32, device=dev)
        rows = torch.full((T,), row, dtype=torch.int32, device=dev)
        residual = self.embed.index_select(0, tokens.to(dev)).contiguous()
        if self.bigram is not None:
            last = st.setdefault('last_token', {})
            ahead_rows = st.get('bigram_rows', {}).pop(row, None)     # read ahead by prefill_chunked
            self.bigram.add_prefill(residual, tokens, prev0=last.get(row, 0) if start > 0 else 0, rows=ahead_rows)
            last[row] = int(tokens[-1])
        h = torch.empty_like(residual)
        moe_out = torch.empty_like(residual)
        q = torch.empty(T, cfg.heads, D, dtype=torch.bfloat16, device=dev)
        # prefill attention: the tcgen05 kernel on a GPU (head dim 128); PyTorch's attention on the CPU and with
        # XTIER_PREFILL_ATTN=sdpa
        attn_flat = (torch.empty(T, cfg.heads * D, dtype=torch.bfloat16, device=dev)
                     if dev.type == 'cuda' and D == 128 and (config.get('XTIER_PREFILL_ATTN') != 'sdpa'
                                                             or tree is not None) else None)
        copy_stream = None
        if T >= config.get('XTIER_GPU_PREFILL_MIN') and dev.type == 'cuda':
            copy_stream = getattr(self, '_copy_stream', None) or torch.cuda.Stream(device=dev)
            self._copy_stream = copy_stream
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.add_rmsnorm(residual, None, L['in_norm'], h, cfg.eps)
            else:
                ops.add_rmsnorm(moe_out, residual, L['in_norm'], h, cfg.eps)
            qkv = ops.linear(h, L['qkv'])
            ops.qk_norm_rope_kv(qkv, L['q_norm'], L['k_norm'], pos, rows, q, st['k'][li], st['v'][li], cfg.heads,
                                cfg.kv_heads, cfg.rope_theta, cfg.eps, slots=slots)
            if attn_flat is not None:   # tcgen05 causal GQA kernel, written straight into the o-projection input
                ops.attn_prefill(q, st['k'][li], st['v'][li], row, start, 1.0 / math.sqrt(D),
                                 out=attn_flat.view(T, cfg.heads, D), tree_mask=tree_mask)
                o = ops.linear(attn_flat, L['o'])
            else:
                kk = st['k'][li][row:row + 1, :, :start + T]
                vv = st['v'][li][row:row + 1, :, :start + T]
                qq = q.transpose(0, 1).unsqueeze(0)
                if start == 0 or T == 1:
                    attn = _sdpa(qq, kk, vv, None, start == 0)
                else:   # a continuation chunk: query i sees keys up to position start + i
                    mask = (torch.arange(start + T, device=dev)[None, :] <=
                            (start + torch.arange(T, device=dev))[:, None])
                    attn = _sdpa(qq, kk, vv, mask, False)
                o = ops.linear(attn[0].transpose(0, 1).reshape(T, -1).contiguous(), L['o'])
            ops.add_rmsnorm(o, residual, L['post_norm'], h, cfg.eps)
            if copy_stream is not None and li + 1 < len(self.layers):
                # the next layer's cold experts cross PCIe while this layer computes; its staging buffer (layer
                # parity) was last read by layer li - 1, whose MoE is done when this layer's starts
                done = torch.cuda.Event()
                done.record()
                self.layers[li + 1]['moe'].upload_async(copy_stream, after=done)
            L['moe'].forward(h, out=moe_out, active=active)
        ops.add_rmsnorm(moe_out, residual, self.final_norm, h, cfg.eps)
        if all_logits:
            logits = self._lm_head(h)
            st['lengths'][row] = start + T
            return torch.argmax(logits, dim=-1), logits
        logits = self._lm_head(h[-1:].contiguous())
        st['lengths'][row] = start + T
        nxt = torch.argmax(logits, dim=-1)
        return (nxt, logits[0]) if return_logits else nxt

    def quantize_lm_head(self):
        """The LM head in FP8 E4M3 with one scale per row and 128 columns (e.g. a speculative draft's, whose step is
        dominated by it): the decode step reads it through the W8A16 GEMV, prefill through the W8A8 block-scaled GEMM
        (weights requantized to MXFP8 once). The BF16 copy is freed."""
        if self.lm_head_fp8 is not None or self.device.type != 'cuda':
            return
        w8, s = ops.fp8_quantize(self.lm_head)
        mx8 = ops.fp8_weight_to_mx8(w8, s) if self.lm_head.shape[0] % 128 == 0 else None
        self.lm_head_fp8 = (w8, s, mx8)
        self.lm_head = None

    def _lm_head(self, h):
        if self.lm_head_fp8 is None:
            return ops.linear(h, self.lm_head)
        w8, s, mx8 = self.lm_head_fp8
        return ops.linear_fp8(h, w8, s, mx8=mx8)

    def compact_tree(self, st: dict, row: int, start: int, path: list[int]):
        """After a tree verify: the KV of the accepted nodes `path` (tree node indices, root first) moves to slots
        start .. start + len(path) - 1 (their RoPE positions already), and the row's length ends after them."""
        idx = torch.tensor([start + int(p) for p in path], dtype=torch.long, device=self.device)
        dst = torch.arange(start, start + len(path), dtype=torch.long, device=self.device)
        if not torch.equal(idx, dst):
            for li in range(len(self.layers)):
                for c in (st['k'][li], st['v'][li]):
                    c[row, :, dst] = c[row, :, idx]   # gathered before it is written
        st['lengths'][row] = start + len(path)

    # ------------------------------------------------------------------ fp32 reference (tests)
    def reference_logits(self, tokens: torch.Tensor) -> torch.Tensor:
        """Plain fp32 PyTorch forward of the whole sequence (dequantized experts, causal attention): logits of the
        last position. The oracle of the model tests."""
        cfg = self.cfg
        dev = self.device
        f = torch.float32
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        T = tokens.shape[0]

        def rms(x, w):
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.eps) * w.float()

        pos = torch.arange(T, device=dev, dtype=torch.float64)
        inv = cfg.rope_theta ** (-torch.arange(0, D // 2, device=dev, dtype=torch.float64) * 2 / D)
        ang = pos[:, None] * inv[None]
        cos, sin = ang.cos().to(f)[:, None], ang.sin().to(f)[:, None]

        def rope(t):
            a, b = t[..., :D // 2], t[..., D // 2:]
            return torch.cat([a * cos - b * sin, b * cos + a * sin], -1)

        x = self.embed.index_select(0, tokens.to(dev)).to(f)
        if self.bigram is not None:
            t = tokens.detach().cpu().long()
            r = self.bigram.rows_host(torch.cat([torch.tensor([0]), t[:-1]]), t).to(dev, f)
            x = x + (r @ self.bigram.proj.to(f).t() if self.bigram.proj is not None else r)
        mask = torch.ones(T, T, device=dev, dtype=torch.bool).tril()
        for li_ref, L in enumerate(self.layers):
            h = rms(x, L['in_norm'])
            qkv = (h @ L['qkv'].to(f).t()).view(T, Hq + 2 * Hkv, D)
            q = rope(rms(qkv[:, :Hq], L['q_norm']))
            k = rope(rms(qkv[:, Hq:Hq + Hkv], L['k_norm']))
            v = qkv[:, Hq + Hkv:]
            G = Hq // Hkv
            k = k.repeat_interleave(G, 1)
            v = v.repeat_interleave(G, 1)
            s = torch.einsum('thd,shd->hts', q, k) / D ** 0.5
            s = s.masked_fill(~mask, float('-inf')).softmax(-1)
            a = torch.einsum('hts,shd->thd', s, v).reshape(T, Hq * D)
            x = x + a @ L['o'].to(f).t()
            h = rms(x, L['post_norm'])
            moe = L['moe']
            logits = h @ moe.router_w.to(f).t() + (moe.router_bias if moe.router_bias is not None else 0)
            p = logits.softmax(-1)
            w, ids = p.topk(cfg.top_k, -1)
            if cfg.norm_topk:
                w = w / w.sum(-1, keepdim=True)
            out = torch.zeros_like(x)
            if moe.host is not None:
                src = {e: (moe.host, e) for e in range(moe.E)}
            elif moe.cold_prefill is not None:   # cold mode: the layer rebuilt from the store's records
                full = moe.cold_prefill.pool.load_layer(li_ref)
                src = {e: (full, e) for e in range(moe.E)}
            else:   # this GPU's slots, and the pinned staging copy of the others (peer mode keeps no full copy)
                src = {e: (moe.pool, s) for s, e in enumerate(moe.hot)}
                hc = getattr(moe, '_host_cold', None)
                if hc is not None:
                    ci = moe._cold_index.cpu()
                    src.update({e: (hc, int(ci[e])) for e in range(moe.E) if e not in src and int(ci[e]) >= 0})
            cache = {}
            for t in range(T):
                for j in range(cfg.top_k):
                    e = int(ids[t, j])
                    if e not in cache:
                        ew, i = src[e]
                        w1, w3, w2 = ew.dequant(i)
                        cache[e] = (w1.to(dev), w3.to(dev), w2.to(dev))
                    w1, w3, w2 = cache[e]
                    g = h[t] @ w1.t()
                    u = h[t] @ w3.t()
                    out[t] += w[t, j] * ((torch.nn.functional.silu(g) * u) @ w2.t())
            x = x + out
        x = rms(x, self.final_norm)
        head = (self.lm_head if self.lm_head is not None
                else ops.fp8_dequant(self.lm_head_fp8[0], self.lm_head_fp8[1]))
        return x[-1] @ head.to(f).t()
