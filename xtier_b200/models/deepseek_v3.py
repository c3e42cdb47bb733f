"""DeepSeek-V3-shaped MoE language model (the EP decode, long-prefill and three-tier benchmark shapes).

Shape by default: hidden 7168, 61 layers (the first 3 dense, intermediate 18432), MLA attention with 128 heads,
q_lora 1536, kv_lora 512, qk_nope 128, qk_rope 64, v_head 128; 256 routed MXFP4 experts (intermediate 2048) plus one
shared expert, grouped top-8 routing (8 groups, top-4 groups, sigmoid scores with a selection bias, renormalized,
routed scale 2.5); vocab 129280; random-init N(0, 0.02) weights.

MLA keeps a latent cache: per token the normalized 512-dim compressed KV and the 64-dim rotary key, shared by all
heads (NVFP4 latent + BF16 rotary key, 416 bytes per token, for the tensor-core kernels; BF16 for the plain PyTorch
path). Decode uses the absorbed form: the queries are projected into the latent space (q_nope . W_uk), attention
runs over the latent rows, and the latent output is projected back per head (. W_uv^T); prefill expands keys and
values per head and runs causal attention.

Two ways to hold the MoE layers:
  * `TieredMoE` (default, one GPU, every expert in the GPU pool): the small test shapes.
  * expert parallelism (`ep=True`): the group's ranks own E / W experts each (`parallel/ep.py` EPMoE); when the GPUs
    cannot hold them all (`gpu_experts`), every owner keeps part of its range in its GPU pool and the rest form a CPU
    tier computed by each rank's CPU engine through the mailbox. Attention is data parallel (each rank serves its own
    requests), so one decode step of the group runs `batch` requests per rank.

The batched decode step (`decode_buffers` / `decode_step`, captured into one CUDA graph by runtime/decode.py
Generator) runs per layer: fused [q_a | kv_a] GEMV, mla_prep (both RMSNorms, RoPE, NVFP4 cache write), q_b GEMV, query
absorption + RoPE (head_gemm), the tcgen05 MLA attention over every cached position, value un-absorption (head_gemm),
o GEMV, MoE (route + EP exchange + expert streams + combine, CPU tier through the mailbox) or the dense MLP.

Reference parity: the reference runs DeepSeek V4.1 through SGLang with its MoE method (xtier/backend/method.py) and
the DeepSeek pack (xtier/packs/deepseek_v4); this model is the framework's own runner of the named shape.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
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

    def expert_bytes(self) -> int:
        """Bytes of one routed expert (codes + block scales, gate/up and down)."""
        bs = formats.BLOCK[self.fmt]
        return 3 * self.inter * self.hidden // 2 + 3 * self.inter * self.hidden // bs

    def moe_layers(self) -> int:
        return self.layers - self.dense_layers

    def dense_bytes(self, indexer: bool = False) -> int:
        """Bytes of everything but the routed experts (BF16 attention, dense MLPs, embeddings, shared experts,
        routers, norms; with `indexer`, the DSA indexer's projections)."""
        H = self.hidden
        qk = self.qk_nope + self.qk_rope
        attn = (H * (self.q_lora + self.kv_lora + self.qk_rope) + self.heads * qk * self.q_lora +
                self.heads * self.qk_nope * self.kv_lora + self.heads * self.kv_lora * self.v_head +
                H * self.heads * self.v_head) * 2
        mlp = 3 * H * self.dense_inter * 2
        moe = self.shared * self.expert_bytes() + self.experts * H * 2
        idx = (self.index_heads * self.index_dim * self.q_lora + self.index_dim * H + self.index_heads * H) * 2
        return (self.layers * (attn + (idx if indexer else 0)) + self.dense_layers * mlp + self.moe_layers() * moe +
                2 * self.vocab * H * 2)


def _rope(x: torch.Tensor, pos: torch.Tensor, theta: float) -> torch.Tensor:
    """NeoX-style rotation of the last dim of x [..., T, d] at positions pos [T] (FP32 math)."""
    d = x.shape[-1]
    inv = theta ** (-torch.arange(0, d // 2, device=x.device, dtype=torch.float64) * 2 / d)
    ang = pos.double()[:, None] * inv[None]
    cos, sin = ang.cos().float(), ang.sin().float()
    a, b = x.float()[..., : d // 2], x.float()[..., d // 2:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], -1).to(x.dtype)


def _fill_random_codes(t: torch.Tensor, gen: torch.Generator):
    """Uniform random bytes into a uint8 tensor (in chunks, so no large temporary)."""
    flat = t.view(-1)
    step = 1 << 28
    for s in range(0, flat.numel(), step):
        torch.randint(0, 256, (min(step, flat.numel() - s),), dtype=torch.uint8, device=t.device, generator=gen,
                      out=flat[s:s + step])


def synthetic_into(ew: formats.ExpertWeights, gen: torch.Generator, std: float):
    """Random experts written in place into preallocated tensors (the generator of formats.synthetic_experts without
    its full-size temporaries): uniform E2M1 codes and one block scale giving roughly N(0, std)-sized weights."""
    _fill_random_codes(ew.w13, gen)
    _fill_random_codes(ew.w2, gen)
    if ew.fmt == formats.NVFP4:
        sv = torch.tensor([std * 2.5 / 6.0], device=ew.s13.device).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        sv = torch.tensor([127 + round(math.log2(std * 2.5 / 4.0))], dtype=torch.uint8, device=ew.s13.device)
    ew.s13.copy_(sv.expand_as(ew.s13))
    ew.s2.copy_(sv.expand_as(ew.s2))
    ew.g13.fill_(1.0)
    ew.g2.fill_(1.0)


def synthetic_experts_by_id(ew: formats.ExpertWeights, ids, seed: int, std: float):
    """Random experts in place, expert ew[i] drawn from a generator seeded by (seed, ids[i]): the bytes of an expert do
    not depend on where it is placed (which rank's pool, the GPU or the CPU tier), so a model is the same at any GPU
    count."""
    synthetic_into(ew, torch.Generator(device=ew.w13.device).manual_seed(seed), std)   # scales
    for i, e in enumerate(ids):
        g = torch.Generator(device=ew.w13.device).manual_seed(seed * 1000003 + int(e))
        _fill_random_codes(ew.w13[i], g)
        _fill_random_codes(ew.w2[i], g)


def empty_experts(n: int, H: int, I: int, fmt: str, device, pin: bool = False) -> formats.ExpertWeights:
    bs = formats.BLOCK[fmt]
    kw = dict(device=device, pin_memory=pin) if str(device) == 'cpu' else dict(device=device)
    return formats.ExpertWeights(fmt, torch.empty(n, 2 * I, H // 2, dtype=torch.uint8, **kw),
                                 torch.empty(n, H, I // 2, dtype=torch.uint8, **kw),
                                 torch.empty(n, 2 * I, H // bs, dtype=torch.uint8, **kw),
                                 torch.empty(n, H, I // bs, dtype=torch.uint8, **kw),
                                 torch.empty(n, 2, dtype=torch.float32, **kw),
                                 torch.empty(n, dtype=torch.float32, **kw))


def ep_layout(E: int, world: int, gpu_per_rank: int, seed: int, stride: int | None = None):
    """Expert placement of one MoE layer over `world` ranks: owner r holds experts [r * El, (r + 1) * El); the
    first `gpu_per_rank` of its range in a seeded order sit in its GPU pool (slot order), the rest in the CPU tier.
    Returns (table [E] int32: owner * stride + slot or -1, per-rank lists of pool experts, CPU-tier experts); stride
    is the pool width (default gpu_per_rank; more when shared experts follow the routed ones)."""
    stride = gpu_per_rank if stride is None else stride
    El = E // world
    g = torch.Generator().manual_seed(seed)
    table = torch.full((E,), -1, dtype=torch.int32)
    pools, cpu = [], []
    for r in range(world):
        order = (torch.randperm(El, generator=g) + r * El).tolist()
        pool = sorted(order[:gpu_per_rank])
        for s, e in enumerate(pool):
            table[e] = r * stride + s
        pools.append(pool)
        cpu += order[gpu_per_rank:]
    return table, pools, sorted(cpu)


def ep_layout_ranked(E: int, world: int, n_gpu: int, popularity, stride: int, width: int | None = None):
    """Expert placement of one MoE layer when a plan gives its node-wide GPU expert count: the `n_gpu` most routed
    experts (by `popularity`, any per-expert score) sit in their owners' pools (owner r holds experts
    [r * El, (r + 1) * El)), the rest in the CPU tier, most routed first. Returns (table, pools, cpu) as ep_layout;
    a pool over `width` slots (default stride) raises."""
    width = stride if width is None else width
    El = E // world
    pop = np.asarray(popularity, dtype=np.float64)
    order = sorted(range(E), key=lambda e: (-pop[e], e))
    gpu = set(order[:max(0, min(E, n_gpu))])
    table = torch.full((E,), -1, dtype=torch.int32)
    pools = []
    for r in range(world):
        pool = [e for e in range(r * El, (r + 1) * El) if e in gpu]
        if len(pool) > width:
            raise ValueError(f'ep_layout_ranked: rank {r} gets {len(pool)} experts, its pool has {width} slots')
        for s, e in enumerate(pool):
            table[e] = r * stride + s
        pools.append(pool)
    return table, pools, [e for e in order if e not in gpu]


def ranked_pool_width(E: int, world: int, plan: dict, popularity: dict) -> int:
    """The largest per-rank pool `ep_layout_ranked` makes over the layers of `plan` ({layer: node-wide GPU experts})."""
    El = E // world
    width = 1
    for li, n in plan.items():
        pop = np.asarray(popularity[li], dtype=np.float64)
        top = sorted(range(E), key=lambda e: (-pop[e], e))[:n]
        counts = np.bincount(np.asarray(top, dtype=np.int64) // El, minlength=world) if top else [0]
        width = max(width, int(max(counts)))
    return width


class DeepSeekV3Model:
    def __init__(self, cfg: DeepSeekV3Config, device='cuda', seed: int = 0, moe_factory=None, max_tokens: int = 64,
                 ep: bool = False, gpu_experts: int | None = None, mailbox=None, engine_threads: int | None = None,
                 decode_tokens: int = 16, ep_timeout_s: float = 30.0, indexer: bool = False,
                 gpu_plan: dict | None = None, popularity: dict | None = None, cold=None,
                 ram_experts: int | None = None, plan_fn=None, pcie_slots: int | None = None):
        """moe_factory(layer, router_w, corr_bias, experts_fn, shared_experts) -> an MoE layer with .forward(x, out);
        experts_fn(ids) generates the quantized experts (synthetic MXFP4 bytes) of the given expert ids.
        Default: every expert on this GPU (TieredMoE, all hot).
        ep: expert parallelism over the process group (world 1 allowed); `gpu_experts` pool slots per rank and MoE
        layer (default: every owned expert), the rest in the CPU tier through `mailbox` (required then) with
        `engine_threads` workers; `decode_tokens` tokens per rank and step. indexer: build the DSA indexer's
        projections whatever the decode attention (the sparse prefill needs them).
        Three tiers (ep only): `gpu_plan` {MoE layer: node-wide GPU experts} (a planner output) places each layer's
        most routed experts by `popularity` {layer: per-expert score} in their owners' pools; with `cold` (a
        cache.cold.ColdPool) the CPU engine of a layer keeps `ram_experts` of the rest in RAM and reads the others
        from the cold store on demand (rank 0 writes the layer's records, the other ranks fill their RAM slots from
        them). `plan_fn({layer: (router_w, corr_bias)}) -> (gpu_plan, popularity)` computes both once every
        layer's router exists.
        pcie_slots (ep with a RAM-only CPU tier; default XTIER_EP_PCIE_SLOTS): GPU staging slots, shared by the
        layers, for CPU-tier experts the GPU reads from the engine's own host memory over PCIe while the engine
        computes the others (the engine's shards are registered with CUDA)."""
        self.cfg = cfg
        dev = self.device = torch.device(device)
        g = torch.Generator(device='cpu').manual_seed(seed)
        H = cfg.hidden
        self.mailbox = mailbox
        self.engines = []
        self.host_maps = []   # engine shards registered with CUDA (unregistered before the engines go)
        self.pcie_slots = 0
        self.ep = None
        self.decode_tokens = decode_tokens
        self.gpu_plan, self.popularity, self.cold, self.ram_experts = gpu_plan, popularity, cold, ram_experts
        self.bigram = None   # tables.engram.BigramTable (attach_bigram)
        self.keep_bf16_cache = False   # alloc_state keeps the BF16 latent cache too (continuations, chunked prompts)
        if gpu_plan is not None and (not ep or popularity is None):
            raise ValueError('gpu_plan places experts by popularity under expert parallelism')

        def randn(*shape):
            t = torch.empty(*shape, dtype=torch.bfloat16, device=dev)
            return t.normal_(0.0, cfg.std, generator=torch.Generator(device=dev).manual_seed(
                int(torch.randint(0, 2 ** 31 - 1, (1,), generator=g))))

        ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)
        self.embed = randn(cfg.vocab, H)
        self.lm_head = randn(cfg.vocab, H)
        self.final_norm = ones(H)
        qk = cfg.qk_nope + cfg.qk_rope
        stage = None
        self.layers = []
        pending = []   # MoE layers: built once every layer's router exists (a plan may depend on all of them)
        for li in range(cfg.layers):
            L = dict(in_norm=ones(H), post_norm=ones(H),
                     qkv_a=randn(cfg.q_lora + cfg.kv_lora + cfg.qk_rope, H), q_a_norm=ones(cfg.q_lora),
                     q_b=randn(cfg.heads * qk, cfg.q_lora), kv_a_norm=ones(cfg.kv_lora),
                     w_uk=randn(cfg.heads, cfg.qk_nope, cfg.kv_lora),      # [h, nope, lora]
                     w_uvT=randn(cfg.heads, cfg.kv_lora, cfg.v_head),      # [h, lora, v] (W_uv transposed)
                     o=randn(H, cfg.heads * cfg.v_head))
            if cfg.attn == 'dsa' or indexer:   # own seeds: the other weights are the same with and without it
                gi = torch.Generator(device=dev).manual_seed(seed * 7919 + li)
                L['idx_q'] = (torch.randn(cfg.index_heads * cfg.index_dim, cfg.q_lora, device=dev, generator=gi)
                              * cfg.std).bfloat16()
                L['idx_k'] = (torch.randn(cfg.index_dim, H, device=dev, generator=gi) * cfg.std).bfloat16()
                L['idx_w'] = (torch.randn(cfg.index_heads, H, device=dev, generator=gi) * cfg.std).bfloat16()
            if li < cfg.dense_layers:
                L['gate_up'] = randn(2 * cfg.dense_inter, H)
                L['down'] = randn(H, cfg.dense_inter)
            else:
                router = randn(cfg.experts, H)
                corr = torch.randn(cfg.experts, generator=g) * 0.01
                seed_l = seed * 1000 + li
                shared = formats.synthetic_experts(cfg.shared, H, cfg.inter, cfg.fmt, dev, seed=seed_l + 500,
                                                   std=cfg.std) if cfg.shared else None
                pending.append((li, router, corr, shared, seed_l))
            self.layers.append(L)
        if plan_fn is not None:   # e.g. the planner's auto-layout over route probabilities of these routers
            self.gpu_plan, self.popularity = plan_fn({li: (r, c) for li, r, c, _, _ in pending})
            gpu_plan, popularity = self.gpu_plan, self.popularity
            if gpu_plan is not None and (not ep or popularity is None):
                raise ValueError('gpu_plan places experts by popularity under expert parallelism')
        if ep:
            from ..parallel import dist as xdist
            from ..parallel.ep import EPComm
            env = xdist.init()
            El = cfg.experts // env.world
            if gpu_plan is not None:
                self.gpu_per_rank = ranked_pool_width(cfg.experts, env.world, gpu_plan, popularity)
                if min(gpu_plan.values()) < cfg.experts and mailbox is None:
                    raise ValueError('a CPU tier (a plan with fewer GPU experts than experts) needs a mailbox')
            else:
                self.gpu_per_rank = El if gpu_experts is None else max(1, min(El, int(gpu_experts)))
                if self.gpu_per_rank < El and mailbox is None:
                    raise ValueError('a CPU tier (gpu_experts < experts per rank) needs a mailbox')
            from .. import config
            S = config.get('XTIER_EP_PCIE_SLOTS') if pcie_slots is None else int(pcie_slots)
            if S < 0:   # a share of the CPU-tier experts one call's routes are expected to touch
                n_cpu = max(0, cfg.experts - env.world * self.gpu_per_rank)
                touched = n_cpu * (1.0 - (1.0 - cfg.top_k / cfg.experts) ** decode_tokens)
                S = math.ceil(config.get('XTIER_EP_PCIE_SHARE') * touched)
            self.pcie_slots = S if (mailbox is not None and cold is None) else 0
            self.ep = EPComm(H, cfg.inter, cfg.experts, cfg.top_k, decode_tokens, dev, timeout_s=ep_timeout_s,
                             slots_per_rank=self.gpu_per_rank + cfg.shared + self.pcie_slots, n_shared=cfg.shared,
                             stage_slots=self.pcie_slots, stage_fmt=cfg.fmt)
            self.ep_rank, self.ep_world = env.rank, env.world
        for li, router, corr, shared, seed_l in pending:
            L = self.layers[li]

            def experts_fn(ids, seed_l=seed_l):
                return formats.synthetic_experts(len(ids), H, cfg.inter, cfg.fmt, dev, seed=seed_l, std=cfg.std)

            if ep:
                L['moe'], stage = self._ep_layer(li, router, corr, shared, seed_l, engine_threads, stage)
            elif moe_factory is None:
                from ..cache.pool import TieredMoE
                L['moe'] = TieredMoE(li, router, experts_fn(list(range(cfg.experts))), cfg.top_k, shared=shared,
                                     mode=1, n_group=cfg.n_group, topk_group=cfg.topk_group, renorm=True,
                                     scale=cfg.routed_scale, corr_bias=corr, device=dev, max_tokens=16)
            else:
                L['moe'] = moe_factory(li, router, corr, experts_fn, shared)
        del stage, pending
        if ep:
            from ..parallel import dist as xdist
            torch.cuda.synchronize()
            xdist.barrier()   # every rank's pools are filled before any rank's dispatch reads them

    def _ep_layer(self, li, router, corr, shared, seed_l, threads, stage):
        """One MoE layer under expert parallelism: this rank's pool generated on the GPU, the CPU tier's experts
        generated on the GPU in chunks and copied into a pinned staging buffer for this rank's engine."""
        from ..parallel.ep import EPMoE
        cfg = self.cfg
        H, I, E = cfg.hidden, cfg.inter, cfg.experts
        if self.gpu_plan is not None:
            table, pools, cpu_ids = ep_layout_ranked(E, self.ep_world, int(self.gpu_plan[li]), self.popularity[li],
                                                     self.ep.spr, self.gpu_per_rank)
        else:
            table, pools, cpu_ids = ep_layout(E, self.ep_world, self.gpu_per_rank, seed_l, stride=self.ep.spr)
        mine = pools[self.ep_rank]
        n_sh = shared.experts if shared is not None else 0
        gp = self.gpu_per_rank
        local = empty_experts(gp + n_sh, H, I, cfg.fmt, self.device)   # the routed pool, then the shared experts
        if mine:
            synthetic_experts_by_id(formats.ExpertWeights(cfg.fmt, *[getattr(local, f)[:len(mine)] for f in
                                                                     ('w13', 'w2', 's13', 's2', 'g13', 'g2')]),
                                    mine, seed_l, cfg.std)
        for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):   # slots a ranked plan leaves empty on this rank
            getattr(local, f)[len(mine):gp].zero_()
            if n_sh:
                getattr(local, f)[gp:].copy_(getattr(shared, f))
        engine = pcie = None
        if cpu_ids and self.cold is not None:
            engine = self._cold_engine(li, cpu_ids, seed_l, threads)
            self.engines.append(engine)
        elif cpu_ids:
            from ..engine import CpuEngine
            n = len(cpu_ids)
            chunk = 16
            if stage is None:   # pinned bounce buffer of one chunk, shared by the layers
                stage = empty_experts(chunk, H, I, cfg.fmt, 'cpu', pin=True)
            # slots filled chunk by chunk (no host copy of a whole layer); the CPU tier's bytes are the same on every
            # rank (every rank's engine holds all of them)
            engine = CpuEngine(stage, threads=threads, slots=n, resident=cpu_ids, total_experts=E, fill=False)
            g13 = torch.empty(n, 2, dtype=torch.float32, device=self.device)
            g2 = torch.empty(n, dtype=torch.float32, device=self.device)
            for s in range(0, n, chunk):
                e = min(n, s + chunk)
                tmp = empty_experts(e - s, H, I, cfg.fmt, self.device)
                synthetic_experts_by_id(tmp, cpu_ids[s:e], seed_l, cfg.std)
                g13[s:e].copy_(tmp.g13.float())
                g2[s:e].copy_(tmp.g2.float())
                for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                    getattr(stage, f)[:e - s].copy_(getattr(tmp, f))
                del tmp
                for j in range(e - s):
                    engine.write_slot(s + j, stage, j)
            self.engines.append(engine)
            if self.pcie_slots:
                pcie = self._map_engine(engine, cpu_ids, g13, g2)
        moe = EPMoE(li, self.ep, router, local, cfg.top_k, shared=shared, mode=1, n_group=cfg.n_group,
                    topk_group=cfg.topk_group, renorm=True, scale=cfg.routed_scale, corr_bias=corr,
                    table=table, mailbox=self.mailbox, engine=engine, stage=pcie, shared_in_pool=True)
        return moe, stage

    def _map_engine(self, engine, cpu_ids: list, g13: torch.Tensor, g2: torch.Tensor) -> dict | None:
        """The engine's weight shards registered with CUDA and mapped for kernels (the PCIe staging reads them in
        place): the `stage` description of EPMoE, or None when the registration is refused."""
        from ..parallel.ep import map_engine
        stage, bases = map_engine(engine, cpu_ids, self.cfg.experts, g13, g2)
        self.host_maps += bases
        return stage

    def attach_bigram(self, table):
        """Adds a hashed-bigram NVMe embedding table (tables/engram.py; rows projected to the hidden size) to the
        token embeddings inside the decode graph. Attach before capturing the decode step."""
        self.bigram = table

    def _cold_engine(self, li: int, cpu_ids: list, seed_l: int, threads):
        """The CPU tier of one layer over RAM and the cold store: the first `ram_experts` of `cpu_ids` (most routed
        first) in the engine's RAM slots, the rest read from the store on demand. Rank 0 writes the layer's records
        (every expert, generated on the GPU in chunks); the other ranks wait for it and fill their RAM slots from the
        records."""
        from ..engine import CpuEngine
        from ..parallel import dist as xdist
        cfg = self.cfg
        H, I, E = cfg.hidden, cfg.inter, cfg.experts
        n_ram = len(cpu_ids) if self.ram_experts is None else max(1, min(len(cpu_ids), int(self.ram_experts)))
        ram_ids = list(cpu_ids[:n_ram])
        engine = CpuEngine(empty_experts(1, H, I, cfg.fmt, 'cpu'), threads=threads, slots=n_ram, resident=ram_ids,
                           total_experts=E, fill=False)
        nodes = engine.nodes()
        if self.ep_rank == 0:
            host = empty_experts(E, H, I, cfg.fmt, 'cpu')
            chunk = 16
            for s0 in range(0, E, chunk):
                ids = list(range(s0, min(E, s0 + chunk)))
                tmp = empty_experts(len(ids), H, I, cfg.fmt, self.device)
                synthetic_experts_by_id(tmp, ids, seed_l, cfg.std)
                for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                    getattr(host, f)[s0:s0 + len(ids)].copy_(getattr(tmp, f))
                del tmp
            self.cold.ensure_layer(li, host, nodes)
            for s, e in enumerate(ram_ids):
                engine.write_slot(s, host, e)
            del host
        xdist.barrier()
        if self.ep_rank != 0:
            self.cold.manifest = self.cold._load_manifest()
            self.cold.fill_engine(engine, li, ram_ids)
        scores = np.zeros(E, np.float32)
        scores[ram_ids] = np.linspace(1.0, 0.5, len(ram_ids), dtype=np.float32)   # initial use counts by rank
        from .. import config
        self.cold.attach(engine, li, scores, config.get('XTIER_COLD_HALF_LIFE'))
        return engine

    # ------------------------------------------------------------------ state
    def kernel_attention(self) -> bool:
        """True when decode attention runs on the MLA kernels (NVFP4 latent cache, tcgen05)."""
        cfg = self.cfg
        fits = cfg.heads == 128 and cfg.kv_lora == 512 and cfg.qk_rope == 64 and self.device.type == 'cuda'
        if cfg.attn in ('mla', 'dsa') and not fits:
            raise ValueError('the MLA kernels need 128 heads, kv_lora 512 and qk_rope 64')
        return cfg.attn in ('mla', 'dsa') or (cfg.attn == 'auto' and fits)

    def alloc_state(self, batch: int, max_len: int, bf16_cache: bool = False) -> dict:
        """KV state of `batch` sequences of up to max_len tokens. The BF16 latent cache (the plain PyTorch decode, and
        the prefill of a continuation) is kept when the kernels do not attend or bf16_cache is set."""
        cfg = self.cfg
        kern = self.kernel_attention()
        bf16_cache = bf16_cache or self.keep_bf16_cache
        st = dict(batch=batch, max_len=max_len,
                  lengths=torch.zeros(batch, dtype=torch.int32, device=self.device))
        if bf16_cache or not kern:
            st['cache'] = [torch.zeros(batch, max_len, cfg.kv_lora + cfg.qk_rope, dtype=torch.bfloat16,
                                       device=self.device) for _ in self.layers]
        if kern:
            from ..attention.mla import FLASH_BLOCK, FlashWorkspace, LatentCache, flash_splits
            st['latent'] = [LatentCache(batch, max_len, self.device) for _ in self.layers]
            nsel = cfg.index_topk if cfg.attn == 'dsa' else (max_len + FLASH_BLOCK - 1) // FLASH_BLOCK * FLASH_BLOCK
            st['nsel'] = nsel
            st['mla_splits'] = flash_splits(batch, nsel)
            st['mla_ws'] = FlashWorkspace(batch, st['mla_splits'], self.device)
            if cfg.attn == 'dsa':
                from ..attention.dsa import IndexCache
                st['index'] = [IndexCache(batch, max_len, self.device) for _ in self.layers]
        return st

    def fill_synthetic_cache(self, st: dict, length: int, seed: int = 0, first_request: int = 0):
        """Writes random latent rows (N(0, 1) latent values, rotary keys) for positions [0, length) of every row
        of every layer and sets the lengths: the state a `length`-token prompt leaves, for decode benchmarks whose
        prompts are random ids (their prefill is measured on its own). Row b holds request first_request + b, whose
        rows are drawn from (seed, layer, request) alone, so a request's cache is the same on any rank."""
        cfg = self.cfg
        B = st['batch']
        pos = torch.arange(length, device=self.device)
        for li in range(len(self.layers)):
            for b in range(B):
                g = torch.Generator(device=self.device).manual_seed((seed * 1009 + li) * 100003 + first_request + b)
                lat = torch.randn(length, cfg.kv_lora + cfg.qk_rope, device=self.device, generator=g).bfloat16()
                sl = b * st['max_len'] + pos
                if 'latent' in st:
                    st['latent'][li].write(lat, sl)
                if 'cache' in st:
                    st['cache'][li].view(-1, cfg.kv_lora + cfg.qk_rope)[sl] = lat
        st['lengths'].fill_(length)

    # ------------------------------------------------------------------ blocks
    def _mla_project(self, L, h, pos):
        """Queries [T, heads, nope+rope] and the latent cache rows [T, kv_lora + rope] of h [T, H]."""
        cfg = self.cfg
        T = h.shape[0]
        qkv = ops.linear(h, L['qkv_a'])
        q_a = ops.rmsnorm(qkv[:, :cfg.q_lora].contiguous(), L['q_a_norm'], cfg.eps)
        self._q_a = q_a
        q = ops.linear(q_a, L['q_b']).view(T, cfg.heads, cfg.qk_nope + cfg.qk_rope)
        q_pe = _rope(q[..., cfg.qk_nope:].transpose(0, 1), pos, cfg.rope_theta).transpose(0, 1)
        q = torch.cat([q[..., :cfg.qk_nope], q_pe], -1)
        kv = qkv[:, cfg.q_lora:]
        c = ops.rmsnorm(kv[:, :cfg.kv_lora].contiguous(), L['kv_a_norm'], cfg.eps)
        k_pe = _rope(kv[:, cfg.kv_lora:], pos, cfg.rope_theta)
        return q, torch.cat([c, k_pe], -1)

    def _mla_decode(self, L, q, cache, lengths):
        """Absorbed MLA over the latent cache (plain PyTorch, FP32): q [B, heads, nope+rope] -> [B, heads * v]."""
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
            out[b] = torch.einsum('hl,hlv->hv', o_lat, L['w_uvT'].float())
        return out.to(torch.bfloat16).view(B, -1)

    def _mla_decode_kernel(self, li, L, st, q, h, q_a, rows, lens):
        """Absorbed MLA decode on the tensor cores over the NVFP4 latent cache: every cached position (dense) or the
        DSA indexer's top-k (sparse). q [B, heads, nope+rope] (rotated) -> [B, heads * v]."""
        from ..attention import dsa
        from ..attention.mla import mla_flash
        cfg = self.cfg
        B = q.shape[0]
        qf = torch.empty(B, cfg.heads, cfg.kv_lora + cfg.qk_rope, dtype=torch.bfloat16, device=q.device)
        ops.head_gemm(q.contiguous(), L['w_uk'], qf)
        qf[..., cfg.kv_lora:] = q[..., cfg.qk_nope:]
        lc = st['latent'][li]
        if cfg.attn == 'dsa':
            qi = ops.linear(q_a, L['idx_q']).view(B, cfg.index_heads, cfg.index_dim)
            w = ops.linear(h, L['idx_w']).float() * cfg.index_heads ** -0.5
            scores = dsa.index_scores(qi, w, st['index'][li], rows, lens)
            idx = dsa.select_slots(scores, rows, cfg.index_topk, st['max_len'])
        else:
            nsel = st['nsel']
            pos = torch.arange(nsel, device=q.device, dtype=torch.int32)[None]
            idx = torch.where(pos < lens[:, None], pos + rows[:, None] * st['max_len'], -1).int()
        o_lat = mla_flash(qf, idx, lc, 1.0 / math.sqrt(cfg.qk_nope + cfg.qk_rope), st['mla_splits'], st['mla_ws'])
        out = torch.empty(B, cfg.heads, cfg.v_head, dtype=torch.bfloat16, device=q.device)
        ops.head_gemm(o_lat, L['w_uvT'], out)
        return out.reshape(B, -1)

    def _mla_prefill(self, L, q, lat, start):
        """Expanded MLA (causal) for one sequence: q [T, h, nope+rope], lat [start+T, lora+rope] -> [T, h*v]."""
        cfg = self.cfg
        T = q.shape[0]
        c, k_pe = lat[:, :cfg.kv_lora], lat[:, cfg.kv_lora:]
        k_nope = torch.einsum('nl,hdl->hnd', c.float(), L['w_uk'].float()).to(torch.bfloat16)   # [h, n, nope]
        v = torch.einsum('nl,hld->hnd', c.float(), L['w_uvT'].float()).to(torch.bfloat16)       # [h, n, v]
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
        a = torch.empty(h.shape[0], g.shape[-1] // 2, dtype=torch.bfloat16, device=h.device)
        ops.silu_mul(g, a)
        ops.linear(a, L['down'], out=out)

    # ------------------------------------------------------------------ forward
    def forward(self, st: dict, tokens: torch.Tensor, rows: torch.Tensor, pos: torch.Tensor, decode: bool,
                all_logits: bool = False):
        """tokens [T] (decode: one per row), rows [T] cache row, pos [T] position. Returns logits of the last token
        (prefill) or of every token (decode, or all_logits)."""
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
            if 'cache' in st:
                st['cache'][li][rows.long(), pos.long()] = lat
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
                    a = self._mla_decode(L, q, st['cache'][li][rows.long()], lens)
            else:
                start = int(pos[0])
                if start and 'cache' not in st:
                    raise ValueError('a continuation prefill needs the BF16 latent cache (alloc_state(bf16_cache))')
                prefix = st['cache'][li][int(rows[0]), :start + T] if 'cache' in st else lat
                a = self._mla_prefill(L, q, prefix, start)
            o = ops.linear(a.contiguous(), L['o'])
            ops.add_rmsnorm(o, residual, L['post_norm'], h, cfg.eps)
            if 'moe' in L:
                L['moe'].forward(h, out=blk)
            else:
                self._mlp(L, h, blk)
        ops.add_rmsnorm(blk, residual, self.final_norm, h, cfg.eps)
        x = h if decode or all_logits else h[-1:]
        return ops.linear(x.contiguous(), self.lm_head)

    def prefill(self, st, tokens, row: int = 0, start: int = 0, return_logits: bool = False,
                all_logits: bool = False):
        """Prompt `tokens` [T] of cache row `row` at positions start.. (start > 0 continues a cached prefix, which
        needs the BF16 latent cache). Returns the greedy next token [1]; with return_logits also the last position's
        logits [V], with all_logits every position's [T, V]."""
        T = tokens.shape[0]
        tokens = tokens.to(self.device)
        # expert parallelism: the exchange buffers (and the CPU tier's mailbox) hold ep.T tokens, so a longer prompt
        # goes through in chunks, each a continuation of the cached prefix
        step = self.ep.T if self.ep is not None else T
        if step < T and 'cache' not in st:
            raise ValueError(f'a prompt over {step} tokens prefills in chunks, which needs the BF16 latent cache '
                             '(alloc_state(bf16_cache=True), or keep_bf16_cache = True before the Generator)')
        parts = []
        for a in range(0, T, step):
            b = min(T, a + step)
            pos = torch.arange(start + a, start + b, dtype=torch.int32, device=self.device)
            rows = torch.full((b - a,), row, dtype=torch.int32, device=self.device)
            parts.append(self.forward(st, tokens[a:b], rows, pos, decode=False, all_logits=all_logits))
        logits = torch.cat(parts) if all_logits else parts[-1]
        st['lengths'][row] = start + T
        nxt = logits[-1:].argmax(-1)
        if all_logits:
            return nxt, logits
        return (nxt, logits[-1]) if return_logits else nxt

    def decode_tokens_step(self, st, tokens, rows):
        """Eager decode of one token per row (plain forward); returns the greedy next tokens."""
        pos = st['lengths'][rows.long()].clone()
        logits = self.forward(st, tokens, rows, pos, decode=True)
        st['lengths'][rows.long()] += 1
        return logits.argmax(-1)

    # ------------------------------------------------------------------ batched decode step (graph capturable)
    def decode_buffers(self, batch: int) -> dict:
        cfg = self.cfg
        dev = self.device
        H = cfg.hidden
        B = batch
        e = lambda *s: torch.empty(*s, dtype=torch.bfloat16, device=dev)
        return dict(
            tokens=torch.zeros(B, dtype=torch.int64, device=dev),
            prev=torch.zeros(B, dtype=torch.int64, device=dev),   # the previous input (hashed bigram rows)
            pos=torch.zeros(B, dtype=torch.int32, device=dev),
            rows=torch.arange(B, dtype=torch.int32, device=dev),
            slot=torch.zeros(B, dtype=torch.int64, device=dev),
            lens=torch.zeros(B, dtype=torch.int32, device=dev),
            residual=e(B, H), h=e(B, H), blk=e(B, H), o=e(B, H),
            qkv_a=e(B, cfg.q_lora + cfg.kv_lora + cfg.qk_rope), q_a=e(B, cfg.q_lora),
            q=e(B, cfg.heads, cfg.qk_nope + cfg.qk_rope), qf=e(B, cfg.heads, cfg.kv_lora + cfg.qk_rope),
            o_lat=e(B, cfg.heads, cfg.kv_lora), a=e(B, cfg.heads, cfg.v_head),
            gu=e(B, 2 * cfg.dense_inter), act=e(B, cfg.dense_inter),
            logits=e(B, cfg.vocab), next=torch.zeros(B, dtype=torch.int64, device=dev),
        )

    def decode_step(self, st: dict, buf: dict):
        """One token per row: reads buf['tokens'], buf['pos'] (device), writes buf['next'] (greedy). Every op is a
        kernel of this package; nothing synchronizes with the host, so the step captures into one CUDA graph."""
        cfg = self.cfg
        if 'latent' not in st:
            raise ValueError('the batched decode step runs on the MLA kernels (NVFP4 latent cache)')
        if cfg.attn == 'dsa':
            raise ValueError('the batched decode step attends densely (attn="mla")')
        B = buf['tokens'].shape[0]
        ws = st['mla_ws']
        nsel = st['nsel']
        scale = 1.0 / math.sqrt(cfg.qk_nope + cfg.qk_rope)
        # per step: cache slots of the new tokens and the dense key list of every row (the same for all layers)
        if 'idx' not in buf or buf['idx'].shape[1] != nsel:
            buf['idx'] = torch.empty(B, nsel, dtype=torch.int32, device=self.device)
            buf['ar'] = torch.arange(nsel, dtype=torch.int32, device=self.device)[None].expand(B, nsel).contiguous()
            buf['rowbase'] = (buf['rows'][:, None] * st['max_len']).contiguous()
            buf['minus1'] = torch.full((B, nsel), -1, dtype=torch.int32, device=self.device)
        torch.add(buf['rows'].long() * st['max_len'], buf['pos'].long(), out=buf['slot'])
        torch.add(buf['pos'], 1, out=buf['lens'])
        torch.where(buf['ar'] < buf['lens'][:, None], buf['ar'] + buf['rowbase'], buf['minus1'], out=buf['idx'])
        torch.index_select(self.embed, 0, buf['tokens'], out=buf['residual'])
        if self.bigram is not None:   # NVMe hashed-bigram rows, looked up inside the graph
            self.bigram.add_decode(buf['residual'], buf['prev'], buf['tokens'])
        for li, L in enumerate(self.layers):
            if li == 0:
                ops.add_rmsnorm(buf['residual'], None, L['in_norm'], buf['h'], cfg.eps)
            else:
                ops.add_rmsnorm(buf['blk'], buf['residual'], L['in_norm'], buf['h'], cfg.eps)
            ops.linear(buf['h'], L['qkv_a'], out=buf['qkv_a'])
            lc = st['latent'][li]
            ops.mla_prep(buf['qkv_a'], cfg.q_lora, L['q_a_norm'], L['kv_a_norm'], buf['pos'], buf['slot'], cfg.eps,
                         cfg.rope_theta, buf['q_a'], lc.codes, lc.scales, lc.rope)
            ops.linear(buf['q_a'], L['q_b'], out=buf['q'].view(B, -1))
            ops.head_gemm(buf['q'], L['w_uk'], buf['qf'], buf['pos'], cfg.qk_nope, cfg.kv_lora, cfg.qk_rope,
                          cfg.rope_theta)
            torch.ops.xtier.mla_flash(buf['qf'], buf['idx'], lc.codes, lc.scales, lc.rope, ws.part_o, ws.part_ml,
                                      buf['o_lat'], float(scale), st['mla_splits'], ws.err)
            ops.head_gemm(buf['o_lat'], L['w_uvT'], buf['a'])
            ops.linear(buf['a'].view(B, -1), L['o'], out=buf['o'])
            ops.add_rmsnorm(buf['o'], buf['residual'], L['post_norm'], buf['h'], cfg.eps)
            if 'moe' in L:
                L['moe'].forward(buf['h'], out=buf['blk'])
            else:
                ops.linear(buf['h'], L['gate_up'], out=buf['gu'])
                ops.silu_mul(buf['gu'], buf['act'])
                ops.linear(buf['act'], L['down'], out=buf['blk'])
        ops.add_rmsnorm(buf['blk'], buf['residual'], self.final_norm, buf['h'], cfg.eps)
        ops.linear(buf['h'], self.lm_head, out=buf['logits'])
        torch.argmax(buf['logits'], dim=-1, out=buf['next'])
        if self.bigram is not None:
            buf['prev'].copy_(buf['tokens'])
        return buf['next']

    def check(self, st: dict | None = None):
        """Raises when a bounded wait of the last steps ran out (EP exchange, mailbox, MLA of state `st`)."""
        code = int(st['mla_ws'].err.item()) if st is not None and 'mla_ws' in st else 0
        if code == 2:
            raise RuntimeError('MLA attention: a cache slot out of range (XTIER_DEBUG_BOUNDS)')
        if code:
            raise RuntimeError('MLA attention: a bounded wait ran out')
        if self.ep is not None:
            self.ep.check()
        if self.mailbox is not None:
            self.mailbox.check()
        if self.bigram is not None:
            self.bigram.check()

    def close(self):
        if self.host_maps:
            from ..parallel.ep import unmap_engine
            torch.cuda.synchronize()
            unmap_engine(self.host_maps)
            self.host_maps = []
        for e in self.engines:
            e.close()
        self.engines = []
        if self.ep is not None:
            self.ep.close()
            self.ep = None
