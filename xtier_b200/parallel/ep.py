"""Expert-parallel MoE over NVLink peer memory, and its NCCL baseline.

Expert e lives on rank e // (E / W). Each rank routes its own tokens, then one op (`torch.ops.xtier.ep_moe`, four
kernels, csrc/cuda/moe_decode.cu) moves every route's token row into the owner's receive slot with in-kernel peer
stores, computes the received routes on the owner's FP4 experts (W4A16, like the hot-slot decode kernels), stores each
weighted result straight back into the source rank's return buffer from the down projection's epilogue, and sums
each token's routes in route order. Flags carry a per-call epoch, so a CUDA graph replays the exchange with no host
work, and every wait is bounded (a timeout sets the error word and the call's output lacks the missing parts).

Tiers: when the GPUs of the group cannot hold every expert, each owner keeps only part of its range in its GPU pool
(`table`: expert -> owner * slots_per_rank + pool slot, or -1) and the others live in a CPU tier. The router then
marks those routes -1 and hands them to this rank's mailbox (the CPU engine of every rank holds all CPU-tier experts,
so such a route never leaves its source); the dispatch skips them and the combine adds the engine's rows after a
bounded wait. With one rank this is the single-GPU tiered MoE on the EP kernels.

`EPComm` is shared by all MoE layers of a model (the layers run one after another): one symmetric buffer, the epoch
state and the scratch. `nccl_ep_moe()` is the baseline the fused path is measured against: all_to_all_single of the
routed rows and metadata, the same expert kernels locally, all_to_all_single back.

(The reference refuses EP, xtier/backend/method.py:105; its second-GPU pool relays through host memory.)
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..formats import NVFP4, ExpertWeights
from . import dist as xdist
from .symm import SymmetricBuffer


class EPComm:
    def __init__(self, hidden: int, inter: int, experts: int, top_k: int, max_tokens: int, device=None,
                 timeout_s: float = 10.0, slots_per_rank: int | None = None, n_shared: int = 0,
                 stage_slots: int = 0, stage_fmt: str = NVFP4):
        """slots_per_rank: pool slots of every rank (routed experts in HBM plus the shared experts plus the staging
        slots; default every owned expert plus the shared ones). n_shared: shared experts per token, computed as routes
        to the local pool's slots after the routed ones. stage_slots: PCIe staging slots (the last local slots), shared
        by the layers: CPU-tier experts the router hands to the GPU, copied from the CPU engine's host memory each
        call (`EPMoE(stage=...)`)."""
        env = xdist.get()
        self.W, self.rank = env.world, env.rank
        self.H, self.I, self.E, self.T = hidden, inter, experts, max_tokens
        self.k = top_k + n_shared     # routes per token on the wire (routed + shared)
        self.n_shared = n_shared
        if experts % self.W:
            raise ValueError(f'{experts} experts do not split over {self.W} ranks')
        self.El = experts // self.W
        self.spr = slots_per_rank or (self.El + n_shared)
        top_k = self.k
        self.R = max_tokens * top_k   # worst case: every route of a source goes to one rank
        self.device = device or env.device
        W, R, H = self.W, self.R, hidden
        off = 0
        offs = []

        def region(nbytes):
            nonlocal off
            offs.append(off)
            off += (nbytes + 255) // 256 * 256

        region(W * R * H * 2)          # rx
        region(W * R * 16)             # meta
        region(W * 128)                # cnt
        region(W * 128)                # flag
        region(max_tokens * top_k * H * 4)   # ret
        region(W * 128)                # rflag
        self.offsets = offs
        self.buf = SymmetricBuffer(off, self.device)
        self.state = torch.zeros(64, dtype=torch.int32, device=self.device)
        self.mid = torch.empty(W * R * inter, dtype=torch.float16, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.timeout_s = timeout_s
        self.S = int(stage_slots)
        if self.S:
            bs = 16 if stage_fmt == NVFP4 else 32
            u8 = lambda *shape: torch.zeros(*shape, dtype=torch.uint8, device=self.device)   # noqa: E731
            self.st_w13, self.st_s13 = u8(self.S, 2 * inter, hidden // 2), u8(self.S, 2 * inter, hidden // bs)
            self.st_w2, self.st_s2 = u8(self.S, hidden, inter // 2), u8(self.S, hidden, inter // bs)
            self.st_g13 = torch.ones(self.S, 2, dtype=torch.float32, device=self.device)
            self.st_g2 = torch.ones(self.S, dtype=torch.float32, device=self.device)
            self.claim = torch.full((experts,), -1, dtype=torch.int32, device=self.device)
            self.claim_list = torch.zeros(experts, dtype=torch.int32, device=self.device)
            self.claim_count = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.stage_done = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.stage_chunks = max(4, 148 * 8 // self.S)

    def check(self):
        if int(self.err.item()):
            self.err.zero_()
            raise RuntimeError('xtier_b200 EP: a wait for a peer rank timed out')

    def close(self):
        self.buf.close()


class EPMoE:
    """One MoE layer's routed experts split over the ranks; the shared experts are routes to the last slots of the
    local pool, so they stream through the same kernels (one weight pass for all of a rank's tokens).

    `local`: this rank's GPU pool of routed experts (all of its El experts in id order, or with `table` the pool
    slots' experts). `table` (int32 [E], optional): expert -> owner * slots_per_rank + pool slot, -1 for the CPU tier,
    whose routes go through `mailbox` to `engine` (this rank's CPU engine of every CPU-tier expert).

    `stage` (optional, with the exchange's staging slots): the CPU engine's weight shards mapped for the GPU --
    dict(cold_index = int32 [E] engine slot of each CPU-tier expert or -1, bases = device address of each node's shard,
    stride, piece_off, piece_bytes (`CpuEngine.shard`), src_g13 [slots, 2] / src_g2 [slots] global scales by engine
    slot). The router then hands up to `comm.S` of the CPU-tier experts its tokens chose to the GPU, which copies them
    over PCIe into the staging slots (`ep_stage`) and computes their routes while the engine computes the others."""

    def __init__(self, layer: int, comm: EPComm, router_w: torch.Tensor, local: ExpertWeights, top_k: int,
                 shared: ExpertWeights | None = None, mode: int = 0, n_group: int = 1, topk_group: int = 1,
                 renorm: bool = True, scale: float = 1.0, router_bias=None, corr_bias=None, table=None,
                 mailbox=None, engine=None, stage: dict | None = None, shared_in_pool: bool = False):
        """shared_in_pool: `local` already ends with the shared experts' slots (`shared` then only gives their
        count): no concatenated copy of the pool, whose transient second copy can be more than the HBM left."""
        self.comm = comm
        self.layer = layer
        self.k = top_k
        n_sh = 0 if shared is None else shared.experts
        if n_sh != comm.n_shared or top_k + n_sh != comm.k:
            raise ValueError('EP MoE: routes per token differ from the exchange buffers (top_k / n_shared)')
        nl = local.experts - (n_sh if shared_in_pool else 0)
        if nl + n_sh + comm.S != comm.spr:
            raise ValueError(f'EP MoE: {nl} pool experts + {n_sh} shared + {comm.S} staging != {comm.spr} slots per '
                             'rank')
        parts = [local] + ([shared] if shared is not None and not shared_in_pool else [])
        fields = ('w13', 'w2', 's13', 's2', 'g13', 'g2')
        self.local = ExpertWeights(local.fmt, *[(torch.cat([getattr(q, f).to(comm.device) for q in parts])
                                                 if len(parts) > 1 else getattr(local, f).to(comm.device)).contiguous()
                                                for f in fields])
        self.local.g13 = self.local.g13.float().contiguous()
        self.local.g2 = self.local.g2.float().contiguous()
        self.fmt_code = 0 if local.fmt == NVFP4 else 1
        if table is None:   # every owned expert in its owner's pool, in id order
            if nl != comm.El:
                raise ValueError('EP MoE: without a table the pool holds every owned expert')
            e = torch.arange(comm.E, dtype=torch.int32)
            table = (e // comm.El) * comm.spr + e % comm.El
            tiered = False
        else:
            tiered = True
        self.table = torch.as_tensor(table, dtype=torch.int32).to(comm.device)
        self.shared_slots = (torch.arange(nl, nl + n_sh, dtype=torch.int32, device=comm.device) + comm.rank * comm.spr
                             if n_sh else None)
        self.mailbox = mailbox if (engine is not None and tiered) else None
        if self.mailbox is not None:
            self.mailbox.register(layer, engine)
        self.engine = engine
        self.stage_base = nl + n_sh
        self.stage = None
        route_stage = None
        if stage is not None and comm.S and self.mailbox is not None:
            self.stage = dict(stage, cold_index=torch.as_tensor(stage['cold_index'], dtype=torch.int32).to(comm.device),
                              src_g13=stage['src_g13'].to(comm.device, torch.float32).contiguous(),
                              src_g2=stage['src_g2'].to(comm.device, torch.float32).contiguous(),
                              bases=[int(b) for b in stage['bases']], piece_off=[int(v) for v in stage['piece_off']],
                              piece_bytes=[int(v) for v in stage['piece_bytes']], stride=int(stage['stride']))
            route_stage = (self.stage['cold_index'], comm.claim, comm.claim_list, comm.claim_count, comm.S,
                           comm.rank * comm.spr + self.stage_base)
        self.router = _Router(router_w, comm.E, top_k, mode, n_group, topk_group, renorm, scale, router_bias,
                              corr_bias, comm.device, comm.T, table=self.table, layer=layer, mailbox=self.mailbox,
                              shared_slots=self.shared_slots, stage=route_stage)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, add: torch.Tensor | None = None):
        c = self.comm
        T = x.shape[0]
        if T > c.T:
            raise ValueError(f'EP MoE: {T} tokens exceed the {c.T} per rank the exchange buffers were sized for')
        out = torch.empty_like(x) if out is None else out
        ids, w = self.router(x)
        st = self.stage
        if st is not None:   # the claimed CPU-tier experts over PCIe into the staging slots
            torch.ops.xtier.ep_stage(c.claim_list, c.claim, c.claim_count, c.stage_done, st['cold_index'],
                                     st['bases'], st['stride'], st['piece_off'], st['piece_bytes'], c.st_w13,
                                     c.st_s13, c.st_w2, c.st_s2, c.st_g13, c.st_g2, st['src_g13'], st['src_g2'], c.I,
                                     c.H, self.fmt_code, c.stage_chunks)
        staged = (c.st_w13, c.st_s13, c.st_w2, c.st_s2, c.st_g13, c.st_g2, self.stage_base) if st is not None else ()
        torch.ops.xtier.ep_moe(x, ids, w, c.buf.peer_table, c.state, c.mid, self.local.w13, self.local.s13,
                               self.local.g13, self.local.w2, self.local.s2, self.local.g2, add, out, c.err, c.W,
                               c.rank, c.E, self.fmt_code, c.R, c.offsets, c.timeout_s, 0xF,
                               self.router.slots[:T], c.spr,
                               self.mailbox.handle if self.mailbox is not None else 0, *staged)
        return out


class _Router:
    def __init__(self, router_w, E, k, mode, n_group, topk_group, renorm, scale, bias, corr, device, max_tokens,
                 table=None, layer: int = 0, mailbox=None, shared_slots=None, stage=None):
        self.table, self.layer, self.mailbox, self.shared_slots = table, layer, mailbox, shared_slots
        self.stage = stage   # (cold_index, claim, claim_list, claim_count, stage_max, stage_slot0) or None
        kk = k + (0 if shared_slots is None else shared_slots.numel())
        self.w = router_w.to(device, torch.bfloat16).contiguous()
        self.E, self.k = E, k
        self.mode, self.n_group, self.topk_group, self.renorm, self.scale = mode, n_group, topk_group, renorm, scale
        self.bias = None if bias is None else bias.to(device, torch.float32).contiguous()
        self.corr = None if corr is None else corr.to(device, torch.float32).contiguous()
        self.ids = torch.empty(max_tokens, kk, dtype=torch.int32, device=device)
        self.wt = torch.empty(max_tokens, kk, dtype=torch.float32, device=device)
        self.slots = torch.empty(max_tokens, kk, dtype=torch.int32, device=device)
        self.ws_logits = torch.empty(max_tokens, E, dtype=torch.float32, device=device)
        self.ws_count = torch.zeros(max_tokens, dtype=torch.int32, device=device)

    def __call__(self, x):
        T = x.shape[0]
        ops.moe_route(x, self.w, self.bias, self.corr, self.table, self.shared_slots, self.ids[:T], self.wt[:T],
                      self.slots[:T],
                      self.ws_logits, self.ws_count, self.k, self.mode, self.n_group, self.topk_group, self.renorm,
                      self.scale, self.layer, self.mailbox.handle if self.mailbox is not None else 0,
                      **(dict(zip(('cold_index', 'claim', 'claim_list', 'claim_count', 'stage_max', 'stage_slot0'),
                                  self.stage)) if self.stage is not None else {}))
        return self.ids[:T], self.wt[:T]


def map_engine(engine, expert_ids: list, E: int, g13: torch.Tensor, g2: torch.Tensor):
    """Registers the CPU engine's weight shards with CUDA (page-locked, mapped) so that kernels read its slots in place
    over PCIe. Returns (the `stage` description EPMoE takes -- engine slot s holds expert_ids[s], whose global scales
    are g13[s] / g2[s] --, the registered host addresses for `unmap_engine`), or (None, []) with a warning when CUDA
    refuses the registration."""
    import ctypes as C
    import logging
    L = ops.cdll()
    L.xt_host_register_mapped.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p]
    bases, regs, sh = [], [], None
    for node in range(engine.nodes()):
        sh = engine.shard(node)
        dev = C.c_void_p()
        rc = L.xt_host_register_mapped(C.c_void_p(sh['base']), C.c_size_t(sh['bytes']), C.byref(dev))
        if rc != 0:
            logging.getLogger('xtier_b200').warning(f'PCIe staging off: cudaHostRegister of an engine shard refused '
                                                    f'(error {rc})')
            unmap_engine(regs)
            return None, []
        regs.append(sh['base'])
        bases.append(dev.value)
    # the staging copy lays node n's rows of each piece at n * piece bytes: the engine must split rows evenly
    N, H, I = len(bases), engine.H, engine.I
    bs = 16 if engine.fmt == NVFP4 else 32
    want = [I // N * (H // 2)] * 2 + [I // N * (H // bs)] * 2 + [H // N * (I // 2), H // N * (I // bs)]
    aligned = all(v % 16 == 0 for v in list(sh['piece_off']) + list(sh['piece_bytes']) + [sh['stride']] + bases)
    if list(sh['piece_bytes']) != want or I % N or H % N or not aligned:
        logging.getLogger('xtier_b200').warning('PCIe staging off: the engine shards do not split the rows evenly')
        unmap_engine(regs)
        return None, []
    idx = torch.full((E,), -1, dtype=torch.int32)
    idx[torch.as_tensor(list(expert_ids), dtype=torch.long)] = torch.arange(len(expert_ids), dtype=torch.int32)
    return dict(cold_index=idx, bases=bases, stride=sh['stride'], piece_off=sh['piece_off'],
                piece_bytes=sh['piece_bytes'], src_g13=g13, src_g2=g2), regs


def unmap_engine(regs: list):
    """Unregisters what `map_engine` registered (before the engine frees its shards)."""
    import ctypes as C
    if not regs:
        return
    L = ops.cdll()
    L.xt_host_unregister.argtypes = [C.c_void_p]
    for base in regs:
        L.xt_host_unregister(C.c_void_p(base))


def nccl_ep_moe(x, ids, w, local: ExpertWeights, E: int, group=None):
    """Baseline: NCCL all-to-all of the routed rows, local expert compute, all-to-all back, route-ordered sum.
    Returns bf16 [T, H]. Not graph-captured (data-dependent split sizes)."""
    env = xdist.get()
    W, T, k = env.world, x.shape[0], ids.shape[1]
    El = E // W
    dest = (ids // El).flatten()
    order = torch.argsort(dest * (T * k) + torch.arange(T * k, device=x.device))   # by destination, route order
    send_counts = torch.bincount(dest, minlength=W)
    recv_counts = torch.empty_like(send_counts)
    a2a = dist.all_to_all_single if W > 1 else (lambda o, i, *a, **k: o.copy_(i))
    a2a(recv_counts, send_counts, group=group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    rows = x.repeat_interleave(k, 0)[order]
    meta = torch.stack([(ids.flatten() % El)[order], w.flatten()[order].view(torch.int32)], 1).contiguous()
    r_rows = torch.empty(sum(rc), x.shape[1], dtype=x.dtype, device=x.device)
    r_meta = torch.empty(sum(rc), 2, dtype=torch.int32, device=x.device)
    a2a(r_rows, rows, rc, sc, group=group)
    a2a(r_meta, meta, rc, sc, group=group)
    n = r_rows.shape[0]
    y = torch.empty(n, x.shape[1], dtype=torch.bfloat16, device=x.device)
    if n:
        slots = r_meta[:, 0:1].contiguous()
        wt = r_meta[:, 1:2].contiguous().view(torch.float32)
        mid = torch.empty(n, local.inter, dtype=torch.float16, device=x.device)
        fmt = 0 if local.fmt == NVFP4 else 1
        ops.moe_gate_up(r_rows, slots, local.w13, local.s13, local.g13, mid, fmt)
        ops.moe_down(mid, slots, wt, local.w2, local.s2, local.g2, None, y, fmt=fmt)
    back = torch.empty(T * k, x.shape[1], dtype=torch.bfloat16, device=x.device)
    a2a(back, y, sc, rc, group=group)
    res = torch.empty_like(back)
    res[order] = back
    return res.view(T, k, -1).float().sum(1).to(torch.bfloat16)
