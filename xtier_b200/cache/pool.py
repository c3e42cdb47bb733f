"""Tiered MoE layer: GPU hot-expert slots + CPU engine for the rest, in the same call.

`TieredMoE` owns one layer's router, a GPU slot pool holding `len(hot)` routed experts (plus the shared experts, which
always live on the GPU) in the checkpoint's FP4 layout, the residency table expert -> slot (-1: CPU), and a CPU engine
holding every routed expert. A decode call (<= 16 tokens) runs three kernels (csrc/cuda/moe_decode.cu): route+split
(publishing the CPU part to the mailbox), gate/up on the hot slots, down + route-ordered combine with the CPU result.
Prefill calls (more tokens) run the GPU part while a host thread runs the CPU engine on the other routes
(hybrid prefill), then add the two.

The residency table is device memory read at replay time, so swapping a slot's expert needs no graph recapture:
`swap()` unpublishes the victim, copies the new expert's bytes into the slot and publishes it, all on the compute
stream, so a replay never reads a slot in flight.

Reference parity: xtier/cache/pool.py:1-43 (decode split, residency tables, adaptive swaps), :418-589 (LayerPool),
xtier/cache/prefill.py:154 (hybrid prefill), xtier/backend/method.py:320-421 (per-call dispatch).
"""
from __future__ import annotations

import threading

import torch

from .. import config, ops
from ..formats import NVFP4, ExpertWeights

MAX_DECODE_TOKENS = 16
_STAGING: dict = {}   # (cold experts, H, I, fmt, device) -> staging ExpertWeights shared by the layers
_PREFILL_BUFS: dict = {}   # (kk, E, I, H, device) -> prefill route buffers shared by the layers
_BUF_NAMES = ('ids', 'w', 'slots', 'mid', 'ws_logits', 'ws_count', 'gpu_part')
_EMPTY_POOLS: dict = {}   # (H, I, fmt, device) -> one all-zero slot: the launch operand of layers without GPU slots


def _pinned(ew: ExpertWeights) -> ExpertWeights:
    """Page-locked copy of a small host ExpertWeights (the source of a copy that must not block the host)."""
    if not torch.cuda.is_available() or ew.w13.is_cuda:
        return ew
    return ExpertWeights(ew.fmt, *[getattr(ew, f).contiguous().pin_memory()
                                   for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2')])


class TieredMoE:
    def __init__(self, layer: int, router_w: torch.Tensor, experts: ExpertWeights, top_k: int,
                 hot: list[int] | None = None, shared: ExpertWeights | None = None, mode: int = 0, n_group: int = 1,
                 topk_group: int = 1, renorm: bool = True, scale: float = 1.0, router_bias: torch.Tensor | None = None,
                 corr_bias: torch.Tensor | None = None, limit: float = 0.0, mailbox=None, engine=None,
                 device='cuda', max_tokens: int = MAX_DECODE_TOKENS, host_experts: ExpertWeights | None = None,
                 pool_storage: dict | None = None):
        self.layer = layer
        self.device = torch.device(device)
        self.E, self.H, self.I = experts.experts, experts.hidden, experts.inter
        self.fmt = experts.fmt
        self.fmt_code = 0 if self.fmt == NVFP4 else 1
        self.k = top_k
        self.mode, self.n_group, self.topk_group, self.renorm, self.scale = mode, n_group, topk_group, renorm, scale
        self.limit = limit
        self.router_w = router_w.to(self.device, torch.bfloat16).contiguous()
        self.router_bias = None if router_bias is None else router_bias.to(self.device, torch.float32).contiguous()
        self.corr_bias = None if corr_bias is None else corr_bias.to(self.device, torch.float32).contiguous()
        self.hot = list(range(self.E)) if hot is None else list(hot)
        self.n_shared = 0 if shared is None else shared.experts
        S = len(self.hot)
        # host copy of every routed expert: the source of swaps (None: the residency is fixed)
        self.host = host_experts
        src = experts
        parts = []
        if S:
            parts.append(src.select(torch.tensor(self.hot, device=src.w13.device)).to(self.device))
        if shared is not None:
            parts.append(shared.to(self.device))
        if parts:
            fields = ('w13', 'w2', 's13', 's2', 'g13', 'g2')
            if pool_storage is not None:   # preallocated (e.g. symmetric peer memory): copy the slots in
                for f in fields:
                    o = 0
                    for part in parts:
                        src = getattr(part, f)
                        pool_storage[f][o:o + src.shape[0]].copy_(src)
                        o += src.shape[0]
                self.pool = ExpertWeights(self.fmt, *[pool_storage[f] for f in fields])
            else:
                self.pool = ExpertWeights(self.fmt, *[torch.cat([getattr(p, f) for p in parts]).contiguous()
                                                      for f in fields])
                self.pool.g13 = self.pool.g13.float().contiguous()
                self.pool.g2 = self.pool.g2.float().contiguous()
        else:
            # no GPU slot at all: every route goes to the CPU tier. The decode kernels still run (every route skips
            # the pool) so that the down kernel collects the CPU part through the mailbox and adds it; they need a
            # pool operand, one zero slot that is never read, shared by every such layer of this shape
            key = (self.H, self.I, self.fmt, self.device)
            if key not in _EMPTY_POOLS:
                one = experts.select(torch.tensor([0], device=experts.w13.device))
                _EMPTY_POOLS[key] = ExpertWeights(self.fmt, *[torch.zeros_like(getattr(one, f), device=self.device)
                                                              for f in ('w13', 'w2', 's13', 's2')],
                                                  torch.zeros(1, 2, dtype=torch.float32, device=self.device),
                                                  torch.zeros(1, dtype=torch.float32, device=self.device))
            self.pool = _EMPTY_POOLS[key]
        self.slotless = S == 0 and self.n_shared == 0
        table = torch.full((self.E,), -1, dtype=torch.int32)
        for s, e in enumerate(self.hot):
            table[e] = s
        self.table = table.to(self.device)
        self.table_host = table.clone()
        self.shared_slots = (torch.arange(S, S + self.n_shared, dtype=torch.int32, device=self.device)
                             if self.n_shared else None)
        self.engine = engine
        self.mailbox = mailbox if (engine is not None and S < self.E) else None
        if self.mailbox is not None:
            self.mailbox.register(layer, engine)
        self.kk = self.k + self.n_shared
        self.elastic = None       # ElasticSlots (cache/elastic.py) when the layer has extra slots
        # peer mode (cache/peer.py): `table` / `shared_slots` hold global slot names read through `peer`; prefill
        # routes with the local names
        self.peer, self.spr = None, 0
        self.table_local, self.shared_local = self.table, self.shared_slots
        # miss share (XTIER_DECODE_MISS_GPU): the pinned host pool's base addresses for the decode kernels
        self.host_table, self.share_min = None, 0
        # cold-backed CPU tier (cache/cold.py ColdPrefill): the prefill staging is gathered from the engine's RAM
        # slots and the drive store instead of a host copy of the layer
        self.cold_prefill = None
        # swap ring (cache/ring.py SwapRing): when set, swaps and fills copy on its stream and the GPU applies them
        self.ring = None
        self._alloc(max_tokens)

    def _make_bufs(self, m: int) -> dict:
        dev = self.device
        return dict(ids=torch.empty(m, self.kk, dtype=torch.int32, device=dev),
                    w=torch.empty(m, self.kk, dtype=torch.float32, device=dev),
                    slots=torch.empty(m, self.kk, dtype=torch.int32, device=dev),
                    mid=torch.empty(m * self.kk, self.I, dtype=torch.float16, device=dev),
                    ws_logits=torch.empty(m, self.E, dtype=torch.float32, device=dev),
                    ws_count=torch.zeros(m, dtype=torch.int32, device=dev),
                    gpu_part=torch.empty(m, self.H, dtype=torch.float32, device=dev))

    def _alloc(self, m: int):
        """The decode buffers: allocated once, so a captured decode graph keeps valid pointers whatever prefills run
        between its replays (prefill calls use separate buffers, `_prefill_bufs`)."""
        self.max_m = m
        for k, v in self._make_bufs(m).items():
            setattr(self, k, v)

    def _prefill_bufs(self, m: int) -> dict:
        """Route / scratch buffers of a prefill chunk of m tokens, shared by the layers of one shape (they run one
        after another on the compute stream)."""
        key = (self.kk, self.E, self.I, self.H, self.device)
        cur = _PREFILL_BUFS.get(key)
        if cur is None or cur['ids'].shape[0] < m:
            cur = _PREFILL_BUFS[key] = self._make_bufs(m)
        return cur

    @property
    def all_hot(self) -> bool:
        return len(self.hot) == self.E

    # ------------------------------------------------------------------ decode (graph capturable)
    def use_peers(self, peer_table: torch.Tensor, spr: int, rank: int, sets: list[list[int]]):
        """Peer mode: routes to experts held by another GPU's pool (sets[r]: rank r's hot experts, slot = index) read
        them over NVLink; only experts no GPU holds go to the CPU tier. Swaps are off in this mode (other GPUs read
        this pool)."""
        from .peer import owners
        own = owners(sets, rank)
        table = torch.full((self.E,), -1, dtype=torch.int32)
        for e, (r, s) in own.items():
            table[e] = r * spr + s
        self.table = table.to(self.device)
        self.peer, self.spr = peer_table, spr
        if self.n_shared:
            S = len(self.hot)
            self.shared_slots = torch.arange(S, S + self.n_shared, dtype=torch.int32, device=self.device) + rank * spr
        self.peer_sets = sets

    def route(self, x: torch.Tensor, use_mailbox: bool, active: torch.Tensor | None = None, local: bool = False):
        """local: route with this GPU's slot names only (the grouped prefill reads the local pool)."""
        m = x.shape[0]
        logits = None
        if m > MAX_DECODE_TOKENS and not use_mailbox:
            # prefill-sized call: the router GEMM on the tensor cores (FP32 out), then per-token selection
            logits = ops.gemm_f32(x, self.router_w, self.ws_logits[:m])
        table = self.table_local if local else self.table
        shared = self.shared_local if local else self.shared_slots
        ops.moe_route(x, self.router_w, self.router_bias, self.corr_bias,
                      None if self.all_hot else table, shared,
                      self.ids[:m], self.w[:m], self.slots[:m], self.ws_logits, self.ws_count, self.k, self.mode,
                      self.n_group, self.topk_group,
                      self.renorm, self.scale, self.layer,
                      self.mailbox.handle if (use_mailbox and self.mailbox is not None) else 0, active, logits,
                      *((self._cold_index, self.share_min, self.HOST_BASE)
                        if (self.host_table is not None and use_mailbox and not local) else (None, 0, 0)))

    def experts_gpu(self, x: torch.Tensor, out: torch.Tensor, add: torch.Tensor | None, use_mailbox: bool,
                    out_f32: torch.Tensor | None = None):
        m = x.shape[0]
        if self.pool is not None:
            hb = self.HOST_BASE if self.host_table is not None else 0
            ops.moe_gate_up(x, self.slots[:m], self.pool.w13, self.pool.s13, self.pool.g13, self.mid[:m * self.kk],
                            self.fmt_code, self.limit, peer=self.peer, spr=self.spr, host=self.host_table,
                            host_base=hb)
            ops.moe_down(self.mid[:m * self.kk], self.slots[:m], self.w[:m], self.pool.w2, self.pool.s2, self.pool.g2,
                         add, out, out_f32, self.fmt_code,
                         self.mailbox.handle if (use_mailbox and self.mailbox is not None) else 0,
                         gpu_part=self.gpu_part[:m], peer=self.peer, spr=self.spr, host=self.host_table, host_base=hb)
        else:
            raise RuntimeError('TieredMoE: no pool operand')

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, add: torch.Tensor | None = None,
                active: torch.Tensor | None = None):
        """x bf16 [m, H] -> out bf16 [m, H] (= MoE(x) + add). `active`: int32 [m] token flags of a decode-sized
        call; flag-0 tokens skip their routed experts (their output is the shared experts' only)."""
        m = x.shape[0]
        out = torch.empty_like(x) if out is None else out
        if m <= MAX_DECODE_TOKENS and m <= self.max_m:
            use_mb = self.mailbox is not None
            self.route(x, use_mb, active)
            self.experts_gpu(x, out, add, use_mb)
            return out
        return self.prefill(x, out, add)

    # ------------------------------------------------------------------ prefill (hybrid: GPU hot || CPU rest)
    def prefill(self, x: torch.Tensor, out: torch.Tensor, add: torch.Tensor | None = None, chunk: int = 1024):
        if self.ring is not None:   # the device tables catch up with the host residency the staging follows
            self.ring.sync()
        grouped = (x.shape[0] >= config.get('XTIER_GPU_PREFILL_MIN') and self.pool is not None
                   and (self.all_hot or self.host is not None or getattr(self, '_host_cold', None) is not None
                        or self.cold_prefill is not None))
        if grouped:   # every expert on the GPU: cold ones uploaded once for the whole call, larger chunks
            stage = None if self.all_hot else self._staged()
            chunk = 8192
        pf = self._prefill_bufs(min(chunk, x.shape[0]))
        saved = {k: getattr(self, k) for k in _BUF_NAMES}, self.max_m
        for k in _BUF_NAMES:
            setattr(self, k, pf[k])
        self.max_m = pf['ids'].shape[0]
        try:
            for s in range(0, x.shape[0], chunk):
                e = min(x.shape[0], s + chunk)
                if grouped:
                    self._prefill_grouped(x[s:e], out[s:e], None if add is None else add[s:e], stage)
                else:
                    self._prefill_chunk(x[s:e], out[s:e], None if add is None else add[s:e])
        finally:
            for k, v in saved[0].items():
                setattr(self, k, v)
            self.max_m = saved[1]
        return out

    def _prefill_chunk(self, x, out, add):
        m = x.shape[0]
        self.route(x, False)
        cpu_thread = None
        cpu_out = None
        if not self.all_hot and self.engine is not None:
            ids = self.ids[:m, :self.k]
            slots = self.slots[:m, :self.k]
            cpu_ids = torch.where(slots < 0, ids, torch.full_like(ids, -1)).cpu()
            w = self.w[:m, :self.k].float().cpu()
            xc = x.cpu()
            cpu_out = torch.empty(m, self.H, dtype=torch.float32).pin_memory()
            box = {}

            def run():
                try:
                    self.engine.forward(xc, cpu_ids, w, out=cpu_out)
                except Exception as ex:   # re-raised on the caller's thread
                    box['err'] = ex

            cpu_thread = threading.Thread(target=run, daemon=True)
            cpu_thread.start()
        gpu = torch.empty(m, self.H, dtype=torch.float32, device=self.device)
        self.experts_gpu(x, out, add, False, out_f32=gpu)
        if cpu_thread is not None:
            cpu_thread.join()
            if 'err' in box:
                raise box['err']
            total = gpu + cpu_out.to(self.device, non_blocking=True)
            if add is not None:
                total += add.float()
            out.copy_(total.to(out.dtype))
        return out

    def _prefill_grouped(self, x, out, add, stage=None):
        """Prefill on the tensor cores: the hot (and shared) routes on the slot pool, the other routes on a staging
        copy of the layer's cold experts uploaded from pinned host memory (the PCIe copy is the cost; every cold expert
        is read once per call instead of once per 8 tokens by the CPU engine)."""
        from .prefill import combine, grouped_routes
        m = x.shape[0]
        self.route(x, False, local=True)
        slots, w = self.slots[:m], self.w[:m]
        parts = [grouped_routes(x, slots, w, self.pool)]
        if not self.all_hot:
            ids = self.ids[:m, :self.k]
            cold = torch.where(slots[:, :self.k] < 0, self._cold_index[ids.long().clamp_min(0)],
                               torch.full_like(ids, -1))
            parts.append(grouped_routes(x, cold, w[:, :self.k], stage))
        return combine(parts, out, None if add is None else add.contiguous())

    def upload_async(self, stream: torch.cuda.Stream, after: torch.cuda.Event | None = None):
        """Starts this layer's cold-expert upload on `stream` (after `after`, e.g. the previous user of the staging
        buffer being done); the next prefill call of the layer waits for it instead of copying itself."""
        if self.cold_prefill is not None:   # the drive reads start now; the copy is enqueued when they are done
            self.cold_prefill.start()
            self._pending = ('cold', stream, after)
            return
        if self.all_hot or (self.host is None and getattr(self, '_host_cold', None) is None):
            return
        with torch.cuda.stream(stream):
            if after is not None:
                stream.wait_event(after)
            stage = self._upload_cold()
            ev = torch.cuda.Event()
            ev.record(stream)
        self._pending = (stage, ev)

    def _staged(self) -> ExpertWeights:
        pending = getattr(self, '_pending', None)
        self._pending = None
        if self.cold_prefill is not None:
            return self._upload_cold_prefill(*(pending[1:] if pending is not None else (None, None)))
        if pending is not None:
            torch.cuda.current_stream(self.device).wait_event(pending[1])
            return pending[0]
        return self._upload_cold()

    def attach_cold_prefill(self, cp):
        """Prefill staging from a cold-backed CPU tier (cache/cold.py ColdPrefill over this layer's non-GPU experts,
        in staging order)."""
        cold = [e for e in range(self.E) if self.table_host[e] < 0]
        if list(cp.cold) != cold:
            raise ValueError(f'layer {self.layer}: the cold prefill covers other experts than the non-GPU ones')
        idx = torch.full((self.E,), -1, dtype=torch.int32)
        idx[cold] = torch.arange(len(cold), dtype=torch.int32)
        self._cold_index = idx.to(self.device)
        self.cold_prefill = cp

    def _gpu_stage(self, like: ExpertWeights) -> ExpertWeights:
        """The GPU staging pool for `like`'s shape (shared by the layers of one shape, two by layer parity)."""
        key = (like.experts, self.H, self.I, self.fmt, self.device, self.layer % 2)
        stage = _STAGING.get(key)
        if stage is None:
            stage = ExpertWeights(self.fmt, *[torch.empty_like(getattr(like, f), device=self.device)
                                              for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2')])
            _STAGING[key] = stage
        return stage

    def _upload_cold_prefill(self, stream=None, after=None) -> ExpertWeights:
        """Waits for the host staging of the cold-backed tier and copies it to the GPU staging on `stream` (after
        `after`); the current stream waits for the copy."""
        hc = self.cold_prefill.stage()
        stage = self._gpu_stage(hc)
        cur = torch.cuda.current_stream(self.device)
        stream = cur if stream is None else stream
        with torch.cuda.stream(stream):
            if after is not None:
                stream.wait_event(after)
            for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                getattr(stage, f).copy_(getattr(hc, f), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
        if stream != cur:
            cur.wait_event(ev)
        self.cold_prefill.uploaded(ev)
        return stage

    def prepare_prefill(self):
        """Pinned host copy of the layer's cold experts (the source of the prefill uploads); done at model build so
        the first prefill does not pay for page-locking. With XTIER_DECODE_MISS_GPU it is also the pool the decode
        kernels read a shared CPU-tier expert from."""
        if (self.all_hot or self.host is None or getattr(self, '_host_cold', None) is not None
                or self.cold_prefill is not None):
            return
        self._upload_cold(copy=False)
        self._setup_miss_share()

    HOST_BASE = 1 << 24   # slot names at and above this are experts of the pinned host pool

    def _setup_miss_share(self):
        import ctypes as C
        import math
        share = config.get('XTIER_DECODE_MISS_GPU')
        if share <= 0 or self.peer is not None or self.device.type != 'cuda':
            return
        hc = self._host_cold
        fields = ('w13', 's13', 'g13', 'w2', 's2', 'g2')
        ptrs = [getattr(hc, f).data_ptr() for f in fields]
        L = ops.cdll()
        L.xt_host_ptr_mapped.argtypes = [C.c_void_p]
        if not all(L.xt_host_ptr_mapped(C.c_void_p(p)) for p in ptrs):
            import logging
            logging.getLogger('xtier_b200').warning('XTIER_DECODE_MISS_GPU: the host pool is not device-mapped; off')
            return
        self.host_table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.share_min = max(1, math.ceil(0.5 / share))

    def _upload_cold(self, copy: bool = True) -> ExpertWeights:
        """The layer's cold experts in a staging pool on the GPU (shared by the layers of one shape), copied from a
        pinned host copy made on first use."""
        if getattr(self, '_host_cold', None) is None:
            cold = [e for e in range(self.E) if self.table_host[e] < 0]
            idx = torch.full((self.E,), -1, dtype=torch.int32)
            idx[cold] = torch.arange(len(cold), dtype=torch.int32)
            self._cold_index = idx.to(self.device)
            hc = self.host.select(torch.tensor(cold))
            pin = (lambda t: t.pin_memory()) if torch.cuda.is_available() else (lambda t: t)   # pinned for fast H2D
            self._host_cold = ExpertWeights(self.fmt, *[pin(getattr(hc, f).contiguous())
                                                        for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2')])
            self._host_cold.g13 = pin(self._host_cold.g13.float())
            self._host_cold.g2 = pin(self._host_cold.g2.float())
        hc = self._host_cold
        stage = self._gpu_stage(hc)
        if copy:
            for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                getattr(stage, f).copy_(getattr(hc, f), non_blocking=True)
        return stage

    # ------------------------------------------------------------------ residency changes
    @property
    def can_refill(self) -> bool:
        """Whether GPU slots can take other experts: a host copy or a cold-backed tier is their source, and no other
        GPU reads this pool."""
        return self.peer is None and (self.host is not None or self.cold_prefill is not None)

    def _expert_host(self, e: int) -> ExpertWeights:
        """Expert e on the host ([1, ...] fields): from the host copy, or gathered from the cold-backed tier."""
        if self.host is not None:
            return self.host.select([e])
        if self.cold_prefill is not None:
            return self.cold_prefill.read_experts([e])
        raise RuntimeError(f'layer {self.layer}: no host source for expert {e}')

    def swap(self, incoming: int, victim: int):
        """Replaces hot expert `victim` by `incoming` (stream-ordered with every kernel launched so far/after)."""
        if self.peer is not None:
            raise RuntimeError('swaps are off in peer mode (other GPUs read this pool)')
        slot = int(self.table_host[victim])
        if slot < 0 or int(self.table_host[incoming]) >= 0:
            raise ValueError(f'swap {incoming} <- {victim}: bad residency')
        src = self._expert_host(incoming)
        self.table_host[victim] = -1
        self.table_host[incoming] = slot
        if self.ring is not None:   # unmapped now, copied on the ring's stream, mapped once the copy has landed
            self.ring.place(self, incoming, slot, _pinned(src), victim=victim)
        else:
            self.table[victim] = -1
            for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                getattr(self.pool, f)[slot].copy_(getattr(src, f)[0], non_blocking=True)
            self.table[incoming] = slot
        if slot >= len(self.hot):   # an elastic slot: both experts keep their prefill staging index
            self.elastic.occupant[slot - self.elastic.first] = incoming
            return
        self.hot[slot] = incoming
        if getattr(self, '_host_cold', None) is not None:
            # the prefill staging covers exactly the non-resident experts: the victim takes the incoming expert's
            # staging index (its pinned host bytes are replaced); an upload made before the swap is stale
            idx = int(self._cold_index[incoming])
            self._cold_index[victim] = idx
            self._cold_index[incoming] = -1
            for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                getattr(self._host_cold, f)[idx].copy_(getattr(self.host, f)[victim])
            self._pending = None
        elif self.cold_prefill is not None:   # the cold-backed staging gathers the victim in the incoming's place
            idx = int(self._cold_index[incoming])
            self._cold_index[victim] = idx
            self._cold_index[incoming] = -1
            self.cold_prefill.cold[idx] = victim

    def fill(self, incoming: int):
        """Puts a non-resident expert into an empty elastic slot (stream-ordered like `swap`). Experts in elastic
        slots keep their prefill staging index, since their slot can be released again."""
        slot = None if self.elastic is None else self.elastic.free_slot()
        if self.peer is not None:
            raise RuntimeError('elastic slots are off in peer mode')
        if slot is None or int(self.table_host[incoming]) >= 0:
            raise ValueError(f'fill {incoming}: no free elastic slot or already resident')
        src = self._expert_host(incoming)
        if self.ring is not None:
            self.ring.place(self, incoming, slot, _pinned(src))
        else:
            for f in ('w13', 'w2', 's13', 's2', 'g13', 'g2'):
                getattr(self.pool, f)[slot].copy_(getattr(src, f)[0], non_blocking=True)
            self.table[incoming] = slot
        self.table_host[incoming] = slot
        self.elastic.occupant[slot - self.elastic.first] = incoming

    def resident(self) -> list[int]:
        return list(self.hot) + (self.elastic.occupants() if self.elastic is not None else [])

    def gpu_bytes(self) -> int:
        if self.pool is None or self.slotless:
            return 0
        n = sum(getattr(self.pool, f).numel() * getattr(self.pool, f).element_size() for f in ('g13', 'g2'))
        if self.elastic is not None:     # reserved address space is not memory: count what is mapped
            return n + self.elastic.mapped_bytes()
        return n + sum(getattr(self.pool, f).numel() * getattr(self.pool, f).element_size()
                       for f in ('w13', 'w2', 's13', 's2'))
