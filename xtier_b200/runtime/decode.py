"""Decode runtime: KV state, CUDA-graph capture of one decode step, and the public `generate` API.

A decode step (all layers, the mailbox round trips to the CPU engine included) is captured once into a CUDA graph and
replayed per token. Inside the graph the step also advances itself (next token -> input, position + 1), so a
device-timed loop is pure replays. `generate()` is the end-to-end path a user calls: per step it copies the input
token from pinned host memory, replays the graph and reads the next token back to the host.

Reference parity: the reference relies on SGLang's CUDA-graph runner and scheduler; this is the
framework's own minimal runner for the named configs.
"""
from __future__ import annotations

import torch


class Generator:
    def __init__(self, model, batch: int = 1, max_len: int = 4096, use_graph: bool = True, policy=None,
                 governor=None, sampling: bool = False):
        """sampling: the decode step draws each row's token with that row's temperature and top-p
        (`set_sampling`; temperature 0 stays greedy) instead of taking the argmax. Decided before capture."""
        self.model = model
        self.sampling = sampling
        model.sampling = sampling
        # between decode steps: adaptive hot-slot swaps and the elastic cache's sizing (the model's, unless given)
        self.policy = policy if policy is not None else getattr(model, 'policy', None)
        self.governor = governor if governor is not None else getattr(model, 'governor', None)
        self.batch = batch
        self.max_len = max_len
        self.state = model.alloc_state(batch, max_len)
        self.buf = model.decode_buffers(batch)
        self.use_graph = use_graph
        self.graph = None
        self.host_tokens = torch.zeros(batch, dtype=torch.int64).pin_memory()
        self.host_next = torch.zeros(batch, dtype=torch.int64).pin_memory()

    # ------------------------------------------------------------------ steps
    def _step_body(self):
        self.model.decode_step(self.state, self.buf)
        self.buf['tokens'].copy_(self.buf['next'])
        self.buf['pos'].add_(1)

    def capture(self, warmup: int = 2, keep_graph: bool = False):
        """Captures one self-advancing decode step. Warm-up runs rewrite the current position only. keep_graph keeps
        the graph's node list for inspection (`graph_kernels`)."""
        saved = {k: self.buf[k].clone() for k in ('pos', 'tokens', 'prev') if k in self.buf}
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self.model.decode_step(self.state, self.buf)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph(keep_graph=keep_graph)
        with torch.cuda.graph(self.graph):
            self._step_body()
        if keep_graph:
            self.graph.instantiate()
        torch.cuda.synchronize()
        for k, v in saved.items():
            self.buf[k].copy_(v)
        self.check()

    def step(self):
        """One decode step on the device (no host synchronization)."""
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_body()

    def check(self):
        dev = getattr(self.model, 'device', None)
        if dev is not None and torch.device(dev).type == 'cuda':
            from .. import ops
            if int(ops.gemm_error_word(dev).item()):
                raise RuntimeError('a tensor-core kernel (GEMM or prefill attention) had a bounded wait run out')
        mb = getattr(self.model, 'mailbox', None)
        if mb is not None:
            mb.check()
        bg = getattr(self.model, 'bigram', None)
        if bg is not None:
            bg.check()

    def set_sampling(self, temperature, top_p=1.0):
        """Per-row (or one for all rows) temperature and top-p of the following steps (device buffers the captured
        step reads; no recapture)."""
        if not self.sampling and torch.any(torch.as_tensor(temperature, dtype=torch.float32) > 0):
            raise ValueError('this Generator decodes greedily: create it with sampling=True')
        self.buf['temp'].copy_(torch.as_tensor(temperature, dtype=torch.float32).expand(self.batch))
        self.buf['top_p'].copy_(torch.as_tensor(top_p, dtype=torch.float32).expand(self.batch))

    # ------------------------------------------------------------------ public API
    def prefill(self, prompts: torch.Tensor, start: int = 0):
        """prompts [batch, T] token ids (host or device): fills the KV cache, sets the first decode input. start > 0:
        the cache already holds the KV of prompts[:, :start] (the same ids at the same positions, e.g. a previous
        request's prefix); only the rest is computed."""
        prompts = torch.as_tensor(prompts)
        first = []
        T = prompts.shape[1]
        if not 0 <= start < T:
            raise ValueError(f'prefill: start {start} outside [0, {T})')
        gov = self.governor

        from .. import config
        chunked = getattr(self.model, 'prefill_chunked', None) if config.get('XTIER_LONG_PREFILL_CHUNK') > 0 else None
        prefill = chunked or self.model.prefill
        kw = {'start': start} if start else {}

        def run(ids, b):
            if not self.sampling:
                return prefill(self.state, ids, row=b, **kw)
            from .sampling import sample     # the first token is drawn like the decode step's
            _, lg = prefill(self.state, ids, row=b, return_logits=True, **kw)
            return sample(lg[None], self.buf['temp'][b:b + 1], self.buf['top_p'][b:b + 1])

        for b in range(self.batch):
            ids = prompts[b, start:].to(self.model.device)
            if gov is None:
                first.append(run(ids, b))
                continue
            gov.before_alloc(T - start, T)     # extra slots go back until the predicted need fits
            torch.cuda.synchronize()
            before = torch.cuda.memory_allocated()
            torch.cuda.reset_peak_memory_stats()
            first.append(gov.guarded(run, ids, b))
            gov.after_forward(T - start, T, before, torch.cuda.max_memory_allocated())
        self.buf['tokens'].copy_(torch.cat(first).view(-1))
        if 'prev' in self.buf:   # the last prompt token precedes the first decode input
            self.buf['prev'].copy_(prompts[:, -1].to(self.buf['prev'].device))
        self.buf['pos'].fill_(T)
        torch.cuda.synchronize()
        self.check()

    def generate(self, prompts: torch.Tensor, max_new_tokens: int) -> torch.Tensor:
        """Greedy generation: [batch, T] prompt ids -> [batch, max_new_tokens] new ids (host tensor)."""
        self.prefill(prompts)
        if self.use_graph and self.graph is None:
            self.capture()
        out = torch.empty(self.batch, max_new_tokens, dtype=torch.int64)
        self.host_tokens.copy_(self.buf['tokens'].cpu())
        for i in range(max_new_tokens):
            self.decode_one()
            out[:, i] = self.host_next
            self.between_steps()
        self.check()
        return out

    def between_steps(self):
        """Host work between two decode steps (no kernel of the step is in flight): swap rounds, elastic sizing."""
        if self.policy is not None:
            self.policy.step()
        if self.governor is not None:
            self.governor.after_decode()

    def decode_one(self):
        """End-to-end step: H2D copy of the input token from pinned memory, replay, D2H read of the next token."""
        self.buf['tokens'].copy_(self.host_tokens, non_blocking=True)
        self.step()
        self.host_next.copy_(self.buf['next'], non_blocking=True)
        torch.cuda.current_stream().synchronize()
        self.host_tokens.copy_(self.host_next)
        return self.host_next

    @property
    def h2d_bytes_per_step(self) -> int:
        return self.host_tokens.numel() * self.host_tokens.element_size()

    @property
    def d2h_bytes_per_step(self) -> int:
        return self.host_next.numel() * self.host_next.element_size()


def graph_kernels(graph: torch.cuda.CUDAGraph) -> dict[str, int]:
    """Kernel nodes of a captured graph (captured with keep_graph), counted by (mangled) kernel name: what one replay
    launches."""
    from cuda.bindings import driver as d
    g = d.CUgraph(graph.raw_cuda_graph())
    err, _, n = d.cuGraphGetNodes(g, 0)
    err, nodes, n = d.cuGraphGetNodes(g, n)
    if err != d.CUresult.CUDA_SUCCESS:
        raise RuntimeError(f'cuGraphGetNodes: {err}')
    counts: dict[str, int] = {}
    for nd in nodes[:n]:
        err, t = d.cuGraphNodeGetType(nd)
        if t != d.CUgraphNodeType.CU_GRAPH_NODE_TYPE_KERNEL:
            continue
        err, prm = d.cuGraphKernelNodeGetParams(nd)
        err, name = d.cuFuncGetName(prm.func)
        name = name.decode() if isinstance(name, (bytes, bytearray)) else str(name)
        counts[name] = counts.get(name, 0) + 1
    return counts


def own_kernel_launches(counts: dict[str, int]) -> int:
    """Launches of this package's kernels (namespace xt) in a graph_kernels() count."""
    return sum(v for k, v in counts.items() if k.startswith('_ZN2xt') or 'xt::' in k)
