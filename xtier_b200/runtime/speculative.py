"""Speculative decoding with a chain draft: draft S tokens with a small model, truncate the chain at the draft's
confidence, verify all of it in one target forward, accept losslessly.

Per round, for one sequence at position `pos` whose last accepted token is `t0`:
1. the draft model proposes d_1..d_S autoregressively, keeping its probabilities q_j (temperature-scaled softmax);
2. `truncate` (csrc/cuda/spec.cu) keeps the leading drafts with q_j(d_j) >= threshold (at least one; all of them for
   greedy decoding), zeroes the q row of the first dropped draft and sets the verify tokens' flags, so the target's
   MoE layers skip the routed experts of tokens whose output nobody reads;
3. the target runs [t0, d_1..d_S] from `pos` in one forward (causal over its KV cache), giving p_0..p_S;
4. `verify_chain` accepts d_j with probability min(1, p_j(d_j) / q_j(d_j)) in order (a zero q row never accepts) and
   on the first rejection samples from the residual (p_j - q_j)+; when every draft is accepted it samples a bonus token
   from p_S. For greedy decoding it accepts while d_j == argmax p_j and then takes argmax p. Either way the output has
   exactly the target's distribution (greedy: the target's own greedy tokens).
Stale KV entries past the accepted prefix are overwritten by the next round (attention reads positions < pos only).
(Reference parity: xtier/packs/speculative/truncate.py (truncation rule, token flags, zeroed q row), the verify rule of
SGLang's chain sampler it relies on.)
"""
from __future__ import annotations

import torch

from .. import ops


def truncate(q: torch.Tensor, tokens: torch.Tensor, threshold: float, greedy: bool = False,
             flags: torch.Tensor | None = None) -> torch.Tensor:
    """q [B, S, V] fp32 (modified in place), tokens [B, S + 1] int64 -> flags int32 [B, S + 1]."""
    B, S, _ = q.shape
    flags = torch.empty(B * (S + 1), dtype=torch.int32, device=q.device) if flags is None else flags
    topk = torch.ones(B, dtype=torch.int32, device=q.device) if greedy else None
    ops.spec_truncate(q, tokens.contiguous(), flags, threshold, topk)
    return flags.view(B, S + 1)


def truncate_reference(q: torch.Tensor, tokens: torch.Tensor, threshold: float, greedy: bool = False):
    """The same rule in plain PyTorch (the tests' oracle); returns (q', flags)."""
    q = q.clone()
    B, S, _ = q.shape
    flags = torch.zeros(B, S + 1, dtype=torch.int32)
    for b in range(B):
        own = q[b, torch.arange(S), tokens[b, 1:]]
        low = (own < threshold).nonzero()
        keep = S if greedy else max(int(low[0]) if low.numel() else S, 1)
        flags[b, :keep + 1] = 1
        if keep < S:
            q[b, keep] = 0
    return q, flags


def verify_chain(p: torch.Tensor, q: torch.Tensor, drafts: torch.Tensor, generator: torch.Generator | None = None,
                 greedy: bool = False) -> list[int]:
    """One sequence: p [S + 1, V] target probabilities, q [S, V] draft probabilities, drafts [S] -> the accepted
    tokens followed by one corrected or bonus token (1 to S + 1 tokens)."""
    S = drafts.shape[0]
    out = []
    if greedy:
        best = torch.argmax(p, dim=-1).tolist()
        for j in range(S):
            if int(drafts[j]) != best[j]:
                return out + [best[j]]
            out.append(best[j])
        return out + [best[S]]
    u = torch.rand(S, generator=generator, device='cpu')
    pc, qc = p.float().cpu(), q.float().cpu()
    for j in range(S):
        d = int(drafts[j])
        pj, qj = float(pc[j, d]), float(qc[j, d])
        if qj > 0 and float(u[j]) * qj <= pj:
            out.append(d)
            continue
        resid = torch.clamp(pc[j] - qc[j], min=0)
        resid = resid if float(resid.sum()) > 0 else pc[j]
        return out + [int(torch.multinomial(resid / resid.sum(), 1, generator=generator))]
    return out + [int(torch.multinomial(pc[S] / pc[S].sum(), 1, generator=generator))]


class SpeculativeDecoder:
    """Chain speculative decoding of one sequence (row 0) of `target` with `draft` (both models with the
    `prefill(st, tokens, start=..., all_logits=...)` interface and their own KV state) and/or copy drafts from a
    `recall` engine (xtier_b200.recall.RecallEngine: continuations of the stream's own context or of the record; a
    copy is a point-mass draft, verified by the same rule). Without a draft model, rounds with no copy are plain
    target steps."""

    def __init__(self, target, draft=None, steps: int = 4, threshold: float | None = None, temperature: float = 0.0,
                 max_len: int = 4096, seed: int = 0, recall=None, hot_ids: torch.Tensor | None = None,
                 draft_temp_scale: float | None = None, tree: bool = False, tree_nodes: int = 16,
                 draft_fp8_head: bool = False):
        """threshold: verify truncation at draft confidence (default XTIER_SPEC_TRUNCATE_Q; 0: off). hot_ids [Vd]:
        the target ids of a draft model whose head covers only a hot vocabulary (its q is scattered into the target
        vocabulary before verification: zero where the draft can never propose, so the accept test and the residual
        stay exact). draft_temp_scale: the draft samples at temperature x this (default XTIER_SPEC_DRAFT_TEMP_SCALE);
        lossless for any scale, since verification uses the q the draft sampled from. tree (greedy decoding): every
        round merges the draft model's chain and the Recall copies into one draft tree of at most `tree_nodes` nodes
        verified in one target forward (runtime/tree.py). draft_fp8_head: the draft's LM head in FP8 (its decode
        step's largest read; `quantize_lm_head`)."""
        from .. import config
        if draft is None and recall is None:
            raise ValueError('speculative decoding needs a draft model or a recall engine')
        self.target, self.draft, self.recall = target, draft, recall
        if draft_fp8_head and draft is not None and hasattr(draft, 'quantize_lm_head'):
            draft.quantize_lm_head()
        self.S, self.temp = steps, temperature
        self.th = config.get('XTIER_SPEC_TRUNCATE_Q') if threshold is None else threshold
        self.draft_scale = (config.get('XTIER_SPEC_DRAFT_TEMP_SCALE') if draft_temp_scale is None
                            else draft_temp_scale)
        self.hot_ids = None if hot_ids is None else torch.as_tensor(hot_ids, dtype=torch.long).cpu()
        self.st_t = target.alloc_state(1, max_len)
        self.st_d = draft.alloc_state(1, max_len) if draft is not None else None
        self.gen = torch.Generator().manual_seed(seed)
        self.tree, self.tree_nodes = tree, tree_nodes
        self.stats = dict(rounds=0, drafted=0, accepted=0, kept=0, copies=0, copied=0, copy_landed=0, plain=0,
                          forwards=0, tree_rounds=0, tree_nodes=0, tree_accepted=0)

    def _probs(self, logits: torch.Tensor, temp: float | None = None) -> torch.Tensor:
        """Target (or draft) distribution per row: one-hot argmax at temperature 0, else softmax(logits / temp)
        restricted to the top-p nucleus (`self.top_p`, 1: all) and renormalized."""
        temp = self.temp if temp is None else temp
        if temp <= 0:
            return torch.nn.functional.one_hot(torch.argmax(logits, -1), logits.shape[-1]).float()
        p = torch.softmax(logits.float() / temp, dim=-1)
        top_p = getattr(self, 'top_p', 1.0)
        if top_p < 1.0:
            ps, idx = torch.sort(p, dim=-1, descending=True)
            drop = (torch.cumsum(ps, -1) - ps) >= top_p      # mass ranked above reaches top_p: outside the nucleus
            drop[..., 0] = False
            p = p.scatter(-1, idx, ps.masked_fill(drop, 0.0))
            p = p / p.sum(-1, keepdim=True)
        return p

    def draft_probs(self, logits: torch.Tensor, V: int) -> torch.Tensor:
        """The draft's proposal distribution over the target vocabulary: at the scaled temperature, and scattered
        from the hot vocabulary when the draft's head covers only that."""
        q = self._probs(logits, self.temp * self.draft_scale if self.temp > 0 else 0.0).float().cpu()
        if self.hot_ids is None:
            return q
        full = torch.zeros(*q.shape[:-1], V)
        full[..., self.hot_ids] = q
        return full

    def _verify(self, pos: int, last: int, drafts: list[int], q: torch.Tensor, active=None,
                keep: int | None = None) -> list[int]:
        """Target forward of [last, drafts...] from `pos` (`active`: the token flags of truncated drafts); the first
        `keep` drafts (default all) are verified against q [keep, V]: the accepted ones plus one corrected / bonus
        token."""
        dev = self.target.device
        keep = len(drafts) if keep is None else keep
        vt = torch.tensor([[last] + drafts], dtype=torch.long, device=dev)
        _, logits = self.target.prefill(self.st_t, vt[0], start=pos, all_logits=True, active=active)
        return verify_chain(self._probs(logits)[:keep + 1], q[:keep], torch.tensor(drafts[:keep]), self.gen,
                            self.temp <= 0)

    def _draft_chain(self, pos: int, last: int, greedy: bool):
        """The draft model's chain of S tokens after `last` (fed at pos ..): (tokens, per-token q rows [S, V])."""
        dev = self.target.device
        seq = self.seq
        if self.dpos < pos:   # the draft catches up on accepted tokens it has not seen
            self.draft.prefill(self.st_d, torch.tensor(seq[self.dpos:pos], device=dev), start=self.dpos)
            self.dpos = pos
        drafts, qs, cur = [], [], last
        V = self.target_vocab(dev)
        for j in range(self.S):
            _, ld = self.draft.prefill(self.st_d, torch.tensor([cur], device=dev), start=pos + j, return_logits=True)
            qj = self.draft_probs(ld, V)
            d = int(torch.argmax(qj)) if greedy else int(torch.multinomial(qj, 1, generator=self.gen))
            drafts.append(d)
            qs.append(qj)
            cur = d
        return drafts, qs

    def _tree_round(self, pos: int, last: int, limit: int | None) -> list[int] | None:
        """One greedy round over a draft tree (the draft chain and the Recall copies); None when no branch exists."""
        from .tree import build_tree, walk_greedy
        chains, copies, drafts = [], [], None
        if self.recall is not None:
            for p in self.recall.candidates(self.rid):
                ids = p.ids[:max(1, limit)] if limit is not None else p.ids
                copies.append((p, ids))
                chains.append((ids, [0.9] * len(ids)))   # a copy is a point mass; longer copies rank lower per node
        if self.draft is not None:
            drafts, qs = self._draft_chain(pos, last, True)
            chains.append((drafts, [float(q.max()) for q in qs]))
        if not chains:
            return None
        tree = build_tree(last, chains, self.tree_nodes)
        if tree.n == 1:
            return None
        dev = self.target.device
        _, logits = self.target.prefill(self.st_t, torch.as_tensor(tree.tokens).to(dev), start=pos, all_logits=True,
                                        tree=tree)
        path, bonus = walk_greedy(tree, torch.argmax(logits, -1).tolist())
        self.target.compact_tree(self.st_t, 0, pos, path)
        acc = [int(tree.tokens[i]) for i in path[1:]] + [int(bonus)]

        def common(a, b):
            n = 0
            while n < min(len(a), len(b)) and a[n] == b[n]:
                n += 1
            return n

        for p, ids in copies:
            self.recall.note(p, common(ids, acc[:-1]))
        if drafts is not None:   # the draft's KV is valid for the accepted prefix of its own chain
            self.dpos = pos + 1 + common(acc, drafts[:self.S - 1])
            if self.recall is not None:
                self.recall.observe_own(self.rid, common(drafts, acc[:-1]))
        self.stats['tree_rounds'] += 1
        self.stats['tree_nodes'] += tree.n
        self.stats['tree_accepted'] += len(acc) - 1
        self.stats['accepted'] += len(acc) - 1
        return acc

    def _sample(self, logits: torch.Tensor) -> int:
        if self.temp <= 0:
            return int(torch.argmax(logits))
        return int(torch.multinomial(self._probs(logits).cpu(), 1, generator=self.gen))

    # ------------------------------------------------------------------ one stream, step by step
    def begin(self, prompt: torch.Tensor) -> int:
        """Prefills `prompt` [T] (target and draft); returns the first new token."""
        dev = self.target.device
        prompt = torch.as_tensor(prompt).to(dev)
        T = prompt.shape[0]
        _, lt = self.target.prefill(self.st_t, prompt, return_logits=True)
        first = self._sample(lt)
        self.seq = prompt.tolist() + [first]
        self.rid = object()
        if self.recall is not None:
            self.recall.begin_stream(self.rid, self.seq, reply_from=T)
        if self.draft is not None and T > 1:
            self.draft.prefill(self.st_d, prompt[:-1])
        self.pos = T            # position of the last accepted token; the target holds KV for positions < pos
        self.dpos = T - 1       # the draft holds KV for positions < dpos
        return first

    def step(self, limit: int | None = None) -> list[int]:
        """One target forward: the accepted drafts plus one corrected / bonus token (a plain step without a draft).
        `limit` caps the copy length (tokens still wanted)."""
        dev = self.target.device
        greedy = self.temp <= 0
        pos, seq = self.pos, self.seq
        last = seq[pos]
        acc = self._tree_round(pos, last, limit) if self.tree and greedy else None
        if acc is None:
            prop = self.recall.propose(self.rid) if self.recall is not None else None
            if prop is not None and prop.ids:
                drafts = prop.ids[:max(1, limit)] if limit is not None else prop.ids
                V = self.target_vocab(dev)
                q = torch.zeros(len(drafts), V)
                q[torch.arange(len(drafts)), torch.tensor(drafts)] = 1.0     # a copy is a point mass
                acc = self._verify(pos, last, drafts, q)
                self.recall.feedback(self.rid, len(acc) - 1)
                self.stats['copies'] += 1
                self.stats['copied'] += len(drafts)
                self.stats['copy_landed'] += len(acc) - 1
            elif self.draft is None:      # a plain target step
                _, lg = self.target.prefill(self.st_t, torch.tensor([last], device=dev), start=pos, return_logits=True)
                acc = [self._sample(lg)]
                self.stats['plain'] += 1
            else:
                if self.dpos < pos:   # the draft catches up on accepted tokens it has not seen
                    self.draft.prefill(self.st_d, torch.tensor(seq[self.dpos:pos], device=dev), start=self.dpos)
                    self.dpos = pos
                drafts, qs, cur = [], [], last
                V = self.target_vocab(dev)
                for j in range(self.S):
                    _, ld = self.draft.prefill(self.st_d, torch.tensor([cur], device=dev), start=pos + j,
                                               return_logits=True)
                    qj = self.draft_probs(ld, V)
                    d = int(torch.argmax(qj)) if greedy else int(torch.multinomial(qj, 1, generator=self.gen))
                    drafts.append(d)
                    qs.append(qj)
                    cur = d
                q = torch.stack(qs)[None].contiguous().float()                  # [1, S, V]
                if self.th > 0:
                    q = q.to(dev)
                    vt = torch.tensor([[last] + drafts], dtype=torch.long, device=dev)
                    flags = truncate(q, vt, self.th, greedy=greedy)
                    keep = int(flags[0].sum()) - 1
                    active = flags[0]
                else:                      # no truncation: every draft is verified
                    keep, active = self.S, None
                acc = self._verify(pos, last, drafts, q[0], active=active, keep=keep)
                self.stats['rounds'] += 1
                self.stats['drafted'] += self.S
                self.stats['kept'] += keep
                self.stats['accepted'] += len(acc) - 1
                if self.recall is not None:
                    self.recall.observe_own(self.rid, len(acc) - 1)
                # the draft fed last, d_1..d_{S-1} at pos..pos+S-1: valid up to the accepted ones
                self.dpos = pos + min(len(acc), self.S)
        self.stats['forwards'] += 1
        seq.extend(acc)
        if self.recall is not None:
            self.recall.extend_stream(self.rid, acc)
        self.pos = len(seq) - 1
        return acc

    def end(self, add: bool = True):
        """Ends the stream (its ids go to the recall record unless add=False)."""
        if self.recall is not None and getattr(self, 'rid', None) is not None:
            self.recall.end_stream(self.rid, add)
        self.rid = None

    def generate(self, prompt: torch.Tensor, max_new_tokens: int) -> list[int]:
        """Up to `max_new_tokens` new tokens after `prompt` [T]."""
        T = torch.as_tensor(prompt).shape[0]
        self.begin(prompt)
        try:
            while len(self.seq) - T < max_new_tokens:
                self.step(max_new_tokens - (len(self.seq) - T))
        finally:
            self.end()
        return self.seq[T:T + max_new_tokens]

    def target_vocab(self, dev) -> int:
        cfg = getattr(self.target, 'cfg', None)
        return cfg.vocab if cfg is not None else int(self.target.vocab)
