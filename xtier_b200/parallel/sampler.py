"""Token choice over a vocabulary-parallel LM head, and the token-id agreement of tensor-parallel ranks.

* `vocab_parallel_argmax`: each rank holds the logits of its slice of the vocabulary; the greedy token is the global
  argmax, found from one all-gather of every rank's (max, index) pair per row instead of gathering the logits (ties go
  to the lowest vocabulary id, as torch.argmax on the full row).
* `vocab_parallel_sample`: temperature sampling with the Gumbel-max rule: each rank perturbs its logits with Gumbel
  noise drawn from a generator seeded by (seed, step, rank) and the global argmax of the perturbed logits is an exact
  sample of softmax(logits / T); again one all-gather of (max, index) pairs.
* `sync_token_ids`: makes every rank use rank 0's ids (the all-reduce that keeps sampled ids identical across TP
  ranks); skipped entirely for one rank, where it has nothing to agree on.
(Reference parity: xtier/platform.py:182-188 -- the TP token-id sync skipped at TP = 1.)
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _world(group) -> int:
    return dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1


def _global_argmax(val: torch.Tensor, idx: torch.Tensor, group=None) -> torch.Tensor:
    """val, idx [rows] of this rank's best -> [rows] global best index (ties: lower index)."""
    W = _world(group)
    if W == 1:
        return idx
    pair = torch.stack([val.double(), idx.double()], 1)                 # [rows, 2]
    allp = [torch.empty_like(pair) for _ in range(W)]
    dist.all_gather(allp, pair, group=group)
    allp = torch.stack(allp, 0)                                           # [W, rows, 2]
    v, i = allp[..., 0], allp[..., 1]
    best = v.max(0).values
    cand = torch.where(v == best[None], i, torch.full_like(i, float('inf')))
    return cand.min(0).values.long()


def vocab_parallel_argmax(local_logits: torch.Tensor, vocab_offset: int, group=None) -> torch.Tensor:
    """local_logits [rows, V_local] (columns vocab_offset ..) -> [rows] global greedy token ids."""
    val, idx = local_logits.float().max(-1)
    return _global_argmax(val, idx + vocab_offset, group)


def vocab_parallel_sample(local_logits: torch.Tensor, vocab_offset: int, temperature: float, seed: int, step: int,
                          group=None) -> torch.Tensor:
    """Gumbel-max sample of softmax(logits / temperature) over the whole vocabulary."""
    if temperature <= 0:
        return vocab_parallel_argmax(local_logits, vocab_offset, group)
    rank = dist.get_rank(group) if _world(group) > 1 else 0
    g = torch.Generator(device=local_logits.device).manual_seed((seed * 1000003 + step) * 1009 + rank)
    u = torch.rand(local_logits.shape, generator=g, device=local_logits.device, dtype=torch.float64)
    gumbel = -torch.log(-torch.log(u.clamp_min(1e-300)))
    val, idx = (local_logits.double() / temperature + gumbel).max(-1)
    return _global_argmax(val, idx + vocab_offset, group)


def sync_token_ids(ids: torch.Tensor, group=None) -> torch.Tensor:
    """Every rank gets rank 0's ids (in place); one rank: returns at once."""
    if _world(group) == 1:
        return ids
    src = dist.get_global_rank(group, 0) if group is not None else 0
    dist.broadcast(ids, src=src, group=group)
    return ids
