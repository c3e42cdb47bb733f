"""Token choice with temperature and nucleus (top-p) sampling, per row, without a host synchronization (capturable in
the decode CUDA graph; the random numbers come from torch's generator, which CUDA graphs advance per replay).

Per row b with temperature t_b > 0: the logits divided by t_b are sorted, the smallest prefix of tokens whose
probability mass reaches top_p_b is kept (the most likely token always), and a token is drawn from the kept ones in
proportion to their probability by the Gumbel-max rule (argmax of log-probability plus Gumbel(0, 1) noise is a draw
from the softmax: Gumbel 1954; used for sampling since Maddison, Tarlow and Minka 2014). Rows with t_b = 0 take the
argmax (greedy).
"""
from __future__ import annotations

import torch


def sample(logits: torch.Tensor, temp: torch.Tensor, top_p: torch.Tensor, out: torch.Tensor | None = None,
           generator: torch.Generator | None = None) -> torch.Tensor:
    """logits [B, V], temp [B] (0: greedy), top_p [B] in (0, 1] -> token ids [B] int64 (written to `out` if
    given)."""
    lf = logits.float()
    greedy = torch.argmax(lf, dim=-1)
    z = lf / temp.float().clamp_min(1e-5)[:, None]
    zs, idx = torch.sort(z, dim=-1, descending=True)
    ps = torch.softmax(zs, dim=-1)
    before = torch.cumsum(ps, dim=-1) - ps              # mass of the tokens ranked above each one
    keep = before < top_p.float()[:, None]
    keep[:, 0] = True
    zs = zs.masked_fill(~keep, float('-inf'))
    u = torch.rand(zs.shape, device=zs.device, generator=generator).clamp_(1e-12, 1.0 - 1e-7)
    choice = torch.argmax(zs - torch.log(-torch.log(u)), dim=-1)
    sampled = idx.gather(-1, choice[:, None])[:, 0]
    res = torch.where(temp > 0, sampled, greedy)
    if out is not None:
        out.copy_(res)
        return out
    return res


def nucleus_probs(logits: torch.Tensor, temp: float, top_p: float) -> torch.Tensor:
    """The distribution `sample` draws one row from (the tests' oracle): softmax(logits / temp) restricted to the
    top-p nucleus and renormalized."""
    p = torch.softmax(logits.double() / temp, dim=-1)
    ps, idx = torch.sort(p, descending=True)
    before = torch.cumsum(ps, 0) - ps
    keep = before < top_p
    keep[0] = True
    out = torch.zeros_like(p)
    out[idx[keep]] = ps[keep]
    return out / out.sum()
