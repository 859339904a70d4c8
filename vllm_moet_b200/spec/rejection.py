"""Rejection samplers for draft verification.

* :func:`greedy_accept` -- temperature 0: a draft token is accepted while it
  equals the target's argmax at that position; positions at or beyond a
  request's ``valid_draft_len`` are force-rejected (padding of a width-varied
  DSpark batch never counts as accepted; reference P:20424-20450).  Returns
  the accepted count and the emitted tokens (accepted drafts + one bonus /
  correction token).
* :func:`rejection_sample` -- temperature > 0 (speculative sampling): draft
  token x_i ~ q is accepted with probability min(1, p(x_i) / q(x_i)); at the
  first rejection the token is resampled from normalize(max(p - q, 0)); if all
  drafts pass, a bonus token is sampled from p at the next position.  The
  output distribution equals sampling from p token by token.
* :func:`filter_probs` -- temperature, top-k and nucleus (top-p) filtering of
  logits into the target distribution p.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def greedy_accept(target_argmax: torch.Tensor, drafts: torch.Tensor,
                  valid_draft_len: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """target_argmax [R, L+1], drafts [R, L] -> (n_accepted [R], emitted [R, L+1] (-1 padded))."""
    R, L = drafts.shape
    match = drafts == target_argmax[:, :L]
    if valid_draft_len is not None:
        pos = torch.arange(L, device=drafts.device)[None, :]
        match &= pos < valid_draft_len[:, None]
    n_acc = torch.cumprod(match.int(), dim=1).sum(dim=1)
    emitted = torch.full((R, L + 1), -1, dtype=target_argmax.dtype, device=drafts.device)
    pos = torch.arange(L + 1, device=drafts.device)[None, :]
    keep = pos <= n_acc[:, None]
    emitted[keep] = target_argmax[keep]
    return n_acc, emitted


def rejection_sample(target_probs: torch.Tensor, draft_probs: torch.Tensor, drafts: torch.Tensor,
                     valid_draft_len: Optional[torch.Tensor] = None, generator: Optional[torch.Generator] = None):
    """target_probs [R, L+1, V], draft_probs [R, L, V], drafts [R, L] -> (n_accepted [R], emitted [R, L+1])."""
    R, L = drafts.shape
    dev = drafts.device
    p_d = target_probs[:, :L].gather(-1, drafts[..., None]).squeeze(-1)
    q_d = draft_probs.gather(-1, drafts[..., None]).squeeze(-1).clamp_min(1e-20)
    u = torch.rand(R, L, generator=generator, device=dev)
    ok = u < (p_d / q_d).clamp(max=1.0)
    if valid_draft_len is not None:
        ok &= torch.arange(L, device=dev)[None, :] < valid_draft_len[:, None]
    n_acc = torch.cumprod(ok.int(), dim=1).sum(dim=1)
    emitted = torch.full((R, L + 1), -1, dtype=torch.long, device=dev)
    for r in range(R):
        a = int(n_acc[r])
        emitted[r, :a] = drafts[r, :a]
        if a < L and (valid_draft_len is None or a < int(valid_draft_len[r])):
            resid = (target_probs[r, a] - draft_probs[r, a]).clamp_min(0)
            s = resid.sum()
            dist = resid / s if s > 0 else target_probs[r, a]
        else:
            dist = target_probs[r, a]
        emitted[r, a] = torch.multinomial(dist, 1, generator=generator)[0]
    return n_acc, emitted


def filter_probs(logits: torch.Tensor, temperature: float, top_k: int = 0, top_p: float = 1.0,
                 min_p: float = 0.0) -> torch.Tensor:
    """logits [R, V] -> probabilities [R, V]: softmax(logits / T) without the tokens below
    min_p x the top probability, restricted to the top_k tokens (0 = all) and to the
    smallest set whose probability reaches top_p (at least one)."""
    x = logits.float() / max(temperature, 1e-6)
    if min_p > 0:
        p0 = torch.softmax(x, dim=-1)
        x = x.masked_fill(p0 < min_p * p0.amax(-1, keepdim=True), float("-inf"))
    if top_k and 0 < top_k < x.shape[-1]:
        kth = torch.topk(x, top_k, dim=-1).values[..., -1:]
        x = x.masked_fill(x < kth, float("-inf"))
    p = torch.softmax(x, dim=-1)
    if top_p < 1.0:
        sp, idx = torch.sort(p, dim=-1, descending=True)
        before = torch.cumsum(sp, dim=-1) - sp            # mass strictly above each token
        keep = before < top_p
        keep[..., 0] = True
        mask = torch.zeros_like(p, dtype=torch.bool).scatter(-1, idx, keep)
        p = torch.where(mask, p, torch.zeros_like(p))
        p = p / p.sum(dim=-1, keepdim=True)
    return p
