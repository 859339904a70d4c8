"""DSpark speculative decoding: semi-autoregressive block drafting.

The drafter (:class:`DSparkDrafter`) proposes a block of ``L`` tokens per
request in one parallel backbone pass over the target's last hidden state
(one position query per draft slot), then walks the block left to right
adding a low-rank **Markov bias** from the previously drafted token, so the
block is coherent without L sequential backbone passes.  A **survival head**
predicts, per position, the probability that the draft survives
verification.

:func:`allocate_widths` is the hardware-aware scheduler: calibrated survival
scores (survival x per-position calibration) are projected to a valid prefix
with a running minimum, positions above ``tau`` become candidates, and a
global verify budget (``budget_frac`` x requests x length tokens) keeps the
best-scored candidates -- ties broken by position, then request, so a tie
never inflates the budget and every request's width is a prefix.
Reference: DSpark drafter and scheduler, patch P:14478-14971 and the tests at
P:753-800.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn


def allocate_widths(survival: torch.Tensor, calibration: torch.Tensor, num_reqs: int, length: int,
                    tau: float, budget_frac: float) -> torch.Tensor:
    """survival [>=num_reqs, >=length], calibration [>=length] -> int32 widths [num_reqs] (<= length)."""
    s = survival[:num_reqs, :length].float() * calibration[:length].float()[None, :]
    s = torch.cummin(s, dim=1).values                     # valid-prefix projection
    cand = s > tau
    budget = int(budget_frac * num_reqs * length + 1e-9)
    if budget <= 0:
        return torch.zeros(num_reqs, dtype=torch.int32)
    r_idx, p_idx = cand.nonzero(as_tuple=True)
    if r_idx.numel() > budget:
        scores = s[r_idx, p_idx]
        # sort by score desc, then position asc, then request asc (stable lexicographic)
        order = sorted(range(r_idx.numel()), key=lambda i: (-float(scores[i]), int(p_idx[i]), int(r_idx[i])))
        keep = torch.zeros_like(cand)
        for i in order[:budget]:
            keep[r_idx[i], p_idx[i]] = True
        cand = keep
    # a width is the length of the selected prefix
    widths = torch.cumprod(cand.int(), dim=1).sum(dim=1)
    return widths.to(torch.int32)


class DSparkDrafter(nn.Module):
    """Block drafter: parallel backbone over [h; position embedding], low-rank
    Markov bias from the previous draft token, survival (confidence) head."""

    def __init__(self, hidden: int, vocab: int, block: int = 4, rank: int = 32, ffn: int = 0):
        super().__init__()
        self.block, self.vocab = block, vocab
        ffn = ffn or 2 * hidden
        self.pos = nn.Parameter(torch.randn(block, hidden) * 0.02)
        self.norm = nn.LayerNorm(hidden)
        self.up = nn.Linear(hidden, ffn, bias=False)
        self.down = nn.Linear(ffn, hidden, bias=False)
        self.head = nn.Linear(hidden, vocab, bias=False)
        self.markov_in = nn.Embedding(vocab, rank)
        self.markov_out = nn.Linear(rank, vocab, bias=False)
        self.survival = nn.Linear(hidden, 1)

    def backbone(self, h: torch.Tensor) -> torch.Tensor:
        """h [R, H] -> per-slot states [R, L, H] (one pass for the whole block)."""
        x = h[:, None, :] + self.pos[None]
        return x + self.down(torch.nn.functional.silu(self.up(self.norm(x))))

    @torch.no_grad()
    def propose(self, h: torch.Tensor, last_token: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """h [R, H] (target hidden at the last verified position), last_token [R]
        -> (drafts [R, L], draft probs [R, L, V], survival [R, L])."""
        z = self.backbone(h)
        base = self.head(z)                                # [R, L, V]
        surv = torch.sigmoid(self.survival(z)).squeeze(-1)
        prev = last_token
        drafts, probs = [], []
        for j in range(self.block):                        # cheap sequential Markov walk
            logits = base[:, j] + self.markov_out(self.markov_in(prev))
            p = torch.softmax(logits.float(), dim=-1)
            prev = p.argmax(-1)
            drafts.append(prev)
            probs.append(p)
        return torch.stack(drafts, 1), torch.stack(probs, 1), surv


def swa_indices(context_len: int, block_len: int, window: int, min_width: int = 512, align: int = 128) -> torch.Tensor:
    """KV positions the DSpark draft block attends to (non-causal within the block):
    the trailing ``window`` context positions plus every query position of the block
    (future ones included), padded with -1 to a width >= ``min_width`` that is a
    multiple of ``align`` (reference: DSpark SWA indices, patch P:17441-17617)."""
    start = max(0, context_len - window)
    ctx = torch.arange(start, context_len, dtype=torch.int32)
    blk = torch.arange(context_len, context_len + block_len, dtype=torch.int32)
    idx = torch.cat([ctx, blk])
    width = max(min_width, -(-idx.numel() // align) * align)
    out = torch.full((width,), -1, dtype=torch.int32)
    out[: idx.numel()] = idx
    return out
