"""DSpark speculative decoding: semi-autoregressive block drafting.

The drafter (:class:`DSparkDrafter`) proposes a block of ``L`` tokens per
request in one parallel backbone pass over the target's last hidden state
(one position query per draft slot), then walks the block left to right
adding a low-rank **Markov bias** from the previously drafted token, so the
block is coherent without L sequential backbone passes.  A **survival head**
predicts, per position, the probability that the draft survives
verification.

:func:`allocate_widths` gives each request its verify width from calibrated
survival scores (survival x per-position calibration, projected to a valid
prefix with a running minimum): a static confidence threshold ``tau``, or with
``tau`` = 0 a global budget (``budget_frac`` x requests x length tokens) spent on
the best scores, ties to earlier positions and requests, so a tie never
inflates the budget and every width is a prefix.  The hardware-aware choice of
the batch-wide verify length lives in :mod:`.dspark_policy`.
Reference: DSpark drafter and scheduler, patch P:14478-14971 and the tests at
P:753-800.
"""
from __future__ import annotations

from typing import Tuple

import torch
import torch.nn as nn


def allocate_widths(survival: torch.Tensor, calibration: torch.Tensor, num_reqs: int, length: int,
                    tau: float, budget_frac: float) -> torch.Tensor:
    """survival [>=num_reqs, >=length], calibration [>=length] -> int32 widths [num_reqs] (<= length).

    Scores are survival x calibration, projected onto a non-increasing curve (running
    minimum) so every selection is a prefix.  tau > 0: each request keeps the positions
    scoring >= tau (a static confidence width).  tau = 0: a global budget of
    budget_frac x requests x length positions goes to the best scores; the flattened
    rows are sorted stably, so equal scores go to earlier positions and requests and
    the budget is used exactly."""
    s = survival[:num_reqs, :length].float() * calibration[:length].float().to(survival.device)[None, :]
    s = torch.cummin(s, dim=1).values
    if tau > 0:
        return (s >= tau).sum(dim=1, dtype=torch.int32).clamp_max(length)
    budget = min(max(int(num_reqs * length * budget_frac + 1e-9), 0), num_reqs * length)
    if budget == 0:
        return torch.zeros(num_reqs, dtype=torch.int32, device=s.device)
    if budget == num_reqs * length:
        return torch.full((num_reqs,), length, dtype=torch.int32, device=s.device)
    # positions in (request, position) order; a non-increasing row keeps its prefix first
    order = torch.sort(s.reshape(-1), descending=True, stable=True).indices
    keep = torch.zeros(num_reqs * length, dtype=torch.bool, device=s.device)
    keep[order[:budget]] = True
    return keep.view(num_reqs, length).sum(dim=1, dtype=torch.int32)


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
        # survival of position j = probability that drafts 1..j all survive (a cumulative product)
        surv = torch.cumprod(torch.sigmoid(self.survival(z)).squeeze(-1), dim=1)
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


def swa_indices_batch(context_lens: torch.Tensor, block_len: int, window: int, width: int) -> torch.Tensor:
    """``swa_indices`` for a batch of draft blocks at one fixed width, as tensor ops on the
    lengths' device (no host loop, no data-dependent shapes: usable inside a captured
    step).  context_lens [B] -> [B, width] int32; row b equals ``swa_indices(context_lens[b],
    block_len, window)`` truncated or -1-padded to ``width``."""
    c = context_lens.to(torch.int64).view(-1, 1)
    start = (c - window).clamp_min(0)
    n_ctx = c - start                                   # trailing context positions kept
    j = torch.arange(width, device=context_lens.device, dtype=torch.int64).view(1, -1)
    out = torch.where(j < n_ctx, start + j, c + (j - n_ctx))
    return torch.where(j < n_ctx + block_len, out, torch.full_like(out, -1)).to(torch.int32)
