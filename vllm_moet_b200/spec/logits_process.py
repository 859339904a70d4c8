"""Logits processing before a token is chosen: repetition / presence / frequency
penalties, logit bias and the allowed-token restriction, with vLLM's semantics
(``SamplingParams`` fields of the same names).  Disallowed tokens get ``DISALLOWED`` added
(a finite -1e30, so no later arithmetic turns a row into NaN).

Speculative verify: row j of a verify pass scores the token after the pending token and
drafts ``d_1 .. d_j``.  The drafts before it count as generated text for row j: if row j's
choice is ever emitted, those drafts were all accepted, so the penalties see exactly the
history that the token would have had in plain one-token decoding.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch

DISALLOWED = -1e30


def allowed_bias(allowed, V: int, device=None) -> torch.Tensor:
    """[V] additive bias: 0 for the allowed tokens, DISALLOWED for every other."""
    b = torch.full((V,), DISALLOWED, dtype=torch.float32, device=device)
    ids = torch.tensor([t for t in allowed if 0 <= t < V], dtype=torch.long, device=device)
    b[ids] = 0.0
    return b


def process_logits(logits: torch.Tensor, sp, prompt: Sequence[int], out: Sequence[int],
                   drafts: Optional[Sequence[int]] = None) -> torch.Tensor:
    """logits [R, V] (row j after `out` + drafts[:j]) -> processed logits [R, V] (f32)."""
    x = logits.float().clone()
    if sp is None or not sp.processes_logits:
        return x
    R, V = x.shape
    drafts = list(drafts or [])[: max(R - 1, 0)]
    dev = x.device
    counts = torch.bincount(torch.as_tensor(list(out), dtype=torch.long, device=dev), minlength=V)[:V]
    counts = counts[None].repeat(R, 1).float()
    for j, d in enumerate(drafts):                 # row j + 1 and later saw draft j
        counts[j + 1:, int(d)] += 1
    if sp.repetition_penalty != 1.0:
        seen = counts > 0
        if len(prompt):
            seen[:, torch.as_tensor(list(prompt), dtype=torch.long, device=dev)] = True
        r = sp.repetition_penalty
        x = torch.where(seen, torch.where(x > 0, x / r, x * r), x)
    if sp.frequency_penalty:
        x = x - sp.frequency_penalty * counts
    if sp.presence_penalty:
        x = x - sp.presence_penalty * (counts > 0).float()
    if sp.logit_bias:
        ids = torch.tensor([t for t in sp.logit_bias if 0 <= t < V], dtype=torch.long, device=dev)
        if len(ids):
            x[:, ids] += torch.tensor([sp.logit_bias[int(t)] for t in ids], device=dev)
    if sp.allowed_token_ids is not None:
        x = x + allowed_bias(sp.allowed_token_ids, V, dev)[None]
    for w in sp.bad_word_ids or []:
        # a bad word's last token is banned on the rows whose history ends with the word's
        # other tokens (a one-token word: always)
        if not 0 <= w[-1] < V:
            continue
        for j in range(R):
            hist = list(out) + [int(d) for d in drafts[:j]]
            if len(w) == 1 or (len(hist) >= len(w) - 1 and hist[len(hist) - len(w) + 1:] == w[:-1]):
                x[j, w[-1]] += DISALLOWED
    return x
