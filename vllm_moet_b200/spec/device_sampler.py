"""Speculative sampling of a whole decode batch in device tensor ops, with no host
synchronisation, so it can sit inside a captured CUDA graph.

Per request row b (verify rows j = 0..k score the pending token and the k greedy MTP
drafts) the target distribution p_j is softmax(logits / T_b) filtered by min-p and top-k,
then top-p over the renormalised survivors (per-row parameters); T_b = 0 makes p_j one-hot at the argmax (lowest id on
ties), so greedy and sampling rows share one batch.  The drafts are greedy, so the draft
distribution q is one-hot and the speculative-sampling rule reduces to:

* draft d_j is accepted with probability p_j(d_j) (u_j < p_j(d_j));
* at the first rejection a the token is drawn from p_a with d_a removed (renormalised),
  which is norm(max(p - q, 0)) for one-hot q; after k acceptances the bonus token is drawn
  from p_k.

The emitted tokens are then distributed exactly as token-by-token sampling from p
(Leviathan et al. 2023, "Fast Inference from Transformers via Speculative Decoding").
Draws use the Gumbel-max trick, argmax(log r + G) with G = -log(-log U).

Random numbers are a counter-based hash of (request seed, sequence position, lane,
vocabulary id), so a replayed step (expert-cache or gate replay) draws the same numbers
and a seeded request is reproducible whatever the batch.  The hash is the public-domain
32-bit integer mixer ``x = ((x >> 16) ^ x) * 0x45d9f3b`` applied twice, then
``x = (x >> 16) ^ x`` (T. Mueller); products stay below 2^63, so int64 tensor arithmetic
is exact on every device.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

_M32 = 0xFFFFFFFF
_MUL = 0x45D9F3B


def hash_u32(x: torch.Tensor) -> torch.Tensor:
    """int64 tensor of values in [0, 2^32) -> mixed values in [0, 2^32)."""
    x = x & _M32
    x = (((x >> 16) ^ x) * _MUL) & _M32
    x = (((x >> 16) ^ x) * _MUL) & _M32
    return (x >> 16) ^ x


def uniform(seed: torch.Tensor, counter: torch.Tensor, lane: int, n: int = 0) -> torch.Tensor:
    """U(0, 1) draws: seed / counter broadcastable int64 -> [..., n] (or [...] with n = 0)."""
    s = seed.long()
    h = hash_u32(hash_u32((s ^ (s >> 32)) & _M32) ^ hash_u32(counter.long() * 4 + lane))
    if n:
        h = hash_u32(h[..., None] + torch.arange(n, device=h.device, dtype=torch.long) * 0x9E3779B1)
    return (h.double() + 0.5).mul_(1.0 / 4294967296.0).float()


def target_probs(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
                 min_p: torch.Tensor) -> torch.Tensor:
    """logits [R, V], per-row parameters [R] -> filtered probabilities [R, V] (f32)."""
    R, V = logits.shape
    greedy = temperature <= 0
    t = torch.where(greedy, torch.ones_like(temperature), temperature).float()
    zs, idx = torch.sort(logits.float() / t[:, None], dim=-1, descending=True, stable=True)
    ps = torch.softmax(zs, dim=-1)
    rank = torch.arange(V, device=logits.device)[None, :]
    k_eff = torch.where(top_k > 0, top_k, torch.full_like(top_k, V)).long()
    # min-p and top-k first, then top-p over the renormalised survivors (vLLM's order)
    keep = (rank < k_eff[:, None]) & (ps >= min_p.float()[:, None] * ps[:, :1])
    keep |= rank == 0
    ps = torch.where(keep, ps, torch.zeros_like(ps))
    ps = ps / ps.sum(-1, keepdim=True)
    keep = (torch.cumsum(ps, dim=-1) - ps) < top_p.float()[:, None]
    keep |= rank == 0
    keep &= ~greedy[:, None] | (rank == 0)
    ps = torch.where(keep, ps, torch.zeros_like(ps))
    ps = ps / ps.sum(-1, keepdim=True)
    return torch.zeros_like(ps).scatter_(-1, idx, ps)


def sample_verify(logits: torch.Tensor, drafts: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor,
                  top_p: torch.Tensor, min_p: torch.Tensor, seed: torch.Tensor,
                  pos: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """logits [B, k+1, V] (row j after the pending token and drafts[:j]), drafts [B, k],
    per-request parameters [B], pos [B] = position of the pending token.
    -> (n_accepted [B] int32, tokens [B, k+1] int32): the accepted drafts, then the token
    drawn at the first rejection (or the bonus), repeated to the end of the row."""
    B, kp1, V = logits.shape
    k = kp1 - 1
    rep = lambda v: v.repeat_interleave(kp1)       # noqa: E731
    p = target_probs(logits.reshape(B * kp1, V), rep(temperature), rep(top_k), rep(top_p),
                     rep(min_p)).view(B, kp1, V)
    j = torch.arange(kp1, device=logits.device)
    ctr = pos.long()[:, None] + 1 + j[None, :]                    # the position each row's token lands at
    d = drafts.long()
    if k:
        p_d = p[:, :k].gather(-1, d[..., None]).squeeze(-1)
        ok = uniform(seed[:, None], ctr[:, :k], 0) < p_d
        n_acc = torch.cumprod(ok.int(), dim=1).sum(dim=1)
        r = p.clone()
        r[:, :k].scatter_(-1, d[..., None], 0.0)
        s = r.sum(-1, keepdim=True)
        r = torch.where(s > 0, r / s.clamp_min(1e-30), p)
    else:
        n_acc = torch.zeros(B, dtype=torch.long, device=logits.device)
        r = p
    g = -torch.log(-torch.log(uniform(seed[:, None], ctr, 1, V)))
    drawn = (torch.log(r) + g).argmax(-1)                          # [B, k+1]
    a = n_acc.long()
    pick = drawn.gather(1, a[:, None])
    dpad = torch.cat([d, d.new_zeros(B, 1)], 1) if k else d.new_zeros(B, 1)
    tok = torch.where(j[None, :] < a[:, None], dpad, pick)
    return n_acc.int(), tok.int()


def gather_vocab(logits: torch.Tensor, group, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Vocab-parallel logits [R, V/tp] (rank r holds ids [r V/tp, (r+1) V/tp)) -> the full
    rows [R, V] on every rank (one all-gather).  Every rank then runs the same sampler on
    the same rows with the same seeds, so all ranks draw the same tokens."""
    import torch.distributed as dist
    W = dist.get_world_size(group)
    R, Vl = logits.shape
    buf = (out if out is not None else logits.new_empty(W, R, Vl)).view(W * R, Vl)
    dist.all_gather_into_tensor(buf, logits.contiguous(), group=group)
    return buf.view(W, R, Vl).permute(1, 0, 2).reshape(R, W * Vl)


def process_batch(logits: torch.Tensor, drafts: torch.Tensor, counts: torch.Tensor, prompt_mask: torch.Tensor,
                  repetition: torch.Tensor, frequency: torch.Tensor, presence: torch.Tensor,
                  bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Penalties and logit bias of a decode batch in tensor ops (the batched form of
    ``logits_process.process_logits``).  logits [B, k+1, V]; drafts [B, k]; counts [B, V]
    (f32 counts of each row's generated tokens so far); prompt_mask [B, V] (bool);
    per-row repetition / frequency / presence [B]; bias [B, V] or None.  Verify row j sees
    the drafts before it as generated.  Rows with neutral parameters come out unchanged."""
    B, kp1, V = logits.shape
    c = counts[:, None, :].expand(B, kp1, V)
    if kp1 > 1:
        inc = torch.zeros(B, kp1, V, dtype=counts.dtype, device=counts.device)
        inc[:, 1:].scatter_(-1, drafts.long()[..., None], 1.0)
        c = c + torch.cumsum(inc, dim=1)
    x = logits.float()
    r = repetition.float()[:, None, None]
    seen = (c > 0) | prompt_mask[:, None, :]
    x = torch.where(seen, torch.where(x > 0, x / r, x * r), x)
    x = x - frequency.float()[:, None, None] * c - presence.float()[:, None, None] * (c > 0).float()
    if bias is not None:
        x = x + bias[:, None, :]
    return x
