"""Context parallelism for long sequences: decode context parallel (DCP)
and sequence-parallel prefill (SP), as collective algorithms over a
torch.distributed group.

* :func:`lse_merge` -- merge per-shard attention outputs with their
  log-sum-exps (exact; rank order fixed, so every rank gets identical bits).
* :func:`dcp_decode_attention` -- each rank attends over its shard of the KV
  (positions ``r, r + W, ...`` interleaved, or a contiguous range), then the
  (o, lse) pairs are all-gathered and merged (reference: DCP combine with
  LSE, patch P:2990-3027, ``cp_lse_ag_out_rs``).
* :func:`dcp_topk` -- sparse-indexer top-k over a sharded key set: local
  top-k, ids lifted to global positions, (score, id) all-gathered, global
  top-k re-selected identically on all ranks (ties: lower id) (reference:
  DCP sparse top-k, C39).
* :func:`sp_prefill_attention` -- sequence-parallel prefill: every rank holds
  a contiguous chunk of the prompt, all-gathers the chunks' (compressed) K/V
  and runs causal attention for its own queries at its global offset
  (new in this framework; the reference has no SP prefill).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.distributed as dist


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _all_gather(t: torch.Tensor, group) -> torch.Tensor:
    W, _ = _world(group)
    out = [torch.empty_like(t) for _ in range(W)]
    dist.all_gather(out, t.contiguous(), group=group)
    return torch.stack(out)


def lse_merge(outs: torch.Tensor, lses: torch.Tensor) -> torch.Tensor:
    """outs [W, ..., D], lses [W, ...] (natural log; -inf = empty shard) -> [..., D]."""
    m = lses.max(dim=0).values
    m = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w = torch.exp(lses - m)                       # [W, ...]
    den = w.sum(dim=0)
    num = (w[..., None] * outs).sum(dim=0)
    return num / den.clamp_min(1e-30)[..., None]


def partial_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                      mask: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """q [T, H, D], k [S, D] (shared by heads, MLA latent form), v [S, Dv] -> (o [T, H, Dv], lse [T, H])."""
    s = torch.einsum("thd,sd->ths", q.float(), k.float()) * scale
    if mask is not None:
        s = s.masked_fill(~mask[:, None, :], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[..., None])
    o = torch.einsum("ths,sd->thd", p, v.float())
    return o, lse


def dcp_decode_attention(q, k_local, v_local, scale, group, mask_local=None):
    """q [T, H, D] replicated; k_local/v_local this rank's KV shard -> full attention [T, H, Dv]."""
    o, lse = partial_attention(q, k_local, v_local, scale, mask_local)
    return lse_merge(_all_gather(o, group), _all_gather(lse, group))


def dcp_topk(scores_local: torch.Tensor, k: int, global_ids: torch.Tensor, group) -> torch.Tensor:
    """scores_local [T, S_r] (-inf = invalid), global_ids [S_r] (position of each local key)
    -> global top-k positions [T, k] (-1 padded), identical on every rank, ties to the lower id."""
    T, S = scores_local.shape
    kk = min(k, S)
    # stable local selection: sort by (-score, id)
    order = torch.argsort(global_ids)
    sc, gid = scores_local[:, order], global_ids[order]
    vals, idx = torch.sort(-sc, dim=1, stable=True)
    vals, idx = -vals[:, :kk], idx[:, :kk]
    ids = gid[idx]
    ids = torch.where(torch.isinf(vals) & (vals < 0), torch.full_like(ids, -1), ids)
    if kk < k:
        vals = torch.cat([vals, torch.full((T, k - kk), float("-inf"), dtype=vals.dtype)], 1)
        ids = torch.cat([ids, torch.full((T, k - kk), -1, dtype=ids.dtype)], 1)
    av, ai = _all_gather(vals, group), _all_gather(ids, group)          # [W, T, k]
    av = av.permute(1, 0, 2).reshape(T, -1)
    ai = ai.permute(1, 0, 2).reshape(T, -1)
    # global order: score desc, then id asc (ids are unique across ranks; -1 entries have -inf)
    big = torch.iinfo(torch.int64).max
    key_id = torch.where(ai < 0, torch.full_like(ai, big), ai)
    o1 = torch.argsort(key_id, dim=1, stable=True)
    av, ai = av.gather(1, o1), ai.gather(1, o1)
    o2 = torch.argsort(-av, dim=1, stable=True)
    out = ai.gather(1, o2)[:, :k]
    return torch.where(torch.isinf(av.gather(1, o2)[:, :k]), torch.full_like(out, -1), out)


def sp_prefill_attention(q_local, k_local, v_local, scale, group):
    """Contiguous chunk per rank (equal lengths): q/k/v_local [Tc, ...] -> causal attention
    of the local queries over all keys up to their global position."""
    W, r = _world(group)
    Tc = q_local.shape[0]
    k_all = _all_gather(k_local, group).reshape(W * Tc, *k_local.shape[1:])
    v_all = _all_gather(v_local, group).reshape(W * Tc, *v_local.shape[1:])
    qpos = r * Tc + torch.arange(Tc)
    mask = torch.arange(W * Tc)[None, :] <= qpos[:, None]
    o, _ = partial_attention(q_local, k_all, v_all, scale, mask)
    return o


# ---------------------------------------------------------------- SP prefill, model level
def sp_chunk(n: int, world: int, rank: int) -> Tuple[int, int, int]:
    """Prompt of n tokens over `world` ranks -> (chunk length Tc, first position, real tokens
    on this rank).  Chunks are equal (the tail is padded); padding sits after every real
    token, so causality keeps it out of every real row."""
    Tc = -(-n // world)
    lo = rank * Tc
    return Tc, lo, max(0, min(n, lo + Tc) - lo)


def sp_attention(cfg, lw, x_local: torch.Tensor, lo: int, cs: torch.Tensor, group, cache=None, li: int = 0):
    """MLA attention for this rank's contiguous chunk (global positions lo..lo+Tc-1).
    All-gathered per token: the compressed row only (normed latent + roped shared key,
    kv_lora + rope values), not per-head K/V; every rank expands the gathered latents
    itself.  With `cache`, the full sequence's K/V is stored for decode."""
    from ..models import reference as ref
    W, _ = _world(group)
    Tc = x_local.shape[0]
    Hh = lw.q_b.shape[0] // cfg.qk_head_dim
    nope, rope, vd, lat = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
    pos = lo + torch.arange(Tc, device=x_local.device)
    qkva = x_local.float() @ lw.qkv_a.dequant().t()
    qa = ref.rms_norm(qkva[:, : cfg.q_lora_rank], lw.q_a_norm, cfg.rms_eps)
    c = ref.rms_norm(qkva[:, cfg.q_lora_rank: cfg.q_lora_rank + lat], lw.kv_a_norm, cfg.rms_eps)
    kr = ref.apply_rope(qkva[:, cfg.q_lora_rank + lat:], cs[pos])
    row = torch.cat([c, kr], dim=-1)                                   # [Tc, lat + rope]
    rows = _all_gather(row, group).reshape(W * Tc, lat + rope)         # the whole (padded) prompt
    q = (qa @ lw.q_b.dequant().t()).view(Tc, Hh, nope + rope)
    q_pe = ref.apply_rope(q[..., nope:].transpose(0, 1), cs[pos]).transpose(0, 1)
    kvb = (rows[:, :lat] @ lw.kv_b.dequant().t()).view(W * Tc, Hh, nope + vd)
    S = W * Tc
    k = torch.cat([kvb[..., :nope], rows[:, None, lat:].expand(S, Hh, rope)], dim=-1).transpose(0, 1)
    v = kvb[..., nope:].transpose(0, 1)
    qf = torch.cat([q[..., :nope], q_pe], dim=-1).transpose(0, 1)       # [Hh, Tc, qk]
    if cache is not None:
        cache.k[li], cache.v[li] = k, v
    s = (qf @ k.transpose(1, 2)) * (1.0 / math.sqrt(nope + rope))
    s = s.masked_fill(torch.arange(S, device=s.device)[None, None, :] > pos[None, :, None], float("-inf"))
    o = torch.softmax(s, dim=-1) @ v
    return o.transpose(0, 1).reshape(Tc, Hh * vd) @ lw.o.dequant().t()


def sp_prefill_forward(mw, tokens: torch.Tensor, cs: torch.Tensor, group, cache=None):
    """Sequence-parallel prefill of one prompt (the full token list on every rank; each
    rank computes its chunk).  -> (logits of the last real token [V], final normed
    hidden of every real token [n, H], gathered on every rank).  `cache` (RefKV) gets the
    full K/V of every layer, truncated to the real tokens."""
    from ..models import reference as ref
    cfg = mw.cfg
    W, r = _world(group)
    n = tokens.shape[0]
    Tc, lo, _ = sp_chunk(n, W, r)
    ids = torch.zeros(Tc, dtype=torch.long, device=tokens.device)
    real = tokens[lo:lo + Tc]
    ids[:real.shape[0]] = real
    x = mw.embed[ids].float()
    for li, lw in enumerate(mw.layers):
        h = ref.rms_norm(x, lw.attn_norm, cfg.rms_eps)
        x = x + sp_attention(cfg, lw, h, lo, cs, group, cache, li)
        h = ref.rms_norm(x, lw.ffn_norm, cfg.rms_eps)
        x = x + (ref.moe_block(cfg, lw, h) if lw.is_moe else ref.dense_ffn(cfg, lw, h))
    hn = ref.rms_norm(x, mw.final_norm, cfg.rms_eps)
    hid = _all_gather(hn, group).reshape(W * Tc, -1)[:n]
    if cache is not None:
        cache.truncate(n)
    logits = hid[-1:] @ mw.lm_head.dequant().t()
    return logits[0], hid


# ---------------------------------------------------------------- DCP, model level
class ShardKV:
    """This rank's share of a sequence's per-layer K/V under decode context parallelism:
    position p lives on rank (p // interleave) % world.  Entries keep their positions, so
    truncation (rejected drafts) is by position.  Same interface as the oracle's RefKV."""

    def __init__(self, n_layers: int, world: int, rank: int, interleave: int = 1):
        self.world, self.rank, self.interleave = world, rank, interleave
        self.k = [None] * n_layers        # [Hh, S_r, qk]
        self.v = [None] * n_layers        # [Hh, S_r, vd]
        self.pos = [None] * n_layers      # [S_r]

    def owns(self, positions: torch.Tensor) -> torch.Tensor:
        return (positions // self.interleave) % self.world == self.rank

    def append(self, li: int, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor):
        m = self.owns(positions)
        k, v, p = k[:, m], v[:, m], positions[m]
        if self.k[li] is None:
            self.k[li], self.v[li], self.pos[li] = k, v, p
        else:
            self.k[li] = torch.cat([self.k[li], k], dim=1)
            self.v[li] = torch.cat([self.v[li], v], dim=1)
            self.pos[li] = torch.cat([self.pos[li], p])

    def truncate(self, length: int):
        for i in range(len(self.k)):
            if self.k[i] is not None:
                keep = self.pos[i] < length
                self.k[i], self.v[i], self.pos[i] = self.k[i][:, keep], self.v[i][:, keep], self.pos[i][keep]


def dcp_attention_fn(group):
    """-> an attention function for the oracle's decoder layers (see
    ``reference.attention_context``): q / K / V of the step's tokens are computed on
    every rank, each rank appends the positions it owns to its ShardKV, attends over its
    shard (causal by position) and the (o, lse) partials are LSE-merged across ranks."""
    from ..models import reference as ref

    def attn(cfg, lw, x, positions, cs, cache, li=0, heads=None):
        Hh = heads or lw.q_b.shape[0] // cfg.qk_head_dim
        T = x.shape[0]
        nope, rope, vd, lat = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
        qkva = x.float() @ lw.qkv_a.dequant().t()
        qa = ref.rms_norm(qkva[:, : cfg.q_lora_rank], lw.q_a_norm, cfg.rms_eps)
        c = ref.rms_norm(qkva[:, cfg.q_lora_rank: cfg.q_lora_rank + lat], lw.kv_a_norm, cfg.rms_eps)
        pcs = cs[positions]
        kr = ref.apply_rope(qkva[:, cfg.q_lora_rank + lat:], pcs)
        q = (qa @ lw.q_b.dequant().t()).view(T, Hh, nope + rope)
        q_pe = ref.apply_rope(q[..., nope:].transpose(0, 1), pcs).transpose(0, 1)
        kvb = (c @ lw.kv_b.dequant().t()).view(T, Hh, nope + vd)
        k = torch.cat([kvb[..., :nope], kr[:, None, :].expand(T, Hh, rope)], dim=-1).transpose(0, 1)
        cache.append(li, k, kvb[..., nope:].transpose(0, 1), positions)
        qf = torch.cat([q[..., :nope], q_pe], dim=-1)                      # [T, Hh, qk]
        ks, vs, ps = cache.k[li], cache.v[li], cache.pos[li]
        s = torch.einsum("thd,hsd->ths", qf.float(), ks.float()) * (1.0 / math.sqrt(nope + rope))
        s = s.masked_fill(ps[None, None, :] > positions[:, None, None], float("-inf"))
        lse = torch.logsumexp(s, dim=-1)                                   # [T, Hh]; -inf: no key here
        p = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[..., None])
        o = torch.einsum("ths,hsd->thd", p, vs.float())
        o = lse_merge(_all_gather(o, group), _all_gather(lse, group))       # [T, Hh, vd]
        return o.reshape(T, Hh * vd) @ lw.o.dequant().t()
    return attn
