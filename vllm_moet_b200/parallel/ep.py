"""Expert parallelism with all-to-all dispatch / combine (data-parallel tokens).

Every rank holds its own tokens (data-parallel attention) and a contiguous range
of the routed experts, ``[rank * E / W, (rank + 1) * E / W)``.  One MoE block:

1. route the local tokens (router and shared expert are replicated);
2. dispatch: each (token, top-k slot) row goes to the rank that owns its expert;
   the per-destination row counts are exchanged first, then the rows and their
   expert ids, with one ``all_to_all_single`` each (variable splits);
3. every rank runs its experts over the rows it received;
4. combine: the results return over the reversed splits, land back in
   (token, slot) order and are summed with the routing weights in a fixed slot
   order, so the output does not depend on arrival order.

This is the collective algorithm of the serving configuration "DP attention + EP
MoE" (the reference refuses EP; its MoE runs replicated or TP-sharded).  It is
written with torch.distributed collectives, so it runs on gloo (CPU tests) and
NCCL alike; the expert math is the oracle's dequantised experts.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def expert_owner(e: torch.Tensor, num_experts: int, world: int) -> torch.Tensor:
    per = num_experts // world
    return e // per


def _a2a(x: torch.Tensor, send_counts: torch.Tensor, recv_counts: torch.Tensor, group) -> torch.Tensor:
    out = x.new_empty((int(recv_counts.sum()),) + tuple(x.shape[1:]))
    dist.all_to_all_single(out, x.contiguous(), recv_counts.tolist(), send_counts.tolist(), group=group)
    return out


def ep_dispatch(ids: torch.Tensor, h: torch.Tensor, num_experts: int, group):
    """ids [T, k] routed experts, h [T, H] local tokens -> (rows received [R, H], their expert
    ids [R], and the state the combine needs)."""
    W = dist.get_world_size(group)
    T, k = ids.shape
    flat_e = ids.reshape(-1).long()
    dest = expert_owner(flat_e, num_experts, W)
    order = torch.argsort(dest, stable=True)                       # rows grouped by destination rank
    send_counts = torch.bincount(dest, minlength=W).to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    tok = torch.arange(T, device=ids.device).repeat_interleave(k)[order]
    rows = _a2a(h[tok].float(), send_counts, recv_counts, group)
    rexp = _a2a(flat_e[order], send_counts, recv_counts, group)
    return rows, rexp, (order, send_counts, recv_counts, T, k)


def ep_combine(y: torch.Tensor, weights: torch.Tensor, state, group) -> torch.Tensor:
    """y [R, H] expert outputs of the received rows -> [T, H] weighted sum per local token."""
    order, send_counts, recv_counts, T, k = state
    back = _a2a(y, recv_counts, send_counts, group)                 # this rank's rows, in `order`
    pairs = torch.empty_like(back)
    pairs[order] = back                                             # (token, slot) order
    pairs = pairs.view(T, k, back.shape[-1]) * weights.view(T, k, 1).float()     # explicit H: T may be 0
    out = pairs[:, 0]
    for j in range(1, k):                                           # fixed slot order
        out = out + pairs[:, j]
    return out


def ep_moe_block(cfg, lw, h: torch.Tensor, group, expert_fn=None) -> torch.Tensor:
    """The MoE block of one rank under DP attention + EP.  `lw.experts` holds this rank's
    expert range (``e_lo`` / ``n_local``) or all experts (then only the owned range is used).
    `expert_fn(e_local, rows) -> [n, H]` overrides the expert math (default: the oracle's)."""
    from ..models import reference as ref
    W, r = dist.get_world_size(group), dist.get_rank(group)
    E = cfg.num_experts
    if E % W:
        raise ValueError(f"{E} experts do not split evenly over {W} ranks")
    ids, w = ref.route(cfg, lw, h)
    rows, rexp, state = ep_dispatch(ids, h, E, group)
    ex = lw.experts
    lo = ex.e_lo if getattr(ex, "n_local", None) is not None else 0
    own_lo = r * (E // W)
    y = torch.zeros_like(rows)
    for e in torch.unique(rexp).tolist():
        sel = (rexp == e).nonzero(as_tuple=True)[0]
        if expert_fn is not None:
            y[sel] = expert_fn(e - own_lo, rows[sel])
            continue
        w13, w2 = ex.dequant_expert(e - lo)
        y[sel] = ref.swiglu(rows[sel] @ w13.float().t(), cfg.swiglu_limit) @ w2.float().t()
    out = ep_combine(y, w, state, group)
    if lw.shared_gate_up is not None:
        out = out + ref.swiglu(h.float() @ lw.shared_gate_up.dequant().t(), cfg.swiglu_limit) @ \
            lw.shared_down.dequant().t()
    return out


def dispatch_bytes(T: int, k: int, hidden: int, world: int, elem_bytes: int = 2) -> Tuple[int, int]:
    """Bytes one rank sends per MoE block at uniform routing: (dispatch, combine) off-rank."""
    off = T * k * (world - 1) // world
    return off * hidden * elem_bytes, off * hidden * elem_bytes


def ep_partition(mw, rank: int, world: int):
    """Keep only this rank's expert range [rank * E / W, (rank + 1) * E / W) in every MoE
    layer (MTP included); attention, dense and shared-expert weights stay replicated."""
    from ..models.weights import ExpertPool
    E = mw.cfg.num_experts
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    n = E // world
    lo = rank * n
    layers = list(mw.layers) + ([mw.mtp.layer] if mw.mtp is not None else [])
    for lw in layers:
        ex = lw.experts
        if ex is None:
            continue
        if ex.dense_w13 is not None:
            pool, table = ex.pool[:n], torch.arange(n, dtype=torch.int32)
            d13, d2 = ex.dense_w13[lo:lo + n], ex.dense_w2[lo:lo + n]
        else:
            idx = ex.slot_table[lo:lo + n].long()
            pool, table = ex.pool[idx].contiguous(), torch.arange(n, dtype=torch.int32, device=ex.pool.device)
            d13 = d2 = None
        lw.experts = ExpertPool(ex.layout, pool, table, dense_w13=d13, dense_w2=d2, e_lo=lo, n_local=n)
    return mw


def ep_dummy_row(mw, k: int, group) -> None:
    """The MoE collectives of one engine row with no tokens: a rank with fewer rows than its
    peers runs these so every rank makes the same sequence of all-to-all calls (each main
    MoE layer once, then the MTP layer k times)."""
    cfg = mw.cfg
    empty = torch.zeros(0, cfg.hidden)
    for lw in mw.layers:
        if lw.is_moe:
            ep_moe_block(cfg, lw, empty, group)
    if k and mw.mtp is not None:
        for _ in range(k):
            ep_moe_block(cfg, mw.mtp.layer, empty, group)
