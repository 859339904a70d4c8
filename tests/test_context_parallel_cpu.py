"""Context parallelism on CPU ranks (gloo): DCP decode attention with the LSE
merge, the DCP sparse top-k merge, and sequence-parallel prefill attention all
equal the single-rank computation."""
import math

import torch

from mp_util import run_ranks


def _dcp(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200.parallel.context import dcp_decode_attention, dcp_topk, partial_attention
    g = torch.Generator().manual_seed(0)
    S, T, H, D, Dv = 70, 3, 4, 24, 16
    q = torch.randn(T, H, D, generator=g)
    k = torch.randn(S, D, generator=g)
    v = torch.randn(S, Dv, generator=g)
    scale = 1 / math.sqrt(D)
    full, _ = partial_attention(q, k, v, scale)
    mine = torch.arange(rank, S, world)                    # interleaved KV shards
    got = dcp_decode_attention(q, k[mine], v[mine], scale, dist.group.WORLD)
    scores = torch.randn(T, S, generator=g)
    scores[:, ::7] = 0.25                                  # ties
    scores[1, 40:] = float("-inf")                         # a shorter context
    want = []
    for t in range(T):
        o = torch.argsort(-scores[t], stable=True)[:16]
        o = torch.where(torch.isinf(scores[t][o]), torch.full_like(o, -1), o)
        want.append(o)
    sel = dcp_topk(scores[:, mine], 16, mine, dist.group.WORLD)
    return float((got - full).abs().max()), torch.equal(sel, torch.stack(want))


def test_dcp_attention_and_topk():
    for err, same in run_ranks(_dcp, 3):
        assert err < 1e-5 and same


def _sp(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200.parallel.context import partial_attention, sp_prefill_attention
    g = torch.Generator().manual_seed(1)
    Tc, H, D = 8, 2, 16
    T = Tc * world
    q = torch.randn(T, H, D, generator=g)
    k = torch.randn(T, D, generator=g)
    v = torch.randn(T, D, generator=g)
    mask = torch.ones(T, T).tril().bool()
    full, _ = partial_attention(q, k, v, 0.25, mask)
    sl = slice(rank * Tc, (rank + 1) * Tc)
    got = sp_prefill_attention(q[sl], k[sl], v[sl], 0.25, dist.group.WORLD)
    return float((got - full[sl]).abs().max())


def test_sp_prefill_attention():
    assert max(run_ranks(_sp, 2)) < 1e-5
