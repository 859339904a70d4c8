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


def _sp_engine(rank, world):
    """SP prefill through the engine: each rank prefills its chunk of the prompt; the
    first token, the MTP drafts and the decode that follows equal the single-rank engine."""
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, sp_group=dist.group.WORLD)
    prompts = [list(range(5, 5 + 37)), [7, 11, 13, 17, 19, 23, 29]]       # uneven chunks, padded tail
    out = llm.generate(prompts, SamplingParams(max_tokens=8, ignore_eos=True))
    return [o.outputs[0].token_ids for o in out]


def test_sp_prefill_engine_matches_single_rank():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    one = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    prompts = [list(range(5, 5 + 37)), [7, 11, 13, 17, 19, 23, 29]]
    want = [o.outputs[0].token_ids for o in one.generate(prompts, SamplingParams(max_tokens=8, ignore_eos=True))]
    for got in run_ranks(_sp_engine, 3):            # 37 = 13 + 13 + 11 and 7 = 3 + 3 + 1: padded tails
        assert got == want, (got, want)


def test_sp_chunking():
    from vllm_moet_b200.parallel.context import sp_chunk
    assert [sp_chunk(10, 3, r) for r in range(3)] == [(4, 0, 4), (4, 4, 4), (4, 8, 2)]
    assert sp_chunk(2, 4, 3) == (1, 3, 0)


def _dcp_engine(rank, world, interleave):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, dcp_group=dist.group.WORLD,
              dcp_interleave=interleave)
    prompts = [list(range(5, 5 + 37)), [7, 11, 13, 17, 19, 23, 29]]
    out = llm.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True))
    # a row kept open: which positions of each layer's K/V this rank holds
    llm.runner.prefill([prompts[0]], [99])
    for _ in range(3):
        llm.runner.step([99])
    st = llm.runner.rows[99]
    held = [st["main"].pos[li].tolist() for li in range(len(st["main"].pos))]
    return [o.outputs[0].token_ids for o in out], held, st["pos"]


def test_dcp_engine_matches_single_rank():
    """KV interleaved over 3 ranks in runs of 2 positions: prefill, MTP verify with
    rejected drafts (truncation by position) and decode equal the single-rank engine;
    each rank holds exactly the positions it owns and the shards tile the sequence."""
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    one = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    prompts = [list(range(5, 5 + 37)), [7, 11, 13, 17, 19, 23, 29]]
    want = [o.outputs[0].token_ids for o in one.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True))]
    for il in (2,):
        res = run_ranks(_dcp_engine, 3, il)
        for rank, (got, held, _) in enumerate(res):
            assert got == want, (il, got, want)
            for layer in held:
                assert all((p // il) % 3 == rank for p in layer)
        n = res[0][2]
        for li in range(len(res[0][1])):
            # contiguous from 0, no position twice; the last verify step's drafts stay cached
            # past `pos` until the next step truncates them, as in the single-rank cache
            union = sorted(p for r in range(3) for p in res[r][1][li])
            assert union == list(range(len(union))) and len(union) >= n, (il, li)


def test_shard_kv_truncates_by_position():
    from vllm_moet_b200.parallel.context import ShardKV
    kv = ShardKV(1, world=2, rank=1, interleave=2)
    pos = torch.arange(10)
    kv.append(0, torch.arange(10.)[None, :, None], torch.arange(10.)[None, :, None], pos)
    assert kv.pos[0].tolist() == [2, 3, 6, 7]
    kv.truncate(7)
    assert kv.pos[0].tolist() == [2, 3, 6] and kv.k[0].shape[1] == 3
