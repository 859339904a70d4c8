"""Tensor-parallel sharding on CPU ranks (gloo): a TP=2 oracle forward over
sharded weights (heads, FFN shards, expert intermediate shards, vocab-parallel
head) computes the same logits as the unsharded model."""
import torch

from mp_util import run_ranks
from vllm_moet_b200.config import tiny_config
from vllm_moet_b200.models import reference as ref
from vllm_moet_b200.models.weights import random_weights


def _tp_forward(rank, world, hc=1):
    import torch.distributed as dist
    cfg = tiny_config(hc_mult=hc)
    toks = torch.tensor([5, 17, 300, 42, 7, 99, 3, 250])
    pos = torch.arange(len(toks))
    cs = ref.rope_cos_sin(cfg, 64)
    full = random_weights(cfg, "cpu", seed=3)
    want, _ = ref.forward(full, toks, pos, cs)
    mw = random_weights(cfg, "cpu", seed=3, tp_rank=rank, tp_size=world)
    with ref.tp_context(dist.group.WORLD):
        got, hid = ref.forward(mw, toks, pos, cs)
        nxt = torch.cat([toks[1:], got[-1:].argmax(-1)])
        mtp_got, _ = ref.mtp_forward(mw, hid, nxt, pos, cs)
    mtp_want, _ = ref.mtp_forward(full, ref.forward(full, toks, pos, cs)[1], nxt, pos, cs)
    return (float((got - want).abs().max()), float(want.abs().max()),
            float((mtp_got - mtp_want).abs().max()), mw.lm_head.shape[0], cfg.vocab)


def _tp_forward_hc(rank, world):
    return _tp_forward(rank, world, hc=4)


def test_tp2_forward_matches_single_rank():
    res = run_ranks(_tp_forward, 2) + run_ranks(_tp_forward_hc, 2)     # plain residual, then 4 hc streams
    for err, scale, mtp_err, v_local, vocab in res:
        assert v_local * 2 == vocab
        assert err <= 1e-4 * max(scale, 1.0), (err, scale)
        assert mtp_err <= 1e-4 * max(scale, 1.0), mtp_err


def _ep_forward(rank, world):
    import torch.distributed as dist
    cfg = tiny_config()
    toks = torch.tensor([5, 17, 300, 42, 7, 99, 3, 250])
    pos = torch.arange(len(toks))
    cs = ref.rope_cos_sin(cfg, 64)
    want, _ = ref.forward(random_weights(cfg, "cpu", seed=4), toks, pos, cs)
    mw = random_weights(cfg, "cpu", seed=4, tp_rank=rank, tp_size=world, expert_parallel=True)
    ex = mw.layers[0].experts
    with ref.tp_context(dist.group.WORLD):
        got, _ = ref.forward(mw, toks, pos, cs)
    return float((got - want).abs().max()), float(want.abs().max()), ex.e_lo, ex.n_local


def test_ep2_forward_matches_single_rank():
    """Expert parallelism inside the TP group: each rank holds half of the experts
    whole (attention still head-sharded); the summed partials equal one rank."""
    res = run_ranks(_ep_forward, 2)
    assert [(r[2], r[3]) for r in res] == [(0, 4), (4, 4)]
    for err, scale, _, _ in res:
        assert err <= 1e-4 * max(scale, 1.0), (err, scale)


def _tp_prefix_chunked(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, tensor_parallel_size=world,
              tp_group=dist.group.WORLD, tp_rank=rank, enable_prefix_caching=True, prefix_block_size=8,
              enable_chunked_prefill=True, max_num_batched_tokens=8)
    pre = list(range(3, 35))
    sp = SamplingParams(max_tokens=8, ignore_eos=True, presence_penalty=0.5)
    outs = [llm.generate([pre + [40 + i]], sp)[0].outputs[0].token_ids for i in range(2)]
    return outs, llm.runner.prefix_stats["hits"]


def test_tp2_prefix_cache_chunked_prefill_and_penalties_match_one_rank():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    res = run_ranks(_tp_prefix_chunked, 2)
    one = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    pre = list(range(3, 35))
    sp = SamplingParams(max_tokens=8, ignore_eos=True, presence_penalty=0.5)
    want = [one.generate([pre + [40 + i]], sp)[0].outputs[0].token_ids for i in range(2)]
    for outs, hits in res:
        assert outs == want and hits == 1


def _tp_unseeded_sampling(rank, world):
    import random

    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    random.seed(1000 + rank)      # each rank's Python RNG differs, as OS seeding makes it
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256,
              tensor_parallel_size=world, tp_group=dist.group.WORLD, tp_rank=rank)
    sp = SamplingParams(max_tokens=12, ignore_eos=True, temperature=1.0)
    return [o.outputs[0].token_ids for o in llm.generate([[5, 6, 7, 8], [9, 10, 11]], sp)]


def test_tp2_unseeded_sampling_agrees_across_ranks():
    """Unseeded temperature > 0 requests draw one seed per request on TP rank 0, shared by
    every rank, so both ranks emit the same tokens."""
    a, b = run_ranks(_tp_unseeded_sampling, 2)
    assert a == b


def _tp_forward_replicated_attention(rank, world):
    import torch.distributed as dist
    cfg = tiny_config()
    toks = torch.tensor([5, 17, 300, 42, 7, 99, 3, 250])
    pos = torch.arange(len(toks))
    cs = ref.rope_cos_sin(cfg, 64)
    want, _ = ref.forward(random_weights(cfg, "cpu", seed=6), toks, pos, cs)
    mw = random_weights(cfg, "cpu", seed=6, tp_rank=rank, tp_size=world, attn_tp=False)
    lw = mw.layers[0]
    with ref.tp_context(dist.group.WORLD):
        got, _ = ref.forward(mw, toks, pos, cs)
    return float((got - want).abs().max()), float(want.abs().max()), lw.attn_tp, tuple(lw.o.shape)


def test_tp2_replicated_attention_matches_single_rank():
    """Replicated TP attention (whole attention on every rank, experts / FFN sharded): the
    attention output is not reduced, the FFN partials are, and the logits equal one rank."""
    res = run_ranks(_tp_forward_replicated_attention, 2)
    cfg = tiny_config()
    for err, scale, attn_tp, o_shape in res:
        assert not attn_tp and o_shape == (cfg.hidden, cfg.num_heads * cfg.v_head_dim)
        assert err <= 1e-4 * max(scale, 1.0), (err, scale)
