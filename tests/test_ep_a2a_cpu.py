"""Expert parallelism with all-to-all dispatch / combine on gloo ranks: each rank's
tokens get the MoE output the single-rank block computes; the combine is
bit-identical across repeats."""
import torch

from mp_util import run_ranks


def _ep_rank(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200.config import tiny_config
    from vllm_moet_b200.models import reference as ref
    from vllm_moet_b200.models.weights import random_weights
    from vllm_moet_b200.parallel.ep import ep_moe_block
    cfg = tiny_config()
    mw = random_weights(cfg, "cpu", seed=0, with_mtp=False)
    lw = next(l for l in mw.layers if l.is_moe)
    g = torch.Generator().manual_seed(100 + rank)
    h = torch.randn(5 + 3 * rank, cfg.hidden, generator=g)        # data-parallel: different tokens per rank
    got = ep_moe_block(cfg, lw, h, dist.group.WORLD)
    again = ep_moe_block(cfg, lw, h, dist.group.WORLD)
    want = ref.moe_block(cfg, lw, h)
    return float((got - want).abs().max() / want.abs().max()), torch.equal(got, again)


def test_ep_a2a_matches_single_rank():
    for world in (2, 4):
        for err, same in run_ranks(_ep_rank, world):
            assert err < 1e-5 and same, (world, err)


def test_dispatch_bytes():
    from vllm_moet_b200.parallel.ep import dispatch_bytes, expert_owner
    assert dispatch_bytes(32, 8, 4096, 8) == (32 * 8 * 7 // 8 * 4096 * 2,) * 2
    assert expert_owner(torch.tensor([0, 31, 32, 255]), 256, 8).tolist() == [0, 0, 1, 7]


def _dp_ep_engine(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, ep_group=dist.group.WORLD)
    assert all(lw.experts.n_local == 8 // world for lw in llm.mw.layers if lw.is_moe)
    # data-parallel: every rank serves different requests, different counts and lengths
    prompts = [[5 + rank, 6, 7, 8], [40, 41 + rank]][: 1 + rank % 2]
    lens = [6 + 3 * rank, 4]
    out = llm.generate(prompts, [SamplingParams(max_tokens=lens[i], ignore_eos=True) for i in range(len(prompts))])
    return prompts, lens, [o.outputs[0].token_ids for o in out]


def test_dp_attention_ep_moe_engine_matches_single_rank():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    one = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    for prompts, lens, got in run_ranks(_dp_ep_engine, 2):
        want = [one.generate([p], SamplingParams(max_tokens=n, ignore_eos=True))[0].outputs[0].token_ids
                for p, n in zip(prompts, lens)]
        assert got == want
