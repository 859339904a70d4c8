"""Sequence-parallel prefill on GPUs (BASELINE config 4's prefill, replicated weights): each
rank runs one block-aligned chunk of a long prompt through every layer and the ranks
all-gather each layer's cache blocks before its attention.  Tokens must equal a one-GPU
chunked prefill with the same chunk size (the same chunks, the same cache contents), on
every rank."""
import pytest
import torch

from mp_util import run_ranks

pytestmark = pytest.mark.gpu


def _cfg():
    from vllm_moet_b200.config import ds4_flash_config
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


def _sp_engine(rank, world, lens):
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    g = torch.Generator().manual_seed(17)
    prompts = [torch.randint(3, 2048, (n,), generator=g).tolist() for n in lens]
    sp = SamplingParams(max_tokens=8, ignore_eos=True)
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=2, seed=0,
              sp_group=dist.group.WORLD)
    got, chunks = [], []
    for p in prompts:
        got.append(llm.generate([p], sp)[0].outputs[0].token_ids)
        chunks.append(llm.runner.sp_chunk(len(p)))
    assert int(llm.runner.status) == 0
    del llm
    torch.cuda.empty_cache()
    want = []
    for p, tc in zip(prompts, chunks):
        ref = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=2, seed=0,
                  enable_chunked_prefill=True, max_num_batched_tokens=tc)
        want.append(ref.generate([p], sp)[0].outputs[0].token_ids)
        del ref
    return got, want, chunks


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sp2_prefill_matches_chunked_prefill():
    res = run_ranks(_sp_engine, 2, [300, 700], backend="nccl", env={"NCCL_NVLS_ENABLE": "0"})
    (g0, w0, c0), (g1, w1, c1) = res
    assert c0 == [192, 384]
    assert g0 == w0 and g1 == w1 and g0 == g1
