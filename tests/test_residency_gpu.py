"""GPU expert cache end to end: a decode served from a host store through a
small GPU cache (misses counted in-graph, fetched, replayed to a fixed point)
emits exactly the tokens of the fully resident engine."""
import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import ds4_flash_config
from vllm_moet_b200.engine.llm import LLM

pytestmark = pytest.mark.gpu


def _cfg():
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(3, 2048, (n,), generator=g).tolist() for n in (29, 50)]


@pytest.fixture(scope="module")
def resident_tokens():
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2)
    out = [o.outputs[0].token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    del llm
    torch.cuda.empty_cache()
    return out


@pytest.mark.parametrize("kind", ["pinned", "tiered"])
def test_cached_experts_match_resident(resident_tokens, kind, tmp_path):
    # 3 MoE layers (2 main + MTP) x 16 experts = 48; a 40-slot cache forces evictions and replays
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              expert_cache_slots=40, expert_store=kind, expert_store_dir=str(tmp_path))
    out = [o.outputs[0].token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    assert out == resident_tokens
    st = llm.cache.stats
    assert st["fetched_rows"] > 0
    assert llm.replay.stats["steps"] > 0
    llm.cache.close()
