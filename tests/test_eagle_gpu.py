"""EAGLE-3 drafting on the GPU runner: the draft module reads the target's aux hidden
states (residual after the target layers, concatenated, through fc), drafts chain on the
draft layer's own output, and verification keeps the greedy output: the EAGLE-3 engine
emits exactly the MTP engine's tokens on the same target weights, and its first draft
pass matches the fp32 oracle of the module."""
import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import ds4_flash_config
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.models import reference
from vllm_moet_b200.models.eagle3_model import eagle3_forward

pytestmark = pytest.mark.gpu


def _cfg():
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


def _prompt(n, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(3, 2048, (n,), generator=g).tolist()


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def test_eagle3_first_draft_pass_matches_oracle():
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=1, speculative_method="eagle3", max_model_len=1024,
              max_num_seqs=2)
    assert llm.runner.eagle is not None and llm.runner.k == 1
    p = _prompt(70, 11)
    st = llm._state(1)
    blocks = llm.blocks.allocate("e3", 200)
    bt = torch.zeros(1, llm.max_blocks, dtype=torch.int32)
    bt[0, :len(blocks)] = torch.tensor(blocks)
    st.block_table.copy_(bt)
    first = llm.runner.prefill([p], [bt[0].tolist()], [0], st)
    mlg = llm.runner.ws_prefill.bufs[("mtp.logits", torch.float32)][: llm.cfg.vocab].clone()
    d1 = int(st.tokens[0, 1])
    llm.blocks.release("e3")
    cs = reference.rope_cos_sin(llm.cfg, 256, "cuda")
    t = torch.tensor(p, device="cuda")
    pos = torch.arange(len(p), device="cuda")
    ref, aux = reference.forward(llm.mw, t, pos, cs)
    assert aux.shape == (len(p), 3 * llm.cfg.hidden)
    nxt = torch.cat([t[1:], first[:1].to(t.dtype)])
    mref, _ = eagle3_forward(llm.mw, aux, nxt, pos, cs)
    e = _rel(mlg, mref[-1])
    assert e < 0.1, e
    assert float(mref[-1][d1]) >= float(mref[-1].max()) - 0.3


def test_eagle3_engine_keeps_greedy_output():
    prompts = [_prompt(40, 12), _prompt(77, 13)]
    sp = SamplingParams(max_tokens=12, ignore_eos=True)
    e3 = LLM(_cfg(), device="cuda", num_speculative_tokens=2, speculative_method="eagle3", max_model_len=1024,
             max_num_seqs=2, seed=0)
    got = [o.outputs[0].token_ids for o in e3.generate(prompts, sp)]
    assert e3.stats["steps"] > 0
    del e3
    torch.cuda.empty_cache()
    mtp = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=1024, max_num_seqs=2, seed=0)
    want = [o.outputs[0].token_ids for o in mtp.generate(prompts, sp)]
    assert got == want
