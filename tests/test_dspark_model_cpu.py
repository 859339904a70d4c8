"""The DSpark draft model (models/dspark_model.py): non-causal block attention over a
sliding-window context derived from the target's aux hidden states, the sequential
Markov walk and the survival curve, and the engine running it (output = the target's
greedy sequence whatever the drafts)."""
import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import tiny_config
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.models import reference as ref
from vllm_moet_b200.models.dspark_model import (DSparkModelDrafter, block_attention, random_dspark_weights)
from vllm_moet_b200.models.weights import random_weights


def _setup(hc=1, window=8, block=4):
    cfg = tiny_config(hc_mult=hc)
    mw = random_weights(cfg, "cpu", seed=0)
    dw = random_dspark_weights(mw, num_layers=2, window=window)
    cs = ref.rope_cos_sin(cfg, 256)
    return cfg, mw, dw, DSparkModelDrafter(mw, dw, block, cs), cs


def _context(d, mw, cs, toks):
    aux = d.aux_request()
    ref.forward(mw, torch.tensor(toks), torch.arange(len(toks)), cs, ref.RefKV(len(mw.layers)), aux=aux)
    c = d.new_context()
    d.extend(c, aux, 0, len(toks))
    return c


def test_block_attention_is_non_causal():
    cfg, mw, dw, d, cs = _setup()
    lw = dw.layers[0]
    x = torch.randn(4, cfg.hidden)
    pos = torch.arange(10, 14)
    a = block_attention(cfg, lw, x, pos, cs, None, None)
    x2 = x.clone()
    x2[3] += 1.0                                        # a later block position ...
    b = block_attention(cfg, lw, x2, pos, cs, None, None)
    assert (a[0] - b[0]).abs().max() > 1e-4            # ... changes the first one's output


def test_context_window_and_dependence():
    cfg, mw, dw, d, cs = _setup(window=8)
    c = _context(d, mw, cs, list(range(5, 25)))
    assert c.end == 20 and all(k.shape[1] == 8 for k in c.k)
    dr, base, surv = d.propose_one(c, 7, 20)
    assert dr.shape == (4,) and base.shape == (4, cfg.vocab)
    assert bool((surv[1:] <= surv[:-1] + 1e-7).all()) and bool(((surv > 0) & (surv < 1)).all())
    c2 = _context(d, mw, cs, list(range(30, 50)))        # another context: other base logits
    _, base2, _ = d.propose_one(c2, 7, 20)
    assert (base - base2).abs().max() > 1e-4


def test_markov_walk_follows_the_transition_bias():
    cfg, mw, dw, d, cs = _setup()
    V, r = dw.markov_w1.shape
    # rank-r transition t -> t + 1 for tokens 0..r-2: embed t as e_t, map e_t to a huge bias on t + 1
    dw.markov_w1.zero_()
    dw.markov_w2.zero_()
    for t in range(r - 1):
        dw.markov_w1[t, t] = 1.0
        dw.markov_w2[t + 1, t] = 1e4
    c = _context(d, mw, cs, [5, 6, 7, 8])
    dr, _, _ = d.propose_one(c, 3, 4)
    assert dr.tolist() == [4, 5, 6, 7]


@pytest.mark.parametrize("hc", [1, 4])
def test_engine_with_the_dspark_model(hc):
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
              dspark={"block": 4, "tau": 0.0, "budget_frac": 1.0, "layers": 2, "window": 16},
              **({"hc_mult": hc} if hc > 1 else {}))
    assert hasattr(llm.runner.dspark["drafter"], "extend")
    prompts = [[5, 6, 7, 8, 9], [11, 12, 13]]
    sp = SamplingParams(max_tokens=10, ignore_eos=True)
    out = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    assert out == [ref.greedy_generate(llm.mw, p, 10) for p in prompts]
    assert llm.stats["steps"] > 0


def test_dflash_is_the_context_drafter_without_markov_heads():
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dflash",
              dspark={"block": 3})
    d = llm.runner.dspark["drafter"]
    assert d.markov is False and llm.runner.dspark["tau"] == 0.0
    p = [5, 6, 7, 8]
    assert llm.generate([p], SamplingParams(max_tokens=9, ignore_eos=True))[0].outputs[0].token_ids == \
        ref.greedy_generate(llm.mw, p, 9)
    c = d.new_context()
    aux = d.aux_request()
    ref.forward(llm.mw, torch.tensor(p), torch.arange(4), d.cs, ref.RefKV(len(llm.mw.layers)), aux=aux)
    d.extend(c, aux, 0, 4)
    dr, base, surv = d.propose_one(c, 9, 4)
    assert dr.tolist() == base.argmax(-1).tolist() and bool((surv == 1).all())


def test_prefix_cache_restores_the_dspark_context():
    """Prefix caching with the DSpark context drafter: the cached prefix carries the
    drafter's window at its end, so a hit drafts exactly as a cold run (same steps and
    acceptance) and still emits the target's greedy tokens; chunked prefill cuts the
    context at every block boundary the same way."""
    kw = dict(device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
              dspark={"block": 3, "tau": 0.0, "budget_frac": 1.0, "window": 12})
    cold = LLM("tiny-moe", **kw)
    warm = LLM("tiny-moe", enable_prefix_caching=True, prefix_block_size=8, enable_chunked_prefill=True,
               max_num_batched_tokens=5, **kw)
    pre = list(range(3, 27))
    sp = SamplingParams(max_tokens=9, ignore_eos=True)
    for tail in ([40, 41], [50]):
        p = pre + tail
        a = cold.generate([p], sp)[0].outputs[0].token_ids
        b = warm.generate([p], sp)[0].outputs[0].token_ids
        assert a == b == ref.greedy_generate(cold.mw, p, 9)
        assert warm.stats["accepted"] == cold.stats["accepted"]
    assert warm.runner.prefix_stats["hits"] == 1
