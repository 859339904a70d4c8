"""LLM.beam_search on the CPU engine against an independent beam search over the fp32
oracle's full-recompute log-probabilities, plus width 1 = greedy and the EOS / length
bookkeeping."""
import pytest
import torch

from vllm_moet_b200 import BeamSearchParams, SamplingParams
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.models import reference


@pytest.fixture(scope="module")
def llm():
    return LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=128)


def _oracle_beams(mw, prompt, W, steps, length_penalty=1.0):
    cs = reference.rope_cos_sin(mw.cfg, 128)
    beams = [(list(prompt), 0.0)]
    for _ in range(steps):
        cand = []
        for toks, cum in beams:
            t = torch.tensor(toks)
            lg, _ = reference.forward(mw, t, torch.arange(len(toks)), cs)
            lp = torch.log_softmax(lg[-1].double(), -1)
            v, i = torch.topk(lp, 2 * W)
            for vv, ii in zip(v.tolist(), i.tolist()):
                cand.append((toks + [ii], cum + vv))
        cand.sort(key=lambda c: (-c[1], c[0]))
        beams = cand[:W]
    n = steps
    return sorted(beams, key=lambda b: (-(b[1] / n ** length_penalty), b[0]))


def test_width_one_is_greedy(llm):
    p = [5, 9, 17, 33, 2, 8]
    out = llm.beam_search([p], BeamSearchParams(beam_width=1, max_tokens=6, ignore_eos=True))[0]
    greedy = llm.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids
    assert len(out.sequences) == 1 and out.sequences[0].generated == greedy
    assert out.sequences[0].finish_reason == "length"


@pytest.mark.parametrize("W", [2, 3])
def test_beams_match_the_oracle(llm, W):
    g = torch.Generator().manual_seed(W)
    prompts = [torch.randint(3, 1024, (n,), generator=g).tolist() for n in (7, 12)]
    outs = llm.beam_search(prompts, BeamSearchParams(beam_width=W, max_tokens=4, ignore_eos=True))
    for p, o in zip(prompts, outs):
        want = _oracle_beams(llm.mw, p, W, 4)
        assert [s.tokens for s in o.sequences] == [b[0] for b in want]
        for s, b in zip(o.sequences, want):
            assert s.cum_logprob == pytest.approx(b[1], abs=1e-3)
            assert len(s.logprobs) == 4 and s.text is not None
        # best first
        scores = [s.cum_logprob for s in o.sequences]
        assert scores == sorted(scores, reverse=True)


def test_eos_finishes_a_beam(llm, monkeypatch):
    p = [5, 9, 17, 33]
    first = llm.beam_search([p], BeamSearchParams(beam_width=2, max_tokens=1, ignore_eos=True))[0]
    top = first.sequences[0].generated[0]
    monkeypatch.setattr(llm.tokenizer, "eos_token_id", top, raising=False)
    out = llm.beam_search([p], BeamSearchParams(beam_width=2, max_tokens=3, length_penalty=0.0))[0]
    fin = [s for s in out.sequences if s.finish_reason == "stop"]
    assert fin and all(s.generated[-1] == top for s in fin)
    assert all(s.finish_reason in ("stop", "length") for s in out.sequences)
    with pytest.raises(ValueError):
        BeamSearchParams(beam_width=0, max_tokens=1)
