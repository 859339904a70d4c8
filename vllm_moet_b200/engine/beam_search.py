"""Beam search over the engine's public generation API (``LLM.beam_search``).

vLLM (the reference's engine) offers ``LLM.beam_search(prompts, BeamSearchParams)``: every
step extends each live beam by one token, scores the candidates by cumulative
log-probability, keeps the best ``beam_width`` per prompt, and ranks the finished beams
by a length-penalised score ``cum_logprob / len ** length_penalty``.  Here every step is
one batched ``LLM.generate`` call (greedy, one token, ``logprobs=2·beam_width``) over all
live beams of all prompts, so the same code serves the CPU and the GPU engine; with
prefix caching enabled the engine reuses the beams' shared prefixes.  Beams that emit EOS
(unless ``ignore_eos``) finish; the rest run to ``max_tokens``.  Ties in cumulative
log-probability keep the lower token sequence, so a search is deterministic.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class BeamSearchParams:
    beam_width: int
    max_tokens: int
    ignore_eos: bool = False
    length_penalty: float = 1.0

    def __post_init__(self):
        if self.beam_width < 1:
            raise ValueError("beam_width must be >= 1")
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")


@dataclass
class BeamSearchSequence:
    tokens: List[int]                       # prompt + generated
    logprobs: List[Dict[int, float]] = field(default_factory=list)   # per generated token
    cum_logprob: float = 0.0
    text: Optional[str] = None
    finish_reason: Optional[str] = None     # "stop" (EOS) or "length"
    num_prompt: int = 0

    @property
    def generated(self) -> List[int]:
        return self.tokens[self.num_prompt:]


@dataclass
class BeamSearchOutput:
    sequences: List[BeamSearchSequence]


def beam_score(seq: BeamSearchSequence, length_penalty: float) -> float:
    n = max(1, len(seq.generated))
    return seq.cum_logprob / (n ** length_penalty)


def search_steps(prompts: List[List[int]], params: BeamSearchParams, eos: Optional[int], decode):
    """The search as a generator: it yields the token lists to extend by one token and is
    sent back, for each, the {token: logprob} entries of its next position (at least the
    top 2·beam_width); it returns the BeamSearchOutputs.  Drivers: ``beam_search`` (the
    ``LLM`` API) and the OpenAI server's ``use_beam_search`` (async requests)."""
    W = params.beam_width
    live = [[BeamSearchSequence(list(p), num_prompt=len(p))] for p in prompts]
    done: List[List[BeamSearchSequence]] = [[] for _ in prompts]
    for _ in range(params.max_tokens):
        batch = [(pi, b) for pi, beams in enumerate(live) for b in beams]
        if not batch:
            break
        entries = yield [b.tokens for _, b in batch]
        cand: List[List[BeamSearchSequence]] = [[] for _ in prompts]
        for (pi, b), lp in zip(batch, entries):
            for tok, l in sorted(lp.items(), key=lambda kv: (-kv[1], kv[0]))[:2 * W]:
                cand[pi].append(BeamSearchSequence(b.tokens + [tok], b.logprobs + [lp], b.cum_logprob + l,
                                                   num_prompt=b.num_prompt))
        for pi, cs in enumerate(cand):
            cs.sort(key=lambda s: (-s.cum_logprob, s.tokens))
            keep = []
            for s in cs:
                if not params.ignore_eos and eos is not None and s.tokens[-1] == eos:
                    s.finish_reason = "stop"
                    done[pi].append(s)
                else:
                    keep.append(s)
                if len(keep) == W:
                    break
            live[pi] = keep
    results = []
    for pi in range(len(prompts)):
        for s in live[pi]:
            s.finish_reason = "length"
        seqs = sorted(done[pi] + live[pi], key=lambda s: (-beam_score(s, params.length_penalty), s.tokens))[:W]
        for s in seqs:
            s.text = decode(s.generated)
        results.append(BeamSearchOutput(seqs))
    return results


def step_params(params: BeamSearchParams):
    """The per-step request: greedy, one token, the top 2·beam_width log-probabilities."""
    from .sampling_params import SamplingParams
    return SamplingParams(max_tokens=1, temperature=0.0, logprobs=2 * params.beam_width, ignore_eos=True)


def beam_search(llm, prompts: List[List[int]], params: BeamSearchParams) -> List[BeamSearchOutput]:
    gen = search_steps(prompts, params, getattr(llm.tokenizer, "eos_token_id", None), llm.tokenizer.decode)
    sp = step_params(params)
    try:
        batch = next(gen)
        while True:
            outs = llm.generate(batch, sp)
            batch = gen.send([o.outputs[0].logprobs[0] for o in outs])
    except StopIteration as stop:
        return stop.value
