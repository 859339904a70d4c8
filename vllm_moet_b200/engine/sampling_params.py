"""vLLM-style request parameters and outputs."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, List, Optional


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0        # 0 = greedy (the MTP verify path is greedy)
    top_p: float = 1.0
    top_k: int = 0
    seed: Optional[int] = None
    stop_token_ids: List[int] = field(default_factory=list)
    ignore_eos: bool = False        # ignore the EOS token only; stop_token_ids and stop still apply
    stop: List[str] = field(default_factory=list)        # stop strings (output text is cut before them)
    include_stop_str_in_output: bool = False
    min_tokens: int = 0             # no stop condition before this many tokens
    logprobs: Optional[int] = None  # per generated token: the chosen token's and the top-N log-probabilities
    n: int = 1                      # completions per prompt (copies i > 0 sample with seed + i when seeded)
    prompt_logprobs: Optional[int] = None   # per prompt token after the first: its and the top-N log-probabilities
    # logits processing (CPU engine), in vLLM's semantics
    presence_penalty: float = 0.0   # minus this for every token already generated
    frequency_penalty: float = 0.0  # minus this times the token's count in the generated text
    repetition_penalty: float = 1.0  # tokens of the prompt or the output: positive logits / r, negative * r
    logit_bias: Optional[Dict[int, float]] = None   # token id -> added to its logit
    min_p: float = 0.0              # sampling: drop tokens below min_p x the top token's probability
    allowed_token_ids: Optional[List[int]] = None   # only these tokens can be chosen (vLLM's field)
    bad_words: Optional[List[str]] = None           # never generate these words (vLLM's field)
    bad_word_ids: Optional[List[List[int]]] = None  # the same as token sequences (filled from bad_words)

    def __post_init__(self):
        if isinstance(self.stop, str):
            self.stop = [self.stop]
        self.stop = [x for x in self.stop if x]
        if self.max_tokens < 1:
            raise ValueError("max_tokens must be >= 1")
        if not 0 <= self.min_tokens <= self.max_tokens:
            raise ValueError("min_tokens must be in [0, max_tokens]")
        if self.n < 1:
            raise ValueError("n must be >= 1")
        if self.temperature < 0:
            raise ValueError("temperature must be >= 0")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must be in (0, 1]")
        if self.repetition_penalty <= 0:
            raise ValueError("repetition_penalty must be > 0")
        if not 0 <= self.min_p <= 1:
            raise ValueError("min_p must be in [0, 1]")
        if not -2 <= self.presence_penalty <= 2 or not -2 <= self.frequency_penalty <= 2:
            raise ValueError("presence_penalty and frequency_penalty must be in [-2, 2]")
        if self.logit_bias:
            self.logit_bias = {int(k): float(v) for k, v in self.logit_bias.items()}
        if isinstance(self.bad_words, str):
            self.bad_words = [self.bad_words]
        if self.bad_word_ids is not None:
            self.bad_word_ids = [[int(t) for t in w] for w in self.bad_word_ids if len(w)]
        if self.allowed_token_ids is not None:
            self.allowed_token_ids = sorted({int(t) for t in self.allowed_token_ids})
            if not self.allowed_token_ids:
                raise ValueError("allowed_token_ids must not be empty")

    @property
    def processes_logits(self) -> bool:
        """Whether the logits are changed before choosing a token (penalties, bias)."""
        return bool(self.presence_penalty or self.frequency_penalty or self.repetition_penalty != 1.0
                    or self.logit_bias or self.allowed_token_ids is not None or bool(self.bad_words)
                    or bool(self.bad_word_ids))


def find_stop(text: str, stops: List[str], start: int = 0):
    """-> (index, stop string) of the earliest stop string in text[start:], or None."""
    best = None
    for s in stops:
        i = text.find(s, start)
        if i >= 0 and (best is None or i < best[0]):
            best = (i, s)
    return best


def cut_at_stop(text: str, stops: List[str], include: bool = False):
    """-> (text up to the first stop string, the stop string or None)."""
    hit = find_stop(text, stops)
    if hit is None:
        return text, None
    i, s = hit
    return text[: i + (len(s) if include else 0)], s


@dataclass
class CompletionOutput:
    index: int
    text: str
    token_ids: List[int]
    finish_reason: Optional[str] = None
    stop_reason: Optional[object] = None      # the stop token id or stop string that ended the request
    logprobs: Optional[List[Dict[int, float]]] = None   # per token: {token id: log-probability}
    cumulative_logprob: Optional[float] = None


@dataclass
class RequestOutput:
    request_id: str
    prompt_token_ids: List[int]
    outputs: List[CompletionOutput]
    finished: bool = True
    metrics: dict = field(default_factory=dict)
    prompt_logprobs: Optional[List[Optional[Dict[int, float]]]] = None   # None for the first prompt token


def logprob_entries(logits, tokens, top_n: int):
    """logits [n, V] (the rows that predicted `tokens`) -> [{token: logprob}] with the chosen
    token and the top_n alternatives of each row (raw model distribution, before sampling
    filters)."""
    import torch
    lp = torch.log_softmax(logits.float(), dim=-1)
    tok = torch.as_tensor(tokens, device=lp.device).long().view(-1, 1)
    chosen = lp.gather(1, tok).squeeze(1).cpu().tolist()
    out = []
    if top_n and top_n > 0:
        v, i = torch.topk(lp, min(top_n, lp.shape[-1]), dim=-1)
        v, i = v.cpu().tolist(), i.cpu().tolist()
    for r, t in enumerate(tok.view(-1).tolist()):
        d = {int(t): float(chosen[r])}
        if top_n and top_n > 0:
            for tt, vv in zip(i[r], v[r]):
                d.setdefault(int(tt), float(vv))
        out.append(d)
    return out


def shared_seeds(n: int, group=None, device=None) -> list:
    """n random seeds for unseeded sampling requests, the same on every rank of `group`.

    Each rank's RNG is seeded independently (Python's from the OS), so ranks that drew
    their own seeds would sample different tokens, write their KV shards for different
    sequences and stop at different steps, and the next collective would hang.  Rank 0
    of the group draws; the draws are broadcast.  Every rank must call this at the same
    point (admission is identical on every rank)."""
    import random
    seeds = [random.getrandbits(62) for _ in range(n)]
    if group is None or n == 0:
        return seeds
    import torch
    import torch.distributed as dist
    dev = device if (device is not None and dist.get_backend(group) == "nccl") else torch.device("cpu")
    t = torch.tensor(seeds, dtype=torch.int64, device=dev)
    dist.broadcast(t, src=dist.get_global_rank(group, 0), group=group)
    return t.tolist()
