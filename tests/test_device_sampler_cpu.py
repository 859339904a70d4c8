"""The graph-safe batch sampler (spec/device_sampler.py) on CPU tensors: greedy rows
reproduce greedy verification, the emitted tokens follow token-by-token sampling from the
filtered target distribution, filters hold, and draws are reproducible per seed and
position."""
import torch

from vllm_moet_b200.spec.device_sampler import sample_verify, target_probs, uniform
from vllm_moet_b200.spec.rejection import filter_probs, greedy_accept


def _params(B, t=0.0, k=0, p=1.0, mp=0.0):
    return (torch.full((B,), t), torch.full((B,), k, dtype=torch.int32), torch.full((B,), p), torch.full((B,), mp))


def test_greedy_rows_equal_greedy_verification():
    g = torch.Generator().manual_seed(0)
    B, k, V = 16, 3, 50
    logits = torch.randn(B, k + 1, V, generator=g)
    am = logits.argmax(-1)
    drafts = torch.where(torch.rand(B, k, generator=g) < 0.6, am[:, :k], torch.randint(0, V, (B, k), generator=g))
    n, tok = sample_verify(logits, drafts, *_params(B), torch.arange(B), torch.full((B,), 7))
    n_ref, em = greedy_accept(am, drafts)
    assert torch.equal(n.long(), n_ref)
    for b in range(B):
        a = int(n_ref[b])
        assert tok[b, : a + 1].tolist() == em[b, : a + 1].tolist() and (tok[b, a:] == tok[b, a]).all()


def test_filters_match_filter_probs():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(6, 40, generator=g) * 2
    for t, k, p, mp in ((0.7, 0, 1.0, 0.0), (1.0, 5, 1.0, 0.0), (1.3, 0, 0.8, 0.0), (0.9, 10, 0.9, 0.05)):
        got = target_probs(x, *_params(6, t, k, p, mp))
        want = filter_probs(x, t, k, p, mp)
        assert torch.allclose(got, want, atol=1e-6), (t, k, p, mp)


def test_emitted_tokens_follow_sequential_sampling():
    """First token ~ p_0; given the first token equals draft d_0, the second ~ p_1 (the
    property that makes speculative sampling exact)."""
    g = torch.Generator().manual_seed(2)
    V, N = 6, 60000
    base = torch.randn(3, V, generator=g)
    logits = base[None].expand(N, -1, -1)
    drafts = torch.tensor([[int(base[0].argmax()), int(base[1].argmax())]]).expand(N, -1)
    t = 0.8
    n, tok = sample_verify(logits, drafts, *_params(N, t, 0, 0.9), torch.arange(N), torch.full((N,), 11))
    p = filter_probs(base, t, 0, 0.9)
    f0 = torch.bincount(tok[:, 0].long(), minlength=V).float() / N
    assert (f0 - p[0]).abs().max() < 0.01, (f0, p[0])
    sel = tok[:, 0] == drafts[0, 0]
    f1 = torch.bincount(tok[sel, 1].long(), minlength=V).float() / int(sel.sum())
    assert (f1 - p[1]).abs().max() < 0.015, (f1, p[1])
    assert set(tok[:, 0].tolist()) <= set(torch.nonzero(p[0] > 0).view(-1).tolist())


def test_draws_are_reproducible_per_seed_and_position():
    g = torch.Generator().manual_seed(3)
    B, V = 8, 100
    logits = torch.randn(B, 3, V, generator=g)
    drafts = torch.randint(0, V, (B, 2), generator=g)
    args = (logits, drafts, *_params(B, 1.0), torch.full((B,), 5), torch.arange(B) * 3)
    a, b = sample_verify(*args), sample_verify(*args)
    assert torch.equal(a[1], b[1]) and torch.equal(a[0], b[0])
    u1 = uniform(torch.tensor([5]), torch.tensor([10]), 1, 1000)
    u2 = uniform(torch.tensor([5]), torch.tensor([11]), 1, 1000)
    u3 = uniform(torch.tensor([6]), torch.tensor([10]), 1, 1000)
    assert not torch.equal(u1, u2) and not torch.equal(u1, u3)
    assert 0 < float(u1.min()) and float(u1.max()) < 1 and abs(float(u1.mean()) - 0.5) < 0.05


def _tp_sample(rank, world):
    import torch.distributed as dist
    from vllm_moet_b200.spec.device_sampler import gather_vocab
    g = torch.Generator().manual_seed(4)
    B, kp1, V = 4, 3, 48
    logits = torch.randn(B * kp1, V, generator=g) * 2
    drafts = torch.randint(0, V, (B, kp1 - 1), generator=g)
    per = V // world
    full = gather_vocab(logits[:, rank * per:(rank + 1) * per], dist.group.WORLD)
    args = (drafts, *_params(B, 0.8, 7, 0.9), torch.arange(B) + 100, torch.arange(B) * 5)
    got = sample_verify(full.view(B, kp1, V), *args)
    want = sample_verify(logits.view(B, kp1, V), *args)
    return torch.equal(full, logits), got[0].tolist(), got[1].tolist(), want[0].tolist(), want[1].tolist()


def test_vocab_parallel_sampling_agrees_across_ranks():
    """TP: the vocab shards gathered on every rank give the unsharded rows, so every rank
    draws the tokens one rank would."""
    from mp_util import run_ranks
    res = run_ranks(_tp_sample, 2)
    for same, n, tok, n_ref, tok_ref in res:
        assert same and n == n_ref and tok == tok_ref
    assert res[0][1:3] == res[1][1:3]


def test_batched_processing_equals_per_row_processing():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.spec.device_sampler import process_batch
    from vllm_moet_b200.spec.logits_process import process_logits
    g = torch.Generator().manual_seed(5)
    B, kp1, V = 3, 3, 40
    logits = torch.randn(B, kp1, V, generator=g) * 3
    drafts = torch.randint(0, V, (B, kp1 - 1), generator=g)
    sps = [SamplingParams(repetition_penalty=1.4, frequency_penalty=0.3, presence_penalty=0.1, logit_bias={3: 1.5}),
           SamplingParams(),
           SamplingParams(presence_penalty=-0.5, logit_bias={7: -2.0})]
    prompts = [[1, 2, 3], [4, 5], [6, 6, 9]]
    outs = [[3, 8, 8], [10], [9, 11]]
    counts = torch.zeros(B, V)
    mask = torch.zeros(B, V, dtype=torch.bool)
    bias = torch.zeros(B, V)
    for b in range(B):
        for t in outs[b]:
            counts[b, t] += 1
        mask[b, prompts[b]] = True
        for t, v in (sps[b].logit_bias or {}).items():
            bias[b, t] = v
    got = process_batch(logits, drafts, counts, mask, torch.tensor([p.repetition_penalty for p in sps]),
                        torch.tensor([p.frequency_penalty for p in sps]), torch.tensor([p.presence_penalty for p in sps]),
                        bias)
    for b in range(B):
        want = process_logits(logits[b], sps[b], prompts[b], outs[b], drafts[b].tolist())
        assert torch.allclose(got[b], want, atol=1e-5), b
    assert torch.equal(got[1], logits[1])


def _tp_logprob_rows(rank, world):
    import types
    import torch.distributed as dist
    from vllm_moet_b200.engine.llm import LLM
    full = torch.arange(6 * 8, dtype=torch.float32).view(6, 8)
    fake = types.SimpleNamespace(_tp_group=dist.group.WORLD, device=types.SimpleNamespace(type="cuda"))
    got = LLM._full_logits(fake, full[:, rank * 4:(rank + 1) * 4].clone())
    return torch.equal(got, full)


def test_logprob_rows_under_tp_are_whole_vocabulary():
    """GPU logprobs under TP: the verify / prefill rows are the ranks' vocab shards
    gathered back into whole rows."""
    from mp_util import run_ranks
    assert run_ranks(_tp_logprob_rows, 2) == [True, True]
