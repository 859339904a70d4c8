"""DSpark width scheduler (the reference's scheduler test semantics), the
DSpark block drafter, and the greedy / stochastic rejection samplers."""
import math

import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.spec import DSparkDrafter, allocate_widths, greedy_accept, rejection_sample


def test_width_never_exceeds_scheduled_length():
    w = allocate_widths(torch.ones(2, 4), torch.ones(4), num_reqs=2, length=2, tau=0.5, budget_frac=1.0)
    assert torch.equal(w, torch.tensor([2, 2], dtype=torch.int32))


def test_tied_budget_never_inflates():
    w = allocate_widths(torch.ones(3, 4), torch.ones(4), num_reqs=3, length=4, tau=0.0, budget_frac=0.25)
    assert int(w.sum()) == 3 and bool((w <= 4).all())


def test_zero_budget_allocates_nothing():
    w = allocate_widths(torch.rand(2, 4), torch.ones(4), num_reqs=2, length=4, tau=0.0, budget_frac=0.0)
    assert torch.equal(w, torch.zeros(2, dtype=torch.int32))


def test_calibration_projected_to_valid_prefix():
    w = allocate_widths(torch.tensor([[0.9, 0.8, 0.7, 0.6]]), torch.tensor([1.0, 0.1, 2.0, 2.0]),
                        num_reqs=1, length=4, tau=0.15, budget_frac=1.0)
    assert torch.equal(w, torch.tensor([1], dtype=torch.int32))


def test_budget_prefers_confident_requests():
    surv = torch.tensor([[0.9, 0.9, 0.9, 0.9], [0.5, 0.4, 0.3, 0.2]])
    w = allocate_widths(surv, torch.ones(4), num_reqs=2, length=4, tau=0.0, budget_frac=0.5)
    assert w.tolist() == [4, 0]
    # tau > 0 is a static confidence width per request, without a budget
    w = allocate_widths(surv, torch.ones(4), num_reqs=2, length=4, tau=0.35, budget_frac=0.5)
    assert w.tolist() == [4, 2]


def test_greedy_accept_valid_len():
    tgt = torch.tensor([[5, 6, 7, 8], [5, 6, 7, 8]])
    dr = torch.tensor([[5, 6, 9], [5, 6, 7]])
    n, em = greedy_accept(tgt, dr, valid_draft_len=torch.tensor([3, 1]))
    assert n.tolist() == [2, 1]
    assert em.tolist() == [[5, 6, 7, -1], [5, 6, -1, -1]]


def test_rejection_sampler_preserves_target_distribution():
    g = torch.Generator().manual_seed(0)
    V = 4
    p = torch.tensor([0.1, 0.2, 0.3, 0.4])
    q = torch.tensor([0.4, 0.3, 0.2, 0.1])
    N = 20000
    drafts = torch.multinomial(q.expand(N, V), 1, replacement=True, generator=g)
    tp = p.expand(N, 2, V).contiguous()
    dp = q.expand(N, 1, V).contiguous()
    n, em = rejection_sample(tp, dp, drafts, generator=g)
    first = em[:, 0]
    freq = torch.bincount(first, minlength=V).float() / N
    assert torch.allclose(freq, p, atol=0.015), freq


def test_dspark_drafter_shapes():
    torch.manual_seed(0)
    d = DSparkDrafter(hidden=32, vocab=50, block=4)
    drafts, probs, surv = d.propose(torch.randn(3, 32), torch.tensor([1, 2, 3]))
    assert drafts.shape == (3, 4) and probs.shape == (3, 4, 50)
    assert bool(((surv > 0) & (surv < 1)).all())
    assert torch.allclose(probs.sum(-1), torch.ones(3, 4))
    w = allocate_widths(surv, torch.ones(4), num_reqs=3, length=4, tau=0.0, budget_frac=0.5)
    assert int(w.sum()) <= 6


def test_dspark_swa_indices():
    from vllm_moet_b200.spec import swa_indices
    idx = swa_indices(context_len=1000, block_len=4, window=256)
    assert idx.numel() == 512 and idx.numel() % 128 == 0
    valid = idx[idx >= 0]
    assert valid.tolist() == list(range(744, 1004))
    big = swa_indices(context_len=5000, block_len=8, window=600)
    assert big.numel() == 640 and int((big >= 0).sum()) == 608


def test_quant_study_orders_formats():
    import torch
    from vllm_moet_b200.tools.quant_study import study
    r = study(torch.randn(64, 256) * 0.02)
    assert r["nvfp4"][0] < r["2-bit codebook (auto)"][0] and r["mxfp4 (delta tier)"][0] < r["2-bit codebook (auto)"][0]
    t = study(torch.randn(64, 256) * 0.02, trellis_L=8)
    # the trellis at 2 bits beats the 2-bit codebook at about the same bits, 3 bits beats both
    assert t["trellis 2-bit (L=8)"][0] < t["2-bit codebook (auto)"][0] < 1.0
    assert t["trellis 3-bit (L=8)"][0] < t["trellis 2-bit (L=8)"][0]
    assert 2.0 < t["trellis 2-bit (L=8)"][1] < 2.5


def test_filter_probs_top_k_top_p():
    from vllm_moet_b200.spec.rejection import filter_probs
    logits = torch.tensor([[4.0, 3.0, 2.0, 1.0, 0.0]])
    p = filter_probs(logits, 1.0, top_k=2)
    assert (p[0, 2:] == 0).all() and abs(float(p.sum()) - 1) < 1e-6
    full = torch.softmax(logits, -1)[0]
    p = filter_probs(logits, 1.0, top_p=float(full[0] + full[1]) - 1e-4)      # needs the top two
    assert (p[0, :2] > 0).all() and (p[0, 2:] == 0).all()
    p = filter_probs(logits, 1.0, top_p=0.01)                                  # always keeps the top token
    assert float(p[0, 0]) == 1.0
    cold = filter_probs(logits, 1e-3)
    assert float(cold[0, 0]) > 0.999


def test_engine_sampling_top1_equals_greedy_and_seeds_reproduce():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    prompts = [[5, 6, 7, 8, 9], [40, 41, 42]]
    greedy = [o.outputs[0].token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True))]
    top1 = [o.outputs[0].token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True,
                                                                                 temperature=0.9, top_k=1))]
    assert top1 == greedy                     # the whole sampling path (prefill, rejection, bonus) at top-1
    sp = SamplingParams(max_tokens=10, ignore_eos=True, temperature=1.5, seed=11)
    a = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    b = [o.outputs[0].token_ids for o in llm.generate(prompts, sp)]
    c = [o.outputs[0].token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True,
                                                                              temperature=1.5, seed=12))]
    assert a == b and a != c and a != greedy


def test_engine_first_token_distribution():
    """The first sampled token follows softmax(logits / T) of the reference model."""
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=64)
    p = [5, 6, 7, 8, 9]
    T = 0.02
    lg, _ = reference.forward(llm.mw, torch.tensor(p), torch.arange(len(p)), reference.rope_cos_sin(llm.cfg, 64))
    want = torch.softmax(lg[-1] / T, -1)
    top = torch.topk(want, 3)
    n = 300
    counts = torch.zeros_like(want)
    outs = llm.generate([p] * n, [SamplingParams(max_tokens=1, ignore_eos=True, temperature=T, seed=s)
                                  for s in range(n)])
    for o in outs:
        counts[o.outputs[0].token_ids[0]] += 1
    freq = counts / n
    for i in top.indices.tolist():
        sd = math.sqrt(float(want[i]) * (1 - float(want[i])) / n) + 1e-3
        assert abs(float(freq[i]) - float(want[i])) < 5 * sd, (i, float(freq[i]), float(want[i]))


def test_dspark_engine_verifies_blocks():
    """DSpark in the engine: whatever the drafter proposes, the output is the target's
    greedy sequence; an oracle drafter (the true continuation, confident) gets every
    allotted draft accepted and needs far fewer steps."""
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    p, n = [5, 6, 7, 8, 9], 12
    rnd = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
              dspark={"block": 4, "tau": 0.0, "budget_frac": 1.0})
    want = reference.greedy_generate(rnd.mw, p, n)
    assert rnd.generate([p], SamplingParams(max_tokens=n, ignore_eos=True))[0].outputs[0].token_ids == want
    full = p + want

    class Oracle:
        def __init__(self, runner):
            self.runner = runner

        def propose(self, h, last):
            (st,) = self.runner.rows.values()
            nxt = full[st["pos"] + 1: st["pos"] + 5]
            nxt = nxt + [0] * (4 - len(nxt))
            R = h.shape[0]
            return torch.tensor([nxt] * R), None, torch.ones(R, 4)
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
              dspark={"block": 4, "tau": 0.5, "budget_frac": 1.0})
    llm.runner.dspark["drafter"] = Oracle(llm.runner)
    out = llm.generate([p], SamplingParams(max_tokens=n, ignore_eos=True))[0].outputs[0].token_ids
    assert out == want
    assert llm.stats["accepted"] >= n - 4 and llm.stats["steps"] <= n // 5 + 2


def _process_oracle(logits, sp, prompt, hist):
    """One row, written out token by token (vLLM semantics)."""
    x = logits.float().clone()
    cnt = {}
    for t in hist:
        cnt[t] = cnt.get(t, 0) + 1
    for t in set(hist) | set(prompt):
        if sp.repetition_penalty != 1.0:
            x[t] = x[t] / sp.repetition_penalty if x[t] > 0 else x[t] * sp.repetition_penalty
    for t, c in cnt.items():
        x[t] -= sp.frequency_penalty * c + sp.presence_penalty
    for t, b in (sp.logit_bias or {}).items():
        x[t] += b
    return x


def test_penalties_and_bias_per_verify_row():
    """Row j of a verify pass is processed with the drafts before it counted as output."""
    from vllm_moet_b200.spec.logits_process import process_logits
    g = torch.Generator().manual_seed(0)
    V = 64
    logits = torch.randn(3, V, generator=g) * 3
    sp = SamplingParams(repetition_penalty=1.3, frequency_penalty=0.4, presence_penalty=0.2,
                        logit_bias={5: 2.0, 60: -1.5})
    prompt, out, drafts = [1, 2, 3, 2], [7, 9, 7], [9, 11]
    got = process_logits(logits, sp, prompt, out, drafts)
    for j in range(3):
        want = _process_oracle(logits[j], sp, prompt, out + drafts[:j])
        assert torch.allclose(got[j], want, atol=1e-6), j
    assert torch.equal(process_logits(logits, SamplingParams(), prompt, out, drafts), logits)


def test_min_p_filter():
    from vllm_moet_b200.spec.rejection import filter_probs
    logits = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]]))
    p = filter_probs(logits, 1.0, min_p=0.25)          # keeps p >= 0.125
    assert torch.allclose(p, torch.tensor([[0.5, 0.3, 0.15, 0.0]]) / 0.95)


def test_engine_penalties_match_token_by_token_decode():
    """The speculative CPU engine with penalties and bias emits what plain one-token greedy
    decoding over processed logits emits (drafts verified against processed rows)."""
    from vllm_moet_b200.models import reference as ref
    from vllm_moet_b200.spec.logits_process import process_logits
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    sp = SamplingParams(max_tokens=16, ignore_eos=True, repetition_penalty=1.5, frequency_penalty=0.5,
                        presence_penalty=0.3, logit_bias={100: 1.0})
    prompt = [5, 6, 7, 5, 6]
    got = llm.generate([prompt], sp)[0].outputs[0].token_ids
    cs = ref.rope_cos_sin(llm.cfg, 64)
    toks, out = list(prompt), []
    for _ in range(16):
        lg, _ = ref.forward(llm.mw, torch.tensor(toks), torch.arange(len(toks)), cs)
        t = int(process_logits(lg[-1:], sp, prompt, out)[0].argmax())
        out.append(t)
        toks.append(t)
    assert got == out
    assert got != llm.generate([prompt], SamplingParams(max_tokens=16, ignore_eos=True))[0].outputs[0].token_ids
    forced = llm.generate([prompt], SamplingParams(max_tokens=6, ignore_eos=True, logit_bias={42: 1e4}))
    assert forced[0].outputs[0].token_ids == [42] * 6


def test_eagle3_drafts_from_aux_hidden_states():
    """EAGLE-3 on the CPU engine: the target returns its concatenated aux states (low /
    middle / high layer), the draft layer chains on its own hidden state, and verification
    keeps the output equal to the target's greedy sequence, with and without prefix
    caching and chunked prefill."""
    from vllm_moet_b200.models import reference
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=3, max_model_len=256, speculative_method="eagle3",
              num_layers=3, enable_prefix_caching=True, prefix_block_size=4, enable_chunked_prefill=True,
              max_num_batched_tokens=6)
    ew = llm.mw.extra["eagle3"]
    assert ew.target_layers == (0, 1, 2) and llm.mw.mtp is None and llm.k == 3
    cs = reference.rope_cos_sin(llm.cfg, 64)
    t = torch.tensor([5, 6, 7, 8])
    _, hid = reference.forward(llm.mw, t, torch.arange(4), cs)
    assert hid.shape == (4, 3 * llm.cfg.hidden)
    lg, h = reference.mtp_forward(llm.mw, hid, torch.tensor([6, 7, 8, 9]), torch.arange(4), cs)
    assert lg.shape == (4, llm.cfg.vocab) and h.shape == (4, llm.cfg.hidden)
    lg2, _ = reference.mtp_forward(llm.mw, h[-1:], torch.tensor([3]), torch.tensor([4]), cs)   # chained step
    assert lg2.shape == (1, llm.cfg.vocab)
    prompts = [[5, 6, 7, 8, 9, 10, 11], [5, 6, 7, 8, 20]]
    out = [o.outputs[0].token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10, ignore_eos=True))]
    assert out == [reference.greedy_generate(llm.mw, p, 10) for p in prompts]
    with pytest.raises(NotImplementedError):       # the GPU runner drafts EAGLE-3 on one GPU per replica
        LLM("tiny-moe", device="cuda", speculative_method="eagle3", tensor_parallel_size=2)
    with pytest.raises(NotImplementedError):
        LLM("tiny-moe", device="cuda", speculative_method="eagle3", hc_mult=4)


def test_dspark_swa_indices_batch_equals_scalar():
    from vllm_moet_b200.spec import swa_indices, swa_indices_batch
    lens = torch.tensor([0, 1, 5, 255, 256, 257, 1000, 5000])
    for block, window, width in ((4, 256, 512), (8, 600, 640), (3, 16, 24)):
        got = swa_indices_batch(lens, block, window, width)
        assert got.shape == (len(lens), width) and got.dtype == torch.int32
        for b, c in enumerate(lens.tolist()):
            ref = swa_indices(c, block, window, min_width=1, align=1)
            want = torch.full((width,), -1, dtype=torch.int32)
            n = min(width, ref.numel())
            want[:n] = ref[:n]
            assert torch.equal(got[b], want), (c, block, window)
