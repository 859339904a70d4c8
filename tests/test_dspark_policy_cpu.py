"""DSpark's hardware-aware verify-length policy: the tokens/s choice over a cost table
with engine overhead and hysteresis, bucket lookups, the batch-size schedule and its
live re-derivation, the overhead regression, survival calibration, and the engine
running the policy."""
import pytest
import torch

from vllm_moet_b200.spec.dspark_policy import (DSparkPolicy, LiveRederivation, accept_curve, bucket_cost,
                                               derive_schedule, schedule_lookup, uniform_length)

R_GRID = [1, 4, 16]
# T(R, L): L = 0..3; verifying more drafts costs more, much more at 16 requests
TIMES = [[1.0, 1.2, 2.0], [1.05, 1.3, 3.0], [1.1, 1.4, 4.5], [1.2, 1.6, 6.5]]


def test_bucket_cost_rounds_up_and_extrapolates():
    assert bucket_cost(R_GRID, TIMES[0], 1) == 1.0
    assert bucket_cost(R_GRID, TIMES[0], 2) == 1.2        # padded to the 4-request bucket
    assert bucket_cost(R_GRID, TIMES[0], 32) == pytest.approx(4.0)


def test_uniform_length_maximises_tokens_per_second():
    acc = accept_curve([0.9, 0.8, 0.7], 3)
    assert acc == pytest.approx([0, 0.9, 1.7, 2.4])
    L1, _ = uniform_length(acc, 1, 3, R_GRID, TIMES)      # cheap drafts at 1 request: verify them all
    assert L1 == 3
    L16, t = uniform_length(acc, 16, 3, R_GRID, TIMES)     # costly at 16: fewer
    want = max(range(4), key=lambda L: 16 * (1 + acc[L]) / TIMES[L][2])
    assert L16 == want and t == pytest.approx(TIMES[want][2])
    # overhead per token favours longer verifies (more tokens per fixed cost)
    assert uniform_length(acc, 16, 3, R_GRID, TIMES, overhead=(5.0, 0.0))[0] >= L16
    assert uniform_length(acc, 1, 3, None, None) == (3, 0.0)     # no table: all drafts


def test_hysteresis_keeps_the_incumbent_within_five_percent():
    acc = accept_curve([0.5, 0.5, 0.5], 3)
    times = [[1.0], [1.0], [1.0], [1.0]]
    best, _ = uniform_length(acc, 1, 3, [1], times)
    assert best == 3
    # length 2 is within 5 % of length 3? tokens 2.0 vs 2.5 -> no, it switches
    assert uniform_length(acc, 1, 3, [1], times, current=2)[0] == 3
    times2 = [[1.0], [1.0], [1.0], [1.02]]
    acc2 = accept_curve([0.5, 0.5, 0.01], 3)
    assert uniform_length(acc2, 1, 3, [1], times2)[0] == 2
    assert uniform_length(acc2, 1, 3, [1], times2, current=3)[0] == 3     # 1 % worse: kept


def test_derived_schedule_and_lookup():
    tab = derive_schedule(R_GRID, TIMES, [0.9, 0.8, 0.7], max_num_reqs=32, c0=0.0, c1=0.0)
    assert tab[0][0] == 1 and tab[-1][1] == 32
    assert all(a[1] + 1 == b[0] for a, b in zip(tab, tab[1:]))            # contiguous ranges
    assert all(a[2] != b[2] for a, b in zip(tab, tab[1:]))                # equal neighbours merged
    look = schedule_lookup(tab, 32, 3)
    for lo, hi, L in tab:
        assert all(look[r] == L for r in range(lo, hi + 1))
    acc = accept_curve([0.9, 0.8, 0.7], 3)
    assert look[16] == uniform_length(acc, 16, 3, R_GRID, TIMES)[0]


def test_live_rederivation_tracks_measured_acceptance():
    lr = LiveRederivation(R_GRID, TIMES, 32, every=100, min_obs=10)
    res = None
    for i in range(100):
        res = lr.observe(3, 0)                      # nothing is ever accepted
    assert res is not None and lr.survival == [0.0, 0.0, 0.0]
    assert all(L == 0 for L in res[1:])            # drafting never pays: length 0 everywhere


def test_overhead_regression_recovers_c0_c1():
    t = [0.0]
    pol = DSparkPolicy(gamma=3, clock=lambda: t[0])
    pol.set_cost_table([1, 64], [[0.01, 0.02]] * 4)
    pol.ema = torch.tensor([0.5, 0.5, 0.5])
    c0, c1 = 0.004, 2e-4
    for i in range(60):
        R = 1 + (i * 7) % 60
        L = pol.begin_step(R, now=t[0])
        # wall time of this step = table prediction + true overhead
        t[0] += pol._gpu_pred + c0 + c1 * pol._tokens
    assert pol.c0 == pytest.approx(c0, rel=0.05) and pol.c1 == pytest.approx(c1, rel=0.05)
    assert 0 <= L <= 3


def test_calibration_follows_realised_acceptance():
    pol = DSparkPolicy(gamma=2)
    surv = torch.full((32, 2), 0.8)
    for _ in range(8):
        # predicted 0.8 at both positions, realised: position 1 always, position 2 half the time
        acc = torch.tensor([2 if i % 2 else 1 for i in range(32)])
        pol.observe(surv, torch.full((32,), 2), acc, 2)
    assert float(pol.cal[0]) > 1.1 and float(pol.cal[1]) < 0.8
    assert pol.survival_curve()[0] == pytest.approx(min(0.8 * float(pol.cal[0]), 1.0))


def test_engine_skips_drafts_when_the_table_says_they_never_pay():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference
    times = [[0.001, 0.004]] + [[10.0, 40.0]] * 4         # verifying any draft costs 10 s
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
              dspark={"block": 4, "tau": 0.0, "budget_frac": 1.0, "cost_table": ([1, 4], times)})
    p = [5, 6, 7, 8]
    out = llm.generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0].outputs[0].token_ids
    assert out == reference.greedy_generate(llm.mw, p, 8)
    pol = llm.runner.dspark["policy"]
    assert pol.history[0] == 4 and all(L == 0 for L in pol.history[1:])   # no survival yet, then the table
    prof = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
               dspark={"block": 2, "profile": True, "r_grid": [1, 2]})
    tab = prof.runner.dspark["policy"].times_by_l
    assert len(tab) == 3 and all(len(r) == 2 and min(r) > 0 for r in tab)
