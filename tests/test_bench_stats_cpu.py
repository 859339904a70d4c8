"""Quality-parity statistics of the bench harness against scipy and by hand."""
import math

import pytest
from scipy.stats import binomtest

from vllm_moet_b200.bench.stats import (binom_two_sided, compare, degenerate, mcnemar_exact, paired_token_stats,
                                        passes)


@pytest.mark.parametrize("k,n", [(0, 0), (1, 10), (5, 10), (3, 20), (12, 30)])
def test_binomial_tail_matches_scipy(k, n):
    want = 1.0 if n == 0 else binomtest(k, n, 0.5).pvalue
    assert binom_two_sided(k, n) == pytest.approx(want, rel=1e-9)


def test_compare_and_gates():
    base = {f"q{i}": {"correct": i % 3 != 0, "tokens": 100 + i} for i in range(30)}
    cand = {f"q{i}": {"correct": i % 3 != 0 or i == 3, "tokens": 110 + i} for i in range(30)}
    c = compare(base, cand, cap=200)
    assert c["only_base"] == 0 and c["only_cand"] == 1 and c["mcnemar_p"] == 1.0
    assert c["token_longer"] == 30 and c["token_sign_p"] < 1e-8
    assert 5 < c["token_ratio_median_delta_pct"] < 10
    assert passes(c, {"min_mcnemar_p": 0.05})
    assert not passes(c, {"max_abs_token_ratio_median_delta_pct": 5})
    assert not passes(c, {"min_token_sign_p": 0.05})
    st = paired_token_stats({"a": 10, "b": 20}, {"a": 20, "b": 10})
    assert st["ratio_geomean"] == pytest.approx(1.0) and st["sign_p"] == 1.0
    assert mcnemar_exact(10, 0) == pytest.approx(2 / 1024)


def test_degenerate_tail():
    assert degenerate("intro " + "abcd" * 20)
    assert not degenerate("a perfectly ordinary sentence that goes on for a while without looping at all.")
