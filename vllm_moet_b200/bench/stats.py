"""Quality-parity statistics for the bench harness: does a candidate configuration
(e.g. 2-bit experts + delta tier) answer as well as a baseline on the same items?

* :func:`mcnemar_exact` -- exact two-sided McNemar test on the discordant pairs (items
  one configuration got right and the other wrong): a binomial(n, 1/2) tail.
* :func:`paired_token_stats` -- per item, candidate completion tokens / baseline
  completion tokens: median and geometric mean of the ratios, and an exact sign test
  on longer vs shorter (token inflation is a quality regression too).
* :func:`compare` -- both, plus accuracies and runaways (completions at the token cap).
* :func:`passes` -- the gates a recipe sets: ``min_mcnemar_p``,
  ``max_abs_token_ratio_median_delta_pct``, ``max_abs_token_ratio_geomean_delta_pct``,
  ``min_token_sign_p``.
(Reference: the quality probe's paired statistics and gates, bench/runner/probes.py.)
"""
from __future__ import annotations

import math
import statistics
from typing import Dict, Mapping, Optional


def binom_two_sided(k: int, n: int) -> float:
    """P(X <= min(k, n - k)) * 2 for X ~ Binomial(n, 1/2), capped at 1."""
    if n <= 0:
        return 1.0
    lo = min(k, n - k)
    tail = sum(math.comb(n, i) for i in range(lo + 1)) / 2.0 ** n
    return min(1.0, 2.0 * tail)


def mcnemar_exact(only_base: int, only_cand: int) -> float:
    return binom_two_sided(only_base, only_base + only_cand)


def paired_token_stats(base: Mapping[str, int], cand: Mapping[str, int], cap: Optional[int] = None) -> Dict:
    """Token counts per item id (items with a zero count in either are skipped)."""
    ids = sorted(i for i in base.keys() & cand.keys() if base[i] > 0 and cand[i] > 0)
    if not ids:
        return {}
    ratios = [cand[i] / base[i] for i in ids]
    longer = sum(r > 1 for r in ratios)
    shorter = sum(r < 1 for r in ratios)
    out = {"paired_items": len(ids), "ratio_median": statistics.median(ratios),
           "ratio_geomean": math.exp(statistics.fmean(math.log(r) for r in ratios)),
           "longer": longer, "shorter": shorter, "sign_p": binom_two_sided(longer, longer + shorter)}
    if cap:
        out["base_runaways"] = sum(base[i] >= cap for i in ids)
        out["cand_runaways"] = sum(cand[i] >= cap for i in ids)
    return out


def compare(base_rows: Mapping[str, dict], cand_rows: Mapping[str, dict], cap: Optional[int] = None) -> Dict:
    """rows: item id -> {"correct": bool, "tokens": int}."""
    ids = sorted(base_rows.keys() & cand_rows.keys())
    only_base = sum(base_rows[i]["correct"] and not cand_rows[i]["correct"] for i in ids)
    only_cand = sum(cand_rows[i]["correct"] and not base_rows[i]["correct"] for i in ids)
    n = max(1, len(ids))
    out = {"items": len(ids), "acc_base": sum(base_rows[i]["correct"] for i in ids) / n,
           "acc_cand": sum(cand_rows[i]["correct"] for i in ids) / n,
           "only_base": only_base, "only_cand": only_cand, "mcnemar_p": mcnemar_exact(only_base, only_cand)}
    tok = paired_token_stats({i: base_rows[i]["tokens"] for i in ids}, {i: cand_rows[i]["tokens"] for i in ids},
                             cap)
    out.update({f"token_{k}": v for k, v in tok.items()})
    for k in ("ratio_median", "ratio_geomean"):
        if f"token_{k}" in out:
            out[f"token_{k}_delta_pct"] = (out[f"token_{k}"] - 1.0) * 100.0
    return out


def passes(cmp_: Mapping, gates: Mapping) -> bool:
    if "min_mcnemar_p" in gates and cmp_.get("mcnemar_p", 0.0) < float(gates["min_mcnemar_p"]):
        return False
    for field, key in (("token_ratio_median_delta_pct", "max_abs_token_ratio_median_delta_pct"),
                       ("token_ratio_geomean_delta_pct", "max_abs_token_ratio_geomean_delta_pct")):
        if key in gates:
            v = cmp_.get(field)
            if v is None or abs(v) > float(gates[key]):
                return False
    if "min_token_sign_p" in gates and cmp_.get("token_sign_p", 0.0) < float(gates["min_token_sign_p"]):
        return False
    return True


def degenerate(text: str) -> bool:
    """A short chunk (4, 8 or 16 characters) repeated back to back at the end of the text."""
    if len(text) < 64:
        return False
    for w in (4, 8, 16):
        chunk = text[-w:]
        if chunk.strip() and text.endswith(chunk * min(8, len(text) // w)):
            return True
    return False
