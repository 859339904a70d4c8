"""Offline delta-tier policy simulator: replay captured routing against a slot budget.

    python -m vllm_moet_b200.tools.delta_sim routes.npy --slots 256 512 1024 --policy lru freq

Input: the ``.npy`` written by the routing capture (``VLLM_MOE_W2_DELTA_CAPTURE``), an
int32 array [steps, moe layers, rows] of routed expert ids (-1 = padding).  Each step's
distinct (layer, expert) pairs are looked up in a cache of ``slots`` entries.  A hit is
served by the FP4 tier.  A miss is promoted, evicting by the policy:
* ``lru``  -- least recently used;
* ``freq`` -- lowest decayed routing count (the tier's ``freq`` policy: counts decay by
  ``decay`` every step; ties go to the least recently used).
The pairs routed in the current step are pinned, as in the engine.  Reported: hit rate
over distinct pairs and over routed rows (token-weighted), promotions and evictions per
step (reference: the delta policy simulator, tools/delta_sim.py).
"""
from __future__ import annotations

import argparse
import json
from collections import Counter
from typing import Dict, List

import numpy as np


def simulate(routes: np.ndarray, slots: int, policy: str = "lru", decay: float = 0.98) -> Dict[str, float]:
    if policy not in ("lru", "freq"):
        raise ValueError("policy must be lru or freq")
    resident: Dict[tuple, float] = {}           # pair -> last use step
    freq: Counter = Counter()
    hits = pairs = tok_hits = toks = promotions = evictions = 0
    for step in range(routes.shape[0]):
        if policy == "freq":
            for key in list(freq):
                freq[key] *= decay
        counts: Counter = Counter()
        for li in range(routes.shape[1]):
            for e in routes[step, li]:
                if e >= 0:
                    counts[(li, int(e))] += 1
        pinned = set(counts)
        for pair, n in counts.items():
            freq[pair] += n
            pairs += 1
            toks += n
            if pair in resident:
                hits += 1
                tok_hits += n
            else:
                if len(resident) >= slots:
                    cands = [p for p in resident if p not in pinned]
                    if not cands:
                        continue            # every slot pinned this step: served by the base tier
                    if policy == "lru":
                        victim = min(cands, key=lambda p: resident[p])
                    else:
                        victim = min(cands, key=lambda p: (freq[p], resident[p]))
                    del resident[victim]
                    evictions += 1
                promotions += 1
            resident[pair] = step
    n = max(1, routes.shape[0])
    return {"slots": slots, "policy": policy, "hit_rate_distinct": hits / max(1, pairs),
            "hit_rate_tokens": tok_hits / max(1, toks), "promotions_per_step": promotions / n,
            "evictions_per_step": evictions / n}


def sweep(routes: np.ndarray, slots: List[int], policies: List[str], decay: float = 0.98) -> List[dict]:
    return [simulate(routes, s, p, decay) for p in policies for s in slots]


def main(argv=None):
    ap = argparse.ArgumentParser(description="delta-tier policy simulator over captured routing")
    ap.add_argument("routes", help=".npy from VLLM_MOE_W2_DELTA_CAPTURE")
    ap.add_argument("--slots", type=int, nargs="+", default=[256, 512, 1024])
    ap.add_argument("--policy", nargs="+", default=["lru", "freq"])
    ap.add_argument("--decay", type=float, default=0.98)
    a = ap.parse_args(argv)
    for row in sweep(np.load(a.routes), a.slots, a.policy, a.decay):
        print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in row.items()}))


if __name__ == "__main__":
    main()
