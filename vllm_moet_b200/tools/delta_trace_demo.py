"""Functional check and demo of the FP4 delta tier's bookkeeping and trace, without a model.

    python -m vllm_moet_b200.tools.delta_trace_demo [--layers 44 --experts 256 --slots 170
        --steps 400 --tokens 3 --top-k 8 --zipf 1.1 --every 50 --dump delta.json]

Drives the real ``DeltaTier`` (frequency promotion between steps, eviction, pinning of
the step's routed experts) and ``DeltaTrace`` (coverage, distinct and token-weighted hit
rates) with a synthetic routing stream: per layer a Zipf-distributed expert popularity
(each layer its own random permutation), each token routed to top-k distinct experts
drawn from it.  Slot rows are a few hundred bytes -- the manager works on slot indices
and (layer, expert) pairs, so the logic is the one that serves full-size slots.  Prints
the trace line every ``--every`` steps and the final snapshot; ``--dump`` writes the
precision map and the trace as JSON (the ``VLLM_MOE_W2_DELTA_DUMP`` format).
(Reference: tools/delta_trace_demo.py, the same check of its delta manager.)
"""
from __future__ import annotations

import argparse
import json
import sys

import torch

from ..residency.delta import DeltaTier, delta_layout
from ..utils.observability import DeltaTrace, precision_map


def routing_stream(L: int, E: int, tokens: int, k: int, zipf: float, seed: int):
    """Endless per-step routing: {(layer, expert): tokens routed} for `tokens` tokens."""
    g = torch.Generator().manual_seed(seed)
    pop = 1.0 / torch.arange(1, E + 1, dtype=torch.float64) ** zipf
    perms = [torch.randperm(E, generator=g) for _ in range(L)]
    while True:
        step = {}
        for li in range(L):
            picks = torch.multinomial(pop.expand(tokens, E), k, replacement=False, generator=g)
            for e in perms[li][picks].flatten().tolist():
                step[(li, e)] = step.get((li, e), 0) + 1
        yield step


def run(layers=44, experts=256, slots=170, steps=400, tokens=3, top_k=8, zipf=1.1, every=50, seed=0,
        max_promote=64, sink=print) -> dict:
    H = I = 64
    sb = delta_layout(H, I)[0]
    tier = DeltaTier([torch.zeros(experts, sb, dtype=torch.uint8) for _ in range(layers)], H, I, slots,
                     device="cpu", policy="freq")
    trace = DeltaTrace(level=2, every=every, sink=sink)
    stream = routing_stream(layers, experts, tokens, top_k, zipf, seed)
    for _ in range(steps):
        routed = next(stream)
        for (li, e), n in routed.items():
            tier.note_routed(li, [e], weight=float(n))
        trace.step(tier, routed)
        tier.step_end()
        tier.tick(max_promote)
    snap = trace.snapshot(tier)
    snap["resident_map"] = precision_map(tier, "fp4-direct8")
    tier.check_invariants()
    return snap


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--layers", type=int, default=44)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--slots", type=int, default=170)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--tokens", type=int, default=3, help="tokens per step (verify rows)")
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--zipf", type=float, default=1.1)
    ap.add_argument("--every", type=int, default=50)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--dump", help="write the final snapshot and precision map here")
    a = ap.parse_args(argv)
    snap = run(a.layers, a.experts, a.slots, a.steps, a.tokens, a.top_k, a.zipf, a.every, a.seed)
    brief = {k: v for k, v in snap.items() if k not in ("fp4_per_layer", "resident_map")}
    print(json.dumps(brief))
    if a.dump:
        with open(a.dump, "w") as f:
            json.dump(snap, f)
    return 0


if __name__ == "__main__":
    sys.exit(main())
