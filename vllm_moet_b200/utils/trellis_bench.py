"""Device time of one routed-expert block served from the trellis base tier.

    python -m vllm_moet_b200.utils.trellis_bench [--hidden 4096] [--inter 1536] [--experts 256]
        [--w13-k 2] [--w2-k 2] [--L 16] [--tokens 1,3,8] [--iters 20] [--device cuda]

Builds one layer's pack of random trellis words (the kernels' cost does not depend on the
words being a good encoding) at the given shape, then times ``forward_topk`` (rotations,
trellis-decode GEMVs, SwiGLU, fixed-order combine) for each token count with top-8 routing
over distinct experts: CUDA events around ``--iters`` calls after warm-up, inputs larger
than L2 only when the routed experts' bytes are (reported).  One JSON line per token count:
microseconds per block, the routed experts' trellis bytes and the implied GB/s against
the measured HBM copy bandwidth (``MEASURED_PEAKS.json``'s ``hbm_gbs`` when present).
"""
from __future__ import annotations

import argparse
import json
import os
import tempfile
import time

import torch


def random_pack(d: str, E: int, H: int, I: int, K13: int, K2: int, L: int, codebook: str = "3inst",
                seed: int = 0) -> None:
    from safetensors.torch import save_file
    from ..formats import trellis as tf
    from ..residency.trellis_tier import pack_path
    g = torch.Generator().manual_seed(seed)
    out = {}
    for e in range(E):
        for name, (n, k, K) in {"w1": (I, H, K13), "w3": (I, H, K13), "w2": (H, I, K2)}.items():
            out[f"e{e}.{name}.k{K}.trellis"] = torch.randint(-32768, 32768, (k // 16, n // 16, 16 * K), generator=g,
                                                             dtype=torch.int32).to(torch.int16)
            out[f"e{e}.{name}.k{K}.suh"] = (torch.randn(k, generator=g) * 0.05).half()
            out[f"e{e}.{name}.k{K}.svh"] = (torch.randn(n, generator=g) * 0.05).half()
    save_file(out, pack_path(d, 0), metadata={"format": tf.FORMAT, "L": str(L), "codebook": codebook,
                                              "num_experts": str(E), "w13_k": str(K13), "w2_k": str(K2)})


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=1536)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--w13-k", type=int, default=2)
    ap.add_argument("--w2-k", type=int, default=2)
    ap.add_argument("--L", type=int, default=16)
    ap.add_argument("--tokens", default="1,3,8")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--device", default="cuda")
    a = ap.parse_args(argv)
    from ..formats import trellis as tf
    from ..residency.trellis_tier import TrellisBaseTier
    hbm = None
    peaks = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                         "MEASURED_PEAKS.json")
    if os.path.exists(peaks):
        with open(peaks) as f:
            hbm = json.load(f).get("hbm_gbs")
    with tempfile.TemporaryDirectory() as d:
        random_pack(d, a.experts, a.hidden, a.inter, a.w13_k, a.w2_k, a.L)
        tier = TrellisBaseTier(d, [0], device=a.device, act_limit=10.0)
    cuda = torch.device(a.device).type == "cuda"
    g = torch.Generator().manual_seed(1)
    per_expert = (2 * tf.linear_bytes(a.inter, a.hidden, a.w13_k) + tf.linear_bytes(a.hidden, a.inter, a.w2_k))
    for T in (int(t) for t in a.tokens.split(",")):
        x = torch.randn(T, a.hidden, generator=g).to(a.device)
        ids = torch.stack([torch.randperm(a.experts, generator=g)[:a.top_k] for _ in range(T)]).to(a.device)
        w = torch.rand(T, a.top_k, generator=g).to(a.device)
        n_exp = int(torch.unique(ids).numel())
        for _ in range(a.warmup):
            tier.forward_topk(0, x, ids, w)
        if cuda:
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(a.iters):
                tier.forward_topk(0, x, ids, w)
            e.record()
            torch.cuda.synchronize()
            us = s.elapsed_time(e) * 1000.0 / a.iters
        else:
            t0 = time.perf_counter()
            for _ in range(a.iters):
                tier.forward_topk(0, x, ids, w)
            us = (time.perf_counter() - t0) * 1e6 / a.iters
        nbytes = n_exp * per_expert
        rec = {"tokens": T, "distinct_experts": n_exp, "us_per_block": round(us, 2), "expert_bytes": nbytes,
               "gb_s": round(nbytes / us / 1e3, 1), "device": a.device,
               "shape": {"hidden": a.hidden, "inter": a.inter, "bits": [a.w13_k, a.w2_k], "L": a.L},
               "inputs_vs_l2": "larger" if nbytes > 126e6 else "smaller (L2-warm after the first call)"}
        if hbm:
            rec["frac_of_measured_hbm"] = round(nbytes / us / 1e3 / hbm, 3)
        print(json.dumps(rec), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
