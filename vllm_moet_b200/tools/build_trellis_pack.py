"""Build trellis (EXL3-style) base-tier packs for a model's routed experts.

    python -m vllm_moet_b200.tools.build_trellis_pack OUT_DIR (--model PRESET | --checkpoint DIR)
        [--layers 3,4,...] [--w13-k 2] [--w2-k 2] [--L 16] [--codebook 3inst|1mad]
        [--device cuda] [--num-layers N] [--seed 0]

One ``exl3-l{li:02d}.safetensors`` per MoE layer (the reference's pack naming; its packs
come from an external exl3 builder, here it is this tool).  The experts are the ones the
engine loads (checkpoint weights, or random-init weights of a preset), dequantised and
trellis-coded by ``formats.trellis.quantize_linear`` (from a checkpoint: its own expert
tensors, bf16 / FP8 / NVFP4 dequantised exactly, not the engine's 2-bit copy): a tail-biting Viterbi search per
16 x 16 tile, 2·256 steps over 2^L states -- run it on a GPU (``--device cuda``) for
L = 16.  Prints one JSON line per layer (bytes, relative weight error of expert 0).
Serve the packs with ``LLM(..., trellis_pack=OUT_DIR)`` or ``VLLM_MOE_W2_EXL3_PACK``.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("out_dir")
    src = ap.add_mutually_exclusive_group(required=True)
    src.add_argument("--model", help="a model preset (random-init weights)")
    src.add_argument("--checkpoint", help="a checkpoint directory")
    ap.add_argument("--layers", default=None, help="comma-separated MoE layer indices (default: all)")
    ap.add_argument("--w13-k", type=int, default=2)
    ap.add_argument("--w2-k", type=int, default=2)
    ap.add_argument("--L", type=int, default=16)
    ap.add_argument("--codebook", default="3inst")
    ap.add_argument("--device", default="cpu", help="where the Viterbi search runs")
    ap.add_argument("--num-layers", type=int, default=None)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)

    from ..engine.llm import LLM
    from ..formats import trellis as tf
    from ..residency import trellis_tier as tt
    llm = LLM(a.checkpoint or a.model, device="cpu", num_speculative_tokens=0, max_model_len=64,
              num_layers=a.num_layers, seed=a.seed)
    layers = None if a.layers is None else [int(x) for x in a.layers.split(",")]
    kw = dict(w13_k=a.w13_k, w2_k=a.w2_k, L=a.L, codebook=a.codebook, seed=a.seed, device=torch.device(a.device))
    if a.checkpoint:
        done = tt.write_checkpoint_packs(a.checkpoint, llm.mw.cfg, a.out_dir, layers, **kw)
    else:
        done = tt.write_model_packs(llm.mw, a.out_dir, layers, **kw)
    if not done:
        print("no MoE layers selected", file=sys.stderr)
        return 1
    tier = tt.TrellisBaseTier(a.out_dir, done)
    for li in done:
        w13, w2 = tier.dequant_expert(li, 0)
        if a.checkpoint:
            o13, o2 = next(tt.checkpoint_experts(a.checkpoint, li, 1))
        else:
            o13, o2 = llm.mw.layers[li].experts.dequant_expert(0)
        print(json.dumps({"layer": li, "pack": tt.pack_path(a.out_dir, li),
                          "bytes": sum(t.numel() * t.element_size() for t in tier.layers[li].values()),
                          "rel_err_w13_e0": round(float((w13 - o13.cpu()).norm() / o13.norm()), 4),
                          "rel_err_w2_e0": round(float((w2 - o2.cpu()).norm() / o2.norm()), 4),
                          "bits": [a.w13_k, a.w2_k], "L": a.L, "codebook": a.codebook,
                          "format": tf.FORMAT}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
