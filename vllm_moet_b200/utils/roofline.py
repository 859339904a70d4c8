"""Roofline of one decode step: the bytes a step must stream from HBM and the time that
takes at a measured copy bandwidth, next to a measured step time.

Per step the engine reads (per GPU, TP-sharded where the engine shards):
* every dense linear of every layer once (FP8: 1 byte per weight + block scales), the
  router (bf16) and the MTP module's layer;
* the routed experts of the step: each distinct expert of a layer once (2-bit codes +
  UE8M0 block-32 scales = 0.28125 bytes per weight); the expected number of distinct
  experts of R routed rows over E experts is E * (1 - (1 - k/E)^rows_tokens);
* the lm_head once per verify pass (1 + k passes with MTP drafting);
* the latent KV of every active sequence (attention reads it once per layer).

    python -m vllm_moet_b200.utils.roofline --streams 1 --measured-ms 6.17
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Optional

from ..config import ModelConfig, get_preset

EXPERT_BYTES_PER_WEIGHT = 2 / 8 + 1 / 32      # 2-bit codes + one UE8M0 byte per 32 weights
FP8_BYTES_PER_WEIGHT = 1 + 1 / (128 * 128)


def _dense_layer_weights(cfg: ModelConfig, moe: bool, tp: int) -> float:
    H, nh = cfg.hidden, cfg.num_heads
    attn = ((cfg.q_lora_rank + cfg.kv_lora_rank + cfg.qk_rope_dim) * H                 # qkv_a (replicated)
            + (nh * cfg.qk_head_dim * cfg.q_lora_rank) / tp                             # q_b
            + (nh * (cfg.qk_nope_dim + cfg.v_head_dim) * cfg.kv_lora_rank) / tp         # W_uk / W_uv (absorbed kv_b)
            + (H * nh * cfg.v_head_dim) / tp)                                            # o
    if cfg.index_heads:
        attn += cfg.index_heads * cfg.index_head_dim * cfg.q_lora_rank + cfg.index_head_dim * H + cfg.index_heads * H
    if not moe:
        return attn + 3 * H * cfg.dense_intermediate / tp
    shared = 3 * H * cfg.moe_intermediate * cfg.num_shared_experts / tp
    return attn + shared


def step_bytes(cfg: ModelConfig, streams: int = 1, k: int = 2, tp: int = 1, context: int = 1024,
               kv_bytes_per_token: int = 1168) -> dict:
    """-> bytes per decode step by component (per GPU)."""
    rows = streams * (1 + k)
    L = cfg.num_layers
    n_moe = L - cfg.num_dense_layers + (1 if k and cfg.num_mtp_layers else 0)
    n_dense = cfg.num_dense_layers
    dense = (n_dense * _dense_layer_weights(cfg, False, tp) + n_moe * _dense_layer_weights(cfg, True, tp)) \
        * FP8_BYTES_PER_WEIGHT
    router = n_moe * cfg.num_experts * cfg.hidden * 2
    distinct = cfg.num_experts * (1 - (1 - cfg.top_k / cfg.num_experts) ** rows)
    expert = n_moe * distinct * 3 * cfg.hidden * cfg.moe_intermediate / tp * EXPERT_BYTES_PER_WEIGHT
    head = (1 + k) * cfg.vocab * cfg.hidden / tp * FP8_BYTES_PER_WEIGHT
    kv = streams * context * kv_bytes_per_token * (L + (1 if k else 0))
    total = dense + router + expert + head + kv
    return {"dense": dense, "router": router, "experts": expert, "experts_distinct_per_layer": distinct,
            "lm_head": head, "kv": kv, "total": total}


def roofline(cfg: ModelConfig, hbm_gbs: float, streams: int = 1, k: int = 2, tp: int = 1,
             measured_ms: Optional[float] = None, **kw) -> dict:
    b = step_bytes(cfg, streams, k, tp, **kw)
    floor_ms = b["total"] / (hbm_gbs * 1e9) * 1e3
    out = {"bytes_gb": {kk: round(v / 1e9, 3) for kk, v in b.items() if kk != "experts_distinct_per_layer"},
           "experts_distinct_per_layer": round(b["experts_distinct_per_layer"], 1),
           "hbm_gbs": hbm_gbs, "floor_ms": round(floor_ms, 3),
           "floor_steps_s": round(1e3 / floor_ms, 1)}
    if measured_ms:
        out["measured_ms"] = measured_ms
        out["fraction_of_roofline"] = round(floor_ms / measured_ms, 3)
    return out


def _measured_hbm(default: float = 6549.1) -> float:
    for p in ("MEASURED_PEAKS.json", os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")):
        if os.path.exists(p):
            with open(p) as f:
                return float(json.load(f).get("hbm_gbs", default))
    return default


def main(argv=None):
    ap = argparse.ArgumentParser(description="decode-step roofline")
    ap.add_argument("--model", default="ds4-flash-shape")
    ap.add_argument("--streams", type=int, default=1)
    ap.add_argument("--k", type=int, default=2)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--context", type=int, default=1024)
    ap.add_argument("--measured-ms", type=float, default=None)
    ap.add_argument("--hbm-gbs", type=float, default=None, help="default: MEASURED_PEAKS.json hbm_gbs")
    a = ap.parse_args(argv)
    cfg = get_preset(a.model)
    print(json.dumps(roofline(cfg, a.hbm_gbs or _measured_hbm(), a.streams, a.k, a.tp, a.measured_ms,
                              context=a.context), indent=1))


if __name__ == "__main__":
    main()
