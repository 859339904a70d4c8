"""Routing policies and layer contracts of the 2-bit expert path.

* :func:`apply_topp` -- expert top-p pruning (opt-in): per token, keep the
  smallest prefix of its routed experts (by weight) whose normalised weight
  reaches ``p`` (at least ``min_keep``); a dropped entry is redirected to the
  token's top-1 expert with weight 0, so shapes stay static inside CUDA graphs
  (reference: ``_apply_topp``, patch P:4404-4432).
* :func:`layer_contract_violations` -- semantics the 2-bit path does not
  implement; a checkpoint config that needs any of them is refused at load
  (reference: ``_layer_contract``, P:4517-4620).
* :func:`is_w2_layer` -- only main-stack routed experts use the 2-bit path;
  drafter / MTP layers keep their own precision unless ``VLLM_MOE_W2_DRAFT=1``
  (reference: ``_layer_cutoff`` / ``is_w2_layer``, P:4442-4515).
"""
from __future__ import annotations

import os
from typing import List, Mapping

import torch


def apply_topp(ids: torch.Tensor, wts: torch.Tensor, p: float, min_keep: int = 1):
    """ids [T, k], wts [T, k] -> (ids, wts) with the tail beyond cumulative p pruned (static shapes)."""
    if p <= 0.0:
        return ids, wts
    w = wts.float()
    order = torch.argsort(-w, dim=1, stable=True)
    ws = w.gather(1, order)
    tot = ws.sum(1, keepdim=True).clamp_min(1e-20)
    before = torch.cumsum(ws, 1) - ws                    # weight mass strictly before each entry
    keep_sorted = (before / tot < p)
    keep_sorted[:, :min_keep] = True
    keep = torch.zeros_like(keep_sorted).scatter(1, order, keep_sorted)
    top1 = ids.gather(1, order[:, :1]).expand_as(ids)
    return torch.where(keep, ids, top1), torch.where(keep, wts, torch.zeros_like(wts))


_UNSUPPORTED = {
    "hidden_act": ("silu",),
    "torch_dtype": ("bfloat16", "bf16", None),
}


def layer_contract_violations(hf_config: Mapping) -> List[str]:
    """-> human-readable reasons this checkpoint config cannot run on the 2-bit expert path."""
    out = []
    act = hf_config.get("hidden_act", "silu")
    if act not in _UNSUPPORTED["hidden_act"]:
        out.append(f"expert activation {act!r} (only silu / SwiGLU)")
    if hf_config.get("swiglu_alpha") not in (None, 1.0) or hf_config.get("swiglu_beta") not in (None, 0.0):
        out.append("non-default SwiGLU alpha / beta")
    if hf_config.get("moe_expert_bias") or hf_config.get("expert_bias"):
        out.append("per-expert output bias")
    if hf_config.get("router_weight_on_input"):
        out.append("router weight applied to the expert input")
    if hf_config.get("torch_dtype") not in _UNSUPPORTED["torch_dtype"]:
        out.append(f"activation dtype {hf_config.get('torch_dtype')!r} (only bf16)")
    return out


def check_layer_contract(hf_config: Mapping) -> None:
    bad = layer_contract_violations(hf_config)
    if bad:
        raise ValueError("model not supported by the 2-bit expert path: " + "; ".join(bad))


def is_w2_layer(layer_idx: int, num_hidden_layers: int, draft: bool = False) -> bool:
    if layer_idx < num_hidden_layers and not draft:
        return True
    return os.environ.get("VLLM_MOE_W2_DRAFT", "0") == "1"
