"""EAGLE-3 draft module: one decoder layer fed by the target's aux hidden states.

The target's residual after three chosen layers (low, middle, high) is concatenated and
projected by ``fc`` [H, 3H] to one hidden state per position; the draft layer reads
``in_proj([rms(embed(token_{i+1})) ; rms(h_i)])`` at position i and predicts token
i + 2 through its own norm and the target's shared lm_head.  Later draft steps feed
the draft layer's own output hidden state back in place of the projected aux states
(a hidden state of width H skips ``fc``), so drafting chains exactly as the MTP module
does and the engine's MTP machinery (prefill pass, verify rows, chained drafts, its
own K/V cache) runs it unchanged.  (EAGLE-3: Li et al. 2025; the serving method the
reference runs upstream for Kimi.)
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence, Tuple

import torch

from .weights import LayerWeights, ModelWeights, _make_layer, _Rng, make_linear


@dataclass
class Eagle3Weights:
    target_layers: Tuple[int, ...]
    fc: object                 # [H, H * len(target_layers)]
    enorm: torch.Tensor
    hnorm: torch.Tensor
    in_proj: object            # [H, 2H]
    layer: LayerWeights
    norm: torch.Tensor


def random_eagle3_weights(mw: ModelWeights, target_layers: Optional[Sequence[int]] = None,
                          seed: int = 0) -> Eagle3Weights:
    cfg = mw.cfg
    H = cfg.hidden
    L = len(mw.layers)
    tl = tuple(target_layers) if target_layers is not None else tuple(sorted({0, L // 2, L - 1}))
    dev = mw.final_norm.device
    g = torch.Generator().manual_seed(seed + 3331)
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    layer = _make_layer(cfg, _Rng(seed + 3332, dev), 2000, dev, False)     # a dense draft layer
    fc = torch.randn(H, H * len(tl), generator=g) / math.sqrt(H * len(tl))
    in_proj = torch.randn(H, 2 * H, generator=g) / math.sqrt(2 * H)
    return Eagle3Weights(tl, make_linear(fc.to(dev), "bf16"), ones.clone(), ones.clone(),
                         make_linear(in_proj.to(dev), "bf16"), layer, ones.clone())


def attach_eagle3(mw: ModelWeights, ew: Eagle3Weights) -> ModelWeights:
    """Route the model's draft module to EAGLE-3 (`reference.forward` then returns the
    concatenated aux hidden states, `reference.mtp_forward` runs this module)."""
    mw.extra["eagle3"] = ew
    return mw


def eagle3_forward(mw: ModelWeights, hidden: torch.Tensor, next_tokens: torch.Tensor, positions: torch.Tensor,
                   cs: torch.Tensor, cache=None):
    """-> (logits [T, V], draft hidden [T, H] for the next chained step)."""
    from . import reference as ref
    cfg, ew = mw.cfg, mw.extra["eagle3"]
    H = cfg.hidden
    h = hidden.float()
    if h.shape[-1] != H:                        # the target's concatenated aux states
        h = h @ ew.fc.dequant().t()
    embed = mw.embed if mw.embed is not None else mw.extra["mtp_embed"]
    e = ref.rms_norm(embed[next_tokens].float(), ew.enorm, cfg.rms_eps)
    x = torch.cat([e, ref.rms_norm(h, ew.hnorm, cfg.rms_eps)], -1) @ ew.in_proj.dequant().t()
    x = ref.decoder_layer(cfg, ew.layer, x, positions, cs, cache, 0)
    out = ref.rms_norm(x, ew.norm, cfg.rms_eps)
    return ref._gather_vocab(out @ mw.lm_head.dequant().t()), x
