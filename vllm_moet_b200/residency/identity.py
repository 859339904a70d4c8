"""Identity of persistent expert caches (packs, planes cache).

A pack or planes-cache entry is raw expert rows; nothing in its geometry
tells two checkpoints with equal expert dimensions apart, so every cache is
keyed by the checkpoint identity, the quantizer ABI and the zero-code mode
(the reference keys its packs the same way: moe_w2_store.py identity
fields, patch P:12886-12998; planes cache ``_ckpt_id`` P:12550-12629).

* A checkpoint directory: sha256 over config.json, the safetensors index and
  the (name, size, mtime) stat record of every shard.
* A random-init model (this repository's benchmarks): sha256 of the model
  config and the seed, prefixed ``random:``.
* ``MOET_CKPT_ID`` (alias ``VLLM_MOE_W2_CKPT_ID``) overrides both.
* Unknown identity -> ``None``; a pack written without identity gets a
  process-local namespace and is never reused by another process.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import os
from typing import Optional

from ..formats.codebook import QUANTIZER_ABI, zero_mode


def _sha(obj) -> str:
    return hashlib.sha256(json.dumps(obj, sort_keys=True, separators=(",", ":"), default=str).encode()).hexdigest()


def checkpoint_id(model_path: Optional[str] = None, cfg=None, seed: Optional[int] = None) -> Optional[str]:
    env = os.environ.get("MOET_CKPT_ID") or os.environ.get("VLLM_MOE_W2_CKPT_ID")
    if env:
        return env
    if model_path and os.path.isdir(model_path):
        rec = {}
        for name in sorted(os.listdir(model_path)):
            p = os.path.join(model_path, name)
            if name in ("config.json", "model.safetensors.index.json"):
                with open(p, "rb") as f:
                    rec[name] = hashlib.sha256(f.read()).hexdigest()
            elif name.endswith(".safetensors"):
                st = os.stat(p)
                rec[name] = [st.st_size, int(st.st_mtime)]
        return "ckpt:" + _sha(rec)[:40]
    if cfg is not None and seed is not None:
        c = dataclasses.asdict(cfg) if dataclasses.is_dataclass(cfg) else dict(cfg)
        return "random:" + _sha({"cfg": c, "seed": seed})[:40]
    return None


def identity_fields(ckpt_id: Optional[str]) -> dict:
    return {"ckpt_id": ckpt_id, "zero_mode": zero_mode(), "quantizer_abi": QUANTIZER_ABI}


def rank_suffix(tp_rank: int = 0, tp_world: int = 1, pp_rank: int = 0, pp_world: int = 1) -> str:
    """``rank{r}of{w}``, plus ``.pp{p}of{P}`` under pipeline parallelism (PP ranks
    hold disjoint layers but reuse TP rank numbers)."""
    s = f"rank{tp_rank}of{tp_world}"
    if pp_world > 1:
        s += f".pp{pp_rank}of{pp_world}"
    return s
