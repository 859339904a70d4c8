"""Boot-from-cache sources for the expert planes (load path).

Quantising a large model's experts to 2-bit planes dominates boot time.  A
source lets the weight builder skip it layer by layer (the reference's
loader-level skip and streaming first-boot build, patch P:4802-5090,
P:5615-5646):

* :class:`PlanesSource` -- the persistent planes cache
  (``<root>/v2/<sha20(meta)>/tp{W}-rank{R}/layer{L}.slots.bin``), for GPU-resident
  configurations;
* :class:`PackSource` -- a pack store (``<tag>.v2.<key>.<rank>.pack``), for tiered
  configurations where the pack doubles as the quantisation cache.

``load(li, n, slot_bytes)`` returns the layer's rows or None (a miss: the
builder quantises and then calls ``store``).  Both count hits and misses.
"""
from __future__ import annotations

from typing import Optional

import torch

from .planes_cache import PlanesCache


class PlanesSource:
    def __init__(self, cache: PlanesCache):
        self.cache = cache
        self.hits = self.misses = 0

    def load(self, li: int, n: int, slot_bytes: int) -> Optional[torch.Tensor]:
        got = self.cache.try_load(li, {"slots": n * slot_bytes})
        if got is None:
            self.misses += 1
            return None
        self.hits += 1
        return got["slots"]

    def store(self, li: int, pool: torch.Tensor):
        self.cache.store(li, {"slots": pool.reshape(-1)})

    def flush(self):
        self.cache.flush()


class PackSource:
    def __init__(self, store):
        self.store_ = store
        self.hits = self.misses = 0

    def load(self, li: int, n: int, slot_bytes: int) -> Optional[torch.Tensor]:
        if li >= self.store_.n_layers or not self.store_.has_layer(li) or self.store_.slot_bytes != slot_bytes:
            self.misses += 1
            return None
        b = self.store_.rows_for(li, list(range(n)), scan=True)
        if b.failed:
            self.misses += 1
            return None
        self.hits += 1
        return torch.stack(b.rows)

    def store(self, li: int, pool: torch.Tensor):
        if li < self.store_.n_layers and not self.store_.has_layer(li):
            self.store_.add_layer(li, pool.cpu())

    def flush(self):
        pass
