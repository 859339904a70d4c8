"""FP4 delta tier: hot experts served at FP4 precision on the GPU.

Each delta slot holds an expert's MXFP4 weights (e2m1 values, UE8M0 block-32
scales) in the direct-8 container (:func:`formats.planes.pack_direct8`):
``[w13 e4m3 (2I*H) | sc13 | w2 e4m3 (H*I) | sc2]``.  The expert GEMV checks
the delta slot table first and reads the delta slot when present, else the
2-bit base (reference: FP4 delta tier and its slot coupling, patch
P:8063-8383, P:10290-10350).  Policies:

* ``freq`` -- the manager promotes the most frequently routed experts
  (recency-decayed counts) every ``tick``;
* ``need`` -- only the confidence gate fills the pool (promote this step's
  routed experts, then replay the step);
* ``lru``  -- like ``need``, evicting the least recently used slot.

Split FP4 (``split=True``, the reference's ``DELTA_SPLIT`` / w4q path, patch
P:8243-8247, P:8811-8827, P:10031-10055): a delta slot holds only the quintal
refinement planes ``[q13 (2I*H*5/16) | q2 (H*I*5/16)]``, read against the
resident 2-bit base slot (its codes pick each element's magnitude class and
sign, its UE8M0 scales are the MXFP4 scales), so the GEMV rebuilds the exact
e2m1 values from 2 + 2.5 bits per weight.  The pair is served from the delta
slot only while the base slot is resident, and a base cache never evicts an
expert that has a delta slot (:meth:`DeltaTier.couple`).

The pool / table / host-store machinery is :class:`.tier.ExpertCache`.
"""
from __future__ import annotations

from typing import List, Tuple

import torch

from ..formats import planes
from .stores import make_store
from .tier import ExpertCache


def delta_slots_for(delta_gb: str, slot_bytes: int, free_bytes: int, reserve_gb: float = 3.0,
                    max_gb: float = 0.0) -> int:
    """Delta-pool size in slots from ``VLLM_MOE_W2_DELTA_GB``: ``"N"`` GiB, or ``"auto"``
    (the free device memory after load minus ``reserve_gb``, capped by ``max_gb`` when
    non-zero).  Reference: delta sizing, patch P:7903-7916."""
    g = 1 << 30
    v = str(delta_gb).strip().lower()
    if v == "auto":
        budget = max(0, int(free_bytes) - int(reserve_gb * g))
        if max_gb > 0:
            budget = min(budget, int(max_gb * g))
    else:
        try:
            budget = int(float(v) * g)
        except ValueError:
            raise ValueError(f"VLLM_MOE_W2_DELTA_GB must be a number of GiB or auto, got {delta_gb!r}") from None
        if budget < 0:
            raise ValueError("VLLM_MOE_W2_DELTA_GB must be >= 0")
    return budget // int(slot_bytes)


def delta_layout(H: int, I: int):
    """-> (slot_bytes, codes13, sc13, codes2, sc2 offsets) of a direct-8 delta slot."""
    c13 = planes.direct8_plane_bytes(2 * I, H)
    s13 = planes.scale_plane_bytes(2 * I, H)
    c2 = planes.direct8_plane_bytes(H, I)
    s2 = planes.scale_plane_bytes(H, I)
    return c13 + s13 + c2 + s2, 0, c13, c13 + s13, c13 + s13 + c2


def split_layout(H: int, I: int):
    """-> (slot_bytes, q13, 0, q2, 0): split-FP4 slot offsets (no scale planes of its own)."""
    q13 = planes.quintal_plane_bytes(2 * I, H)
    q2 = planes.quintal_plane_bytes(H, I)
    return q13 + q2, 0, 0, q13, 0


def pack_split_slot(nib13: torch.Tensor, nib2: torch.Tensor) -> torch.Tensor:
    """e2m1 nibbles of w13 [2I, H] and w2 [H, I] (the nibbles the base codes were
    derived from) -> one split-FP4 delta slot row (u8)."""
    return torch.cat([planes.pack_quintal(nib13.cpu()), planes.pack_quintal(nib2.cpu())])


def dequant_split_slot(row: torch.Tensor, codes13: torch.Tensor, sc13: torch.Tensor, codes2: torch.Tensor,
                       sc2: torch.Tensor, H: int, I: int):
    """Split slot + the base's codes / UE8M0 scales ([N, K] / [N, K/32]) -> float (w13, w2)."""
    from ..formats.codebook import E2M1_VALUES
    sb, _, _, o2, _ = split_layout(H, I)
    out = []
    for plane, codes, sc, (N, K) in ((row[:o2], codes13, sc13, (2 * I, H)), (row[o2:sb], codes2, sc2, (H, I))):
        nib = planes.quintal_reconstruct(codes, planes.unpack_quintal_digits(plane, N, K))
        v = E2M1_VALUES[nib.long()].float()
        out.append((v.view(N, K // 32, 32) * torch.exp2(sc.float() - 127.0)[..., None]).view(N, K))
    return tuple(out)


def pack_delta_slot(w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """float expert matrices w13 [2I, H], w2 [H, I] -> one delta slot row (u8)."""
    parts = []
    for m in (w13, w2):
        nib, sc = planes.mxfp4_quantize(m)
        parts.append(planes.pack_direct8(planes.e2m1_to_e4m3_bytes(nib)))
        parts.append(planes.pack_scales(sc))
    return torch.cat([p.cpu() for p in parts])


def dequant_delta_slot(row: torch.Tensor, H: int, I: int):
    sb, o13, os13, o2, os2 = delta_layout(H, I)
    w13 = planes.dequant_direct8(row[o13:os13], row[os13:o2], 2 * I, H)
    w2 = planes.dequant_direct8(row[o2:os2], row[os2:sb], H, I)
    return w13, w2


class DeltaTier(ExpertCache):
    def __init__(self, rows_per_layer: List[torch.Tensor], H: int, I: int, n_slots: int, device="cuda",
                 policy: str = "freq", decay: float = 0.98, split: bool = False, promo_hyst: float = 0.0):
        L = len(rows_per_layer)
        E = rows_per_layer[0].shape[0]
        self.split = split
        self.base = None
        self.layout = split_layout(H, I) if split else delta_layout(H, I)
        sb = self.layout[0]
        store = make_store("pinned", L, E, sb)
        for li, r in enumerate(rows_per_layer):
            store.add_layer(li, r)
        super().__init__(store, L, E, sb, n_slots, device=device, policy="lru" if policy == "lru" else "freq",
                         decay=decay, manager=True)
        self.delta_policy = policy
        # promotion hysteresis (PROMO_HYST = h > 1): with the pool full, a background candidate
        # displaces a resident expert only when its decayed frequency exceeds h x the weakest
        # evictable resident's + 4, so a drifting working set does not ping-pong slots.
        # Mandatory promotions (gate fires, misses) call promote() directly and are never gated.
        self.promo_hyst = float(promo_hyst)

    def couple(self, base_cache) -> None:
        """Split FP4 over a base expert cache: promotions make the base resident
        first, and the base never evicts an expert that has a delta slot."""
        if not self.split:
            return
        self.base = base_cache
        base_cache.protect = lambda li, e: self.resident(li, e)

    def promote(self, pairs, stream=None, sync: bool = True) -> int:
        if self.base is not None:
            self.base.promote(pairs, stream=stream, sync=sync)   # a refinement is read against its base
        return super().promote(pairs, stream=stream, sync=sync)

    @property
    def offsets(self):
        _, o13, _, o2, _ = self.layout
        return o13, self.layout[2], o2, self.layout[4]

    def tick(self, max_promote: int = 64) -> int:
        """freq policy: promote the hottest non-resident experts (host-side, between steps)."""
        if self.delta_policy != "freq":
            return 0
        with self.lock:
            hot = torch.argsort(self.freq.view(-1), descending=True)[: self.n_slots]
            want: List[Tuple[int, int]] = []
            for i in hot.tolist():
                li, e = divmod(int(i), self.E)
                if float(self.freq[li, e]) <= 0:
                    break
                if int(self.mirror[li, e]) < 0:
                    want.append((li, e))
                if len(want) >= max_promote:
                    break
            want = self._hysteresis(want)
        return self.promote(want) if want else 0

    def _hysteresis(self, want):
        """Drop the candidates that would only displace a near-equal resident (see promo_hyst)."""
        h = self.promo_hyst
        if h <= 1.0 or not want:
            return want
        n_free = len(self.free)
        victims = sorted(float(self.freq[o[0], o[1]]) for s, o in enumerate(self.owner)
                         if o is not None and s not in self.pinned
                         and not (self.protect is not None and self.protect(*o)))
        kept, vi = [], 0
        for li, e in want:                          # hottest first
            if n_free > 0:
                n_free -= 1
                kept.append((li, e))
            elif vi < len(victims) and float(self.freq[li, e]) > h * victims[vi] + 4.0:
                vi += 1
                kept.append((li, e))
            else:
                self.stats["hyst_blocked"] += 1
        return kept
