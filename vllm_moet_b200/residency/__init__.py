"""Expert residency: host stores, the persistent planes cache, the GPU expert
cache with in-graph miss counting and replay, the confidence gate, the
speculation guard and the routing prefetchers."""
from .control import (ConfidenceGate, DraftAffinity, LookaheadPrefetcher, Pilot, ReplayEngine, SpecGuard,  # noqa: F401
                      gate_fire_floor, pp_gate_barrier, gate_promote_consensus)
from .identity import checkpoint_id, identity_fields, rank_suffix  # noqa: F401
from .planes_cache import PlanesCache  # noqa: F401
from .stores import (MmapPackStore, PinnedHostStore, RowBatch, TieredPackStore, make_store,  # noqa: F401
                     pack_has_layer, stride_for)
from .tier import ExpertCache, FetchError, resident_fit, working_set_floor  # noqa: F401


def moe_layers(mw):
    """MoE layers of a model in cache order: main stack first, then the MTP layer."""
    out = [lw for lw in mw.layers if lw.is_moe]
    if mw.mtp is not None and mw.mtp.layer.is_moe:
        out.append(mw.mtp.layer)
    return out


def build_expert_cache(mw, n_slots: int, kind: str = "pinned", device="cuda", policy: str = "lru", **store_kw):
    """Move every MoE layer's routed experts into a host store and serve them
    through one GPU expert cache of `n_slots` slots.  Each layer's ExpertPool
    then points at the shared pool and its row of the slot table."""
    import torch
    layers = moe_layers(mw)
    L = len(layers)
    lay0 = layers[0].experts.layout
    E = layers[0].experts.pool.shape[0]
    sb = lay0.slot_bytes
    store = make_store(kind, L, E, sb, **store_kw)
    for li, lw in enumerate(layers):
        if not store.has_layer(li):
            store.add_layer(li, lw.experts.pool.cpu())
    cache = ExpertCache(store, L, E, sb, n_slots, device=device, policy=policy)
    for li, lw in enumerate(layers):
        lw.experts.pool = cache.pool
        lw.experts.slot_table = cache.slot_table[li]
    if torch.cuda.is_available():
        torch.cuda.empty_cache()
    return cache
