"""Trellis (EXL3-style) base tier for routed experts.

An alternative to the 2-bit codebook base tier: every routed expert of the chosen layers
is served from trellis-coded weights (``formats/trellis.py``) held resident on the
device.  Like the reference's ``Exl3BaseTier`` (moe_w2_exl3.py,
patch/vllm-moet-v0.24.0.patch:10624-10700 and its ``forward_topk``, P:10780-10795), the
tier computes the routed block ``y[t] = sum_j w[t, j] · expert_{ids[t, j]}(x[t])`` and
leaves out the (t, j) pairs that another tier serves (``fp4_mask``): those pairs get a
zero weight, so the FP4 delta tier's contribution is simply added on top.

Decode groups (the reference's M8 "decode wave", ``build_m8_groups`` P:10456-10510):
each expert of the step is decoded ONCE for all of its rows.  ``group_pairs`` builds the
groups on the device with fixed shapes (no host sync, so the step can be captured): the
T·k routing pairs sorted by expert, each expert's pairs cut into groups of up to 8 rows,
``P = T·k`` group slots of which the unused ones have no rows.

On a GPU the tier runs three kernels (``csrc/kernels/trellis.cu``) per projection: the
input rotation ``x' = H(x ⊙ su)`` per pair, the trellis-decode GEMV over the groups and
the output rotation ``H(z) ⊙ sv`` (times the routing weight for the down projection); the
SwiGLU between them and the fixed-order sum over k are tensor ops.  On the CPU the same
arithmetic runs through ``formats.trellis``.

Packs: one safetensors file per layer, ``exl3-l{li:02d}.safetensors``, keys
``e{e}.{w1|w3|w2}.k{K}.{trellis|suh|svh}`` (w1 = gate, w3 = up, w2 = down: the
reference's naming, P:10660-10668), metadata ``format`` / ``L`` / ``codebook``.
Environment aliases of the reference: ``VLLM_MOE_W2_EXL3_PACK`` (pack directory),
``VLLM_MOE_W2_EXL3_W2K`` (down-projection bits).
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterable, Optional

import torch
import torch.nn.functional as F

from ..formats import trellis as tf

PROJS = ("w1", "w3", "w2")


def pack_path(pack_dir: str, li: int) -> str:
    return os.path.join(pack_dir, f"exl3-l{li:02d}.safetensors")


def write_layer_pack(pack_dir: str, li: int, experts: Iterable, w13_k: int = 2, w2_k: int = 2,
                     L: int = 16, codebook: str = "3inst", seed: int = 0, device=None) -> str:
    """Trellis-code one layer's routed experts and write its pack.

    ``experts`` yields ``(w13 [2I, H], w2 [H, I])`` per expert in expert order (gate rows
    first in w13).  Each projection gets its own sign seed (seed, layer, expert, proj)."""
    from safetensors.torch import save_file
    os.makedirs(pack_dir, exist_ok=True)
    out: Dict[str, torch.Tensor] = {}
    E = 0
    for e, (w13, w2) in enumerate(experts):
        I = w13.shape[0] // 2
        mats = {"w1": (w13[:I], w13_k), "w3": (w13[I:], w13_k), "w2": (w2, w2_k)}
        for pi, (name, (w, K)) in enumerate(mats.items()):
            t = tf.quantize_linear(w.float(), K, L, codebook, seed=(seed * 1000003 + li * 10007 + e * 31 + pi) & 0x7FFFFFFF,
                                   device=device)
            for part, v in t.items():
                out[f"e{e}.{name}.k{K}.{part}"] = v.contiguous()
        E = e + 1
    meta = {"format": tf.FORMAT, "L": str(L), "codebook": codebook, "num_experts": str(E),
            "w13_k": str(w13_k), "w2_k": str(w2_k)}
    path = pack_path(pack_dir, li)
    save_file(out, path, metadata=meta)
    return path


def write_model_packs(mw, pack_dir: str, layers: Optional[Iterable[int]] = None, **kw) -> list:
    """Packs for the MoE layers of loaded model weights (the experts as the engine holds
    them, dequantised).  Returns the layer indices written."""
    done = []
    for li, lw in enumerate(mw.layers):
        if not lw.is_moe or (layers is not None and li not in layers):
            continue
        ex = lw.experts
        n = ex.n_local if ex.n_local is not None else mw.cfg.num_experts
        write_layer_pack(pack_dir, li, (ex.dequant_expert(e) for e in range(n)), **kw)
        done.append(li)
    return done


def checkpoint_experts(path: str, li: int, num_experts: int):
    """The routed experts of layer li as the checkpoint stores them (bf16 / FP8 / NVFP4
    dequantised exactly), ``(w13 [2I, H], w2 [H, I])`` per expert: the source a trellis
    pack should be coded from, rather than another quantisation of it."""
    from ..models.loader import CheckpointReader
    rd = CheckpointReader(path)
    P = f"model.layers.{li}.mlp.experts."
    for e in range(num_experts):
        g, u = rd.dense64(P + f"{e}.gate_proj"), rd.dense64(P + f"{e}.up_proj")
        yield torch.cat([g, u], 0).float(), rd.dense64(P + f"{e}.down_proj").float()


def write_checkpoint_packs(path: str, cfg, pack_dir: str, layers: Optional[Iterable[int]] = None, **kw) -> list:
    """Packs for the MoE layers of a checkpoint, coded from its own expert weights."""
    done = []
    moe = [li for li in range(cfg.num_layers) if li >= cfg.num_dense_layers]
    for li in moe:
        if layers is not None and li not in layers:
            continue
        write_layer_pack(pack_dir, li, checkpoint_experts(path, li, cfg.num_experts), **kw)
        done.append(li)
    return done


def group_pairs(ids: torch.Tensor, rows: int = 8):
    """Decode groups of one step, fixed shapes, on ids' device.

    ids [T, k] -> (experts [P] int32, row_map [P, rows] int32) with P = T·k.  Group g
    serves expert ``experts[g]`` for the pairs ``row_map[g, r]`` (pair index t·k + j, -1 =
    empty row).  An expert's pairs are in ascending pair order, packed from row 0, cut
    into consecutive groups of ``rows``; real groups come first in ascending expert order;
    empty groups carry expert 0 (a valid pointer) and rows of -1 only."""
    T, k = ids.shape
    P = T * k
    dev = ids.device
    flat = ids.reshape(P).to(torch.int64)
    sv, order = torch.sort(flat, stable=True)               # pairs by expert, pair order inside
    pos = torch.arange(P, device=dev)
    new_e = torch.ones(P, dtype=torch.bool, device=dev)
    new_e[1:] = sv[1:] != sv[:-1]
    first = torch.cummax(torch.where(new_e, pos, torch.zeros_like(pos)), 0).values
    rank = pos - first                                       # rank of the pair inside its expert
    start = new_e | (rank % rows == 0)
    gid = torch.cumsum(start.to(torch.int64), 0) - 1
    experts = torch.zeros(P, dtype=torch.int64, device=dev)
    experts.scatter_(0, gid, sv)
    row_map = torch.full((P * rows,), -1, dtype=torch.int64, device=dev)
    row_map.scatter_(0, gid * rows + rank % rows, order)
    return experts.to(torch.int32), row_map.view(P, rows).to(torch.int32)


class TrellisBaseTier:
    """Resident trellis-coded routed experts for a set of layers."""

    def __init__(self, pack_dir: str, layers: Iterable[int], device="cpu", num_experts: Optional[int] = None,
                 hidden: Optional[int] = None, inter: Optional[int] = None, w13_k: Optional[int] = None,
                 w2_k: Optional[int] = None, act_limit: Optional[float] = None):
        """Bits per weight default to the pack's own (``w13_k`` / ``w2_k`` metadata);
        ``VLLM_MOE_W2_EXL3_W2K`` picks the down-projection variant of packs that hold
        several."""
        from safetensors import safe_open
        self.dev = torch.device(device)
        self.act_limit = act_limit
        env_w2k = os.environ.get("VLLM_MOE_W2_EXL3_W2K")
        self.w13_k: Optional[int] = w13_k
        self.w2_k: Optional[int] = w2_k if w2_k is not None else (int(env_w2k) if env_w2k else None)
        self.L: Optional[int] = None
        self.codebook: Optional[str] = None
        self.layers: Dict[int, Dict[str, torch.Tensor]] = {}
        self._q: Dict[tuple, torch.Tensor] = {}               # CPU path: decoded Q per (layer, expert, proj)
        for li in layers:
            path = pack_path(pack_dir, li)
            with safe_open(path, "pt") as f:
                meta = f.metadata() or {}
                if meta.get("format") != tf.FORMAT:
                    raise ValueError(f"{path}: not a {tf.FORMAT} pack (format={meta.get('format')!r}); "
                                     "packs written by other trellis tools use another bit order")
                L, cb = int(meta["L"]), meta["codebook"]
                if self.w13_k is None:
                    self.w13_k = int(meta["w13_k"])
                if self.w2_k is None:
                    self.w2_k = int(meta["w2_k"])
                if self.L is None:
                    self.L, self.codebook = L, cb
                elif (L, cb) != (self.L, self.codebook):
                    raise ValueError(f"{path}: trellis L / codebook differ between layers")
                E = int(meta["num_experts"]) if num_experts is None else num_experts
                st: Dict[str, torch.Tensor] = {}
                for name, K in (("w1", self.w13_k), ("w3", self.w13_k), ("w2", self.w2_k)):
                    for part in ("trellis", "suh", "svh"):
                        st[f"{name}.{part}"] = torch.stack(
                            [f.get_tensor(f"e{e}.{name}.k{K}.{part}") for e in range(E)]).to(self.dev).contiguous()
            self.layers[li] = st
        first = next(iter(self.layers.values()))
        self.E = first["w1.trellis"].shape[0]
        self.H = first["w1.suh"].shape[1] if hidden is None else hidden
        self.I = first["w1.svh"].shape[1] if inter is None else inter
        self.inv_rms = 1.0 / tf.codebook_rms(self.L, self.codebook)

    def total_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for st in self.layers.values() for t in st.values())

    def _K(self, name: str) -> int:
        return self.w2_k if name == "w2" else self.w13_k

    def _t(self, li: int, e: int, name: str) -> dict:
        st = self.layers[li]
        return {p: st[f"{name}.{p}"][e] for p in ("trellis", "suh", "svh")}

    def dequant_expert(self, li: int, e: int):
        """-> (w13 [2I, H], w2 [H, I]) fp32 on the CPU: the weights the tier serves."""
        def w(name):
            t = {p: v.cpu() for p, v in self._t(li, e, name).items()}
            return tf.dequant_linear(t, self._K(name), self.L, self.codebook)
        return torch.cat([w("w1"), w("w3")]), w("w2")

    # ------------------------------------------------------------------ forward
    def _swiglu(self, g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
        if self.act_limit:
            g = g.clamp(max=self.act_limit)
            u = u.clamp(-self.act_limit, self.act_limit)
        return F.silu(g) * u

    def _stream(self, li: int) -> dict:
        """The base stream of layer li: trellis tensors indexed by expert id."""
        return dict(st=self.layers[li], K13=self.w13_k, K2=self.w2_k, L=self.L, codebook=self.codebook,
                    inv_rms=self.inv_rms, slot_of=None, qcache=self._q, key=("base", li))

    @torch.no_grad()
    def forward_topk(self, li: int, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                     fp4_mask: Optional[torch.Tensor] = None,
                     delta: Optional["TrellisDeltaPool"] = None) -> torch.Tensor:
        """x [T, H], ids [T, k], weights [T, k] -> routed output [T, H] fp32 without the
        pairs marked in fp4_mask [T, k] (served by another tier).

        With a delta pool, the pairs whose expert holds a slot are served base + delta: the
        delta's gate / up outputs are added before the SwiGLU and its down output after
        (weight-level additivity, (Wb + D) x = Wb x + D x), the reference's unified Δ-pool
        semantics (forward_topk_unified, patch P:10796-10818)."""
        w = weights.float()
        if fp4_mask is not None:
            w = w.masked_fill(fp4_mask, 0.0)
        streams = [self._stream(li)]
        if delta is not None and li in delta.layers:
            streams.append(delta._stream(li))
        if x.is_cuda:
            return self._forward_native(x, ids, w, streams)
        return self._forward_ref(x, ids, w, streams)

    def _swiglu_sum(self, parts_g, parts_u):
        return self._swiglu(sum(parts_g), sum(parts_u))

    def _forward_ref(self, x, ids, w, streams):
        out = torch.zeros(x.shape[0], self.H, dtype=torch.float32)

        def lin(sm, row, inp, name):
            K = sm["K2"] if name == "w2" else sm["K13"]
            key = sm["key"] + (row, name)
            if key not in sm["qcache"]:
                sm["qcache"][key] = tf.decode_q(sm["st"][f"{name}.trellis"][row].cpu(), K, sm["L"], sm["codebook"])
            t = {p: sm["st"][f"{name}.{p}"][row].cpu() for p in ("trellis", "suh", "svh")}
            return tf.apply_linear(inp, t, K, sm["L"], sm["codebook"], q=sm["qcache"][key])
        for e in torch.unique(ids).tolist():
            rows, slot = (ids == e).nonzero(as_tuple=True)
            xe = x[rows].float().cpu()
            live = []
            for sm in streams:
                row = e if sm["slot_of"] is None else int(sm["slot_of"][e])
                if row >= 0:
                    live.append((sm, row))
            h = self._swiglu_sum([lin(sm, r, xe, "w1") for sm, r in live], [lin(sm, r, xe, "w3") for sm, r in live])
            y = sum(lin(sm, r, h, "w2") for sm, r in live)
            out.index_add_(0, rows.cpu(), y * w[rows, slot, None].cpu())
        return out.to(x.device)

    @torch.no_grad()
    def forward_pairs(self, li: int, x: torch.Tensor, ids: torch.Tensor,
                      delta: Optional["TrellisDeltaPool"] = None) -> torch.Tensor:
        """Per routing pair, unweighted: [T·k, H] fp32, row t·k + j = expert ids[t, j] on
        x[t] (base + delta for pooled experts).  The GPU engine's expert combine applies the
        routing weights, the residual and the shared expert.  CUDA tensors only."""
        streams = [self._stream(li)]
        if delta is not None and li in delta.layers:
            streams.append(delta._stream(li))
        return self._forward_native(x, ids, None, streams)

    def _forward_native(self, x, ids, w, streams):
        from ..ops import native
        C = native()
        T, k = ids.shape
        P = T * k
        dev = x.device
        xf = x.float().contiguous()
        src = torch.arange(P, device=dev, dtype=torch.int32) // k
        own = torch.arange(P, device=dev, dtype=torch.int32)
        wp = w.reshape(P).contiguous() if w is not None else None
        plans = []
        for sm in streams:
            if sm["slot_of"] is None:     # base: every pair, groups of distinct experts per token
                rid, sel, maxr = ids, None, min(T, 8)
            else:                         # delta: pooled pairs; the others read slot 0, weighted 0
                so = sm["slot_dev"][ids.long()]      # device tensor: no copy inside a captured step
                sel = (so >= 0).float().reshape(P).contiguous()
                rid, maxr = so.clamp_min(0), 8
            experts, row_map = group_pairs(rid)
            plans.append((sm, rid.reshape(P).to(torch.int32).contiguous(), experts, row_map, sel, maxr))

        def proj(plan, inp, src_rows, name, scale):
            sm, eid, experts, row_map, _, maxr = plan
            st = sm["st"]
            K = sm["K2"] if name == "w2" else sm["K13"]
            kin, n = st[f"{name}.suh"].shape[1], st[f"{name}.svh"].shape[1]
            xr = torch.empty(P, kin, dtype=torch.float32, device=dev)
            C.trellis_rot_in(inp, src_rows, eid, st[f"{name}.suh"], xr)
            z = torch.empty(P, n, dtype=torch.float32, device=dev)
            C.trellis_gemv(xr, st[f"{name}.trellis"], experts, row_map, z, K, sm["L"], sm["codebook"] == "1mad",
                           sm["inv_rms"], maxr)
            y = torch.empty_like(z)
            C.trellis_rot_out(z, eid, st[f"{name}.svh"], scale, y)
            return y
        g = sum(proj(pl, xf, src, "w1", pl[4]) for pl in plans)
        u = sum(proj(pl, xf, src, "w3", pl[4]) for pl in plans)
        h = self._swiglu(g, u).contiguous()
        if wp is None:                                  # per pair, unweighted
            return sum(proj(pl, h, own, "w2", pl[4]) for pl in plans)
        y = sum(proj(pl, h, own, "w2", wp if pl[4] is None else wp * pl[4]) for pl in plans)
        return y.view(T, k, self.H).sum(1)              # fixed order over k: deterministic

    def moe_fn(self, mw, layer_offset: int = 0):
        """A ``reference.moe_context`` function: routed experts from this tier for its
        layers (the model's own experts elsewhere), plus the shared expert.
        ``layer_offset``: the global index of ``mw.layers[0]`` (a pipeline stage's range)."""
        from ..models import reference as ref
        index = {id(lw): li + layer_offset for li, lw in enumerate(mw.layers)}
        if self.act_limit is None:
            self.act_limit = mw.cfg.swiglu_limit

        def fn(cfg, lw, h):
            li = index.get(id(lw))
            if li not in self.layers:
                return ref.moe_block(cfg, lw, h)
            ids, w = ref.route(cfg, lw, h)
            if ref._TOPP[0] > 0:
                from ..models.moe_policy import apply_topp
                ids, w = apply_topp(ids, w, *ref._TOPP)
            out = self.forward_topk(li, h, ids, w, delta=getattr(self, "delta", None)).to(h.device)
            if lw.shared_gate_up is not None:
                out = out + ref.swiglu(h.float() @ lw.shared_gate_up.dequant().t(), cfg.swiglu_limit) \
                    @ lw.shared_down.dequant().t()
            return out
        return fn

    def attach_delta(self, pool: "TrellisDeltaPool"):
        """Serve this tier's layers base + delta through ``moe_fn``."""
        self.delta = pool

    def describe(self) -> str:
        return json.dumps({"layers": sorted(self.layers), "E": self.E, "H": self.H, "I": self.I, "L": self.L,
                           "codebook": self.codebook, "w13_k": self.w13_k, "w2_k": self.w2_k,
                           "bytes": self.total_bytes()})


class TrellisDeltaPool:
    """Correction slots over the trellis base tier (the reference's EXL3 Δ pool,
    ``delta_slot_geom`` / ``delta_ptr_tables``, patch P:10411-10446): a promoted expert's
    residual ``W_true - W_base`` (the base as the tier serves it) is trellis-coded into a
    slot at its own bits (``dk13`` / ``dk2``) and codebook (1MAD by default, the base packs
    use 3INST), and the tier then serves that expert base + delta.  Slot tensors are
    stacked [slots, ...] per layer on the tier's device; ``slot_of[li]`` maps expert -> slot
    (-1: not pooled).  Promotion reuses the slot of an expert already pooled, takes a free
    one, or evicts the oldest promotion (FIFO)."""

    def __init__(self, tier: TrellisBaseTier, slots: int, layers: Optional[Iterable[int]] = None,
                 dk13: int = 2, dk2: int = 2, L: Optional[int] = None, codebook: str = "1mad", seed: int = 1):
        if slots < 1:
            raise ValueError("delta pool needs at least one slot")
        self.tier, self.slots = tier, int(slots)
        self.dk13, self.dk2 = dk13, dk2
        self.L = L if L is not None else tier.L
        self.codebook, self.seed = codebook, seed
        self.inv_rms = 1.0 / tf.codebook_rms(self.L, codebook)
        H, I, dev = tier.H, tier.I, tier.dev
        self.layers: Dict[int, Dict[str, torch.Tensor]] = {}
        self.slot_of: Dict[int, torch.Tensor] = {}
        self.slot_dev: Dict[int, torch.Tensor] = {}
        self.order: Dict[int, list] = {}
        self._q: Dict[tuple, torch.Tensor] = {}
        for li in (layers if layers is not None else tier.layers):
            st = {}
            for name, (n, kin, K) in (("w1", (I, H, dk13)), ("w3", (I, H, dk13)), ("w2", (H, I, dk2))):
                st[f"{name}.trellis"] = torch.zeros(self.slots, kin // 16, n // 16, 16 * K, dtype=torch.int16,
                                                    device=dev)
                st[f"{name}.suh"] = torch.ones(self.slots, kin, dtype=torch.float16, device=dev)
                st[f"{name}.svh"] = torch.zeros(self.slots, n, dtype=torch.float16, device=dev)
            self.layers[li] = st
            self.slot_of[li] = torch.full((tier.E,), -1, dtype=torch.int32)
            self.slot_dev[li] = self.slot_of[li].to(dev)     # the device copy the kernels' step reads
            self.order[li] = []
        self.stats = {"promoted": 0, "evicted": 0}

    def _stream(self, li: int) -> dict:
        return dict(st=self.layers[li], K13=self.dk13, K2=self.dk2, L=self.L, codebook=self.codebook,
                    inv_rms=self.inv_rms, slot_of=self.slot_of[li], slot_dev=self.slot_dev[li], qcache=self._q,
                    key=("delta", li))

    def promote(self, li: int, e: int, w13: torch.Tensor, w2: torch.Tensor, device=None) -> int:
        """Code expert e's residual against the base tier into a slot; returns the slot.
        ``w13`` [2I, H] (gate rows first) and ``w2`` [H, I] are the expert's true weights."""
        so = self.slot_of[li]
        s = int(so[e])
        if s < 0:
            used = set(int(v) for v in so.tolist() if v >= 0)
            free = [i for i in range(self.slots) if i not in used]
            if free:
                s = free[0]
            else:
                old = self.order[li].pop(0)
                s = int(so[old])
                so[old] = -1
                self.stats["evicted"] += 1
        else:
            self.order[li].remove(e)
        b13, b2 = self.tier.dequant_expert(li, e)
        I = w13.shape[0] // 2
        res = {"w1": w13[:I].float().cpu() - b13[:I], "w3": w13[I:].float().cpu() - b13[I:],
               "w2": w2.float().cpu() - b2}
        st = self.layers[li]
        for pi, name in enumerate(("w1", "w3", "w2")):
            K = self.dk2 if name == "w2" else self.dk13
            t = tf.quantize_linear(res[name], K, self.L, self.codebook,
                                   seed=(self.seed * 1000003 + li * 10007 + e * 31 + pi) & 0x7FFFFFFF, device=device)
            for part, v in t.items():
                st[f"{name}.{part}"][s].copy_(v.to(st[f"{name}.{part}"].device))
            for key in [k_ for k_ in self._q if k_[:2] == ("delta", li) and k_[2] == s]:
                del self._q[key]
        so[e] = s
        self.slot_dev[li].copy_(so)
        self.order[li].append(e)
        self.stats["promoted"] += 1
        return s

    def evict(self, li: int, e: int) -> None:
        so = self.slot_of[li]
        if int(so[e]) >= 0:
            so[e] = -1
            self.slot_dev[li].copy_(so)
            self.order[li].remove(e)
            self.stats["evicted"] += 1

    def dequant_expert(self, li: int, e: int):
        """-> (w13, w2) the tier serves for expert e with the pool: base + delta (or base)."""
        b13, b2 = self.tier.dequant_expert(li, e)
        s = int(self.slot_of[li][e])
        if s < 0:
            return b13, b2
        st = self.layers[li]

        def d(name):
            K = self.dk2 if name == "w2" else self.dk13
            t = {p: st[f"{name}.{p}"][s].cpu() for p in ("trellis", "suh", "svh")}
            return tf.dequant_linear(t, K, self.L, self.codebook)
        return b13 + torch.cat([d("w1"), d("w3")]), b2 + d("w2")
