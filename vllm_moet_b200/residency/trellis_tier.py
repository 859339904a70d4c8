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

    @torch.no_grad()
    def forward_topk(self, li: int, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                     fp4_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x [T, H], ids [T, k], weights [T, k] -> routed output [T, H] fp32 without the
        pairs marked in fp4_mask [T, k] (served by another tier)."""
        w = weights.float()
        if fp4_mask is not None:
            w = w.masked_fill(fp4_mask, 0.0)
        if x.is_cuda:
            return self._forward_native(li, x, ids, w)
        return self._forward_ref(li, x, ids, w)

    def _forward_ref(self, li, x, ids, w):
        out = torch.zeros(x.shape[0], self.H, dtype=torch.float32)
        for e in torch.unique(ids).tolist():
            rows, slot = (ids == e).nonzero(as_tuple=True)
            xe = x[rows].float().cpu()

            def lin(inp, name):
                key = (li, e, name)
                if key not in self._q:
                    self._q[key] = tf.decode_q(self.layers[li][f"{name}.trellis"][e].cpu(), self._K(name),
                                               self.L, self.codebook)
                t = {p: v.cpu() for p, v in self._t(li, e, name).items()}
                return tf.apply_linear(inp, t, self._K(name), self.L, self.codebook, q=self._q[key])
            h = self._swiglu(lin(xe, "w1"), lin(xe, "w3"))
            out.index_add_(0, rows.cpu(), lin(h, "w2") * w[rows, slot, None].cpu())
        return out.to(x.device)

    def _forward_native(self, li, x, ids, w):
        from ..ops import native
        C = native()
        st = self.layers[li]
        T, k = ids.shape
        P = T * k
        experts, row_map = group_pairs(ids)
        eid = ids.reshape(P).to(torch.int32)
        src = torch.arange(P, device=x.device, dtype=torch.int32) // k
        maxr = min(T, 8)
        xf = x.float().contiguous()

        def proj(inp, src_rows, name, scale=None):
            K = self._K(name)
            kin = st[f"{name}.suh"].shape[1]
            n = st[f"{name}.svh"].shape[1]
            xr = torch.empty(P, kin, dtype=torch.float32, device=x.device)
            C.trellis_rot_in(inp, src_rows, eid, st[f"{name}.suh"], xr)
            z = torch.empty(P, n, dtype=torch.float32, device=x.device)
            C.trellis_gemv(xr, st[f"{name}.trellis"], experts, row_map, z, K, self.L,
                           self.codebook == "1mad", self.inv_rms, maxr)
            y = torch.empty_like(z)
            C.trellis_rot_out(z, eid, st[f"{name}.svh"], scale, y)
            return y
        h = self._swiglu(proj(xf, src, "w1"), proj(xf, src, "w3")).contiguous()
        own = torch.arange(P, device=x.device, dtype=torch.int32)
        y = proj(h, own, "w2", w.reshape(P).contiguous())
        return y.view(T, k, self.H).sum(1)              # fixed order over k: deterministic

    def moe_fn(self, mw):
        """A ``reference.moe_context`` function: routed experts from this tier for its
        layers (the model's own experts elsewhere), plus the shared expert."""
        from ..models import reference as ref
        index = {id(lw): li for li, lw in enumerate(mw.layers)}
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
            out = self.forward_topk(li, h, ids, w).to(h.device)
            if lw.shared_gate_up is not None:
                out = out + ref.swiglu(h.float() @ lw.shared_gate_up.dequant().t(), cfg.swiglu_limit) \
                    @ lw.shared_down.dequant().t()
            return out
        return fn

    def describe(self) -> str:
        return json.dumps({"layers": sorted(self.layers), "E": self.E, "H": self.H, "I": self.I, "L": self.L,
                           "codebook": self.codebook, "w13_k": self.w13_k, "w2_k": self.w2_k,
                           "bytes": self.total_bytes()})
