"""Load a Hugging Face DeepSeek-style MoE checkpoint (config.json + safetensors shards).

The reference serves real checkpoints through upstream vLLM's DeepSeek loader plus
its quant-method hooks, which re-quantise the routed experts to the 2-bit codebook
at load time (``moe_w2_planes.py``: ``fp8_block_to_codes_scales``,
``nvfp4_to_codes_scales``, ``mxfp4_to_codes``).  Here one loader maps the
checkpoint's tensor names onto :class:`ModelWeights`, with the same TP / EP / PP
slicing as the synthetic builder:

* dense linears (attention, dense FFN, shared expert, head): bf16 / f32, or FP8 e4m3
  with ``weight_scale_inv`` 128x128 block scales.  Power-of-two block scales (the UE8M0
  convention) are kept bit-exactly when no TP slice cuts a block; otherwise the block
  product is taken in float64 and re-quantised (``Fp8Linear.from_float``);
* routed experts: bf16 / f32, FP8 blocks, or NVFP4 (``weight`` packed e2m1,
  ``weight_scale`` e4m3 block-16, ``weight_scale_2`` f32) are dequantised to exact
  float64 products and converted with ``codebook.f64_to_codes_scales`` -- the
  conversion the reference's FP8 and NVFP4 paths end in -- then packed into
  fragment-major slots;
* the MTP module (DeepSeek layout: decoder layer ``num_hidden_layers`` with
  ``enorm``, ``hnorm``, ``eh_proj`` -- or its ``e_proj`` / ``h_proj`` halves -- and
  ``shared_head.norm``);
* hyper-connections (``hc_mult`` > 1 in config.json): ``model.layers.{i}.hc_attn_*`` /
  ``hc_ffn_*`` (``fn``, ``base``, ``scale``, f32), the head's ``model.hc_head_*`` and the
  MTP layer's ``hc_head_*``.

Names follow the DeepSeek-V3 layout (``model.layers.{i}.self_attn.q_a_proj`` ...,
``mlp.experts.{e}.gate_proj``, ``mlp.gate.e_score_correction_bias``).
"""
from __future__ import annotations

import json
import math
import os
from typing import Dict, Optional

import torch

from ..config import ModelConfig
from ..formats import codebook, planes
from .weights import (ExpertLayout, ExpertPool, Fp8Linear, FloatLinear, HyperConn, LayerWeights, ModelWeights, MTPWeights,
                      _derive_absorb, _shard_ffn, _vocab_shard, make_linear, pp_layer_range, tp_ffn_shard)


# ------------------------------------------------------------------ config
def hf_config(path: str, **overrides) -> ModelConfig:
    """config.json of a DeepSeek-V3-style checkpoint -> ModelConfig."""
    with open(os.path.join(path, "config.json")) as f:
        c = json.load(f)
    qc = c.get("quantization_config") or {}
    algo = str(qc.get("quant_algo", "") or qc.get("quant_method", "")).lower()
    dense = ("fp8" if qc.get("quant_method") == "fp8" or qc.get("fmt") == "e4m3" else
             "nvfp4" if "nvfp4" in algo or "modelopt" in algo else "bf16")
    kw = dict(
        name=c.get("model_type", os.path.basename(os.path.normpath(path))),
        num_layers=c["num_hidden_layers"], hidden=c["hidden_size"], vocab=c["vocab_size"],
        num_dense_layers=c.get("first_k_dense_replace", 0), dense_intermediate=c.get("intermediate_size", 0),
        num_heads=c["num_attention_heads"], q_lora_rank=c.get("q_lora_rank"), kv_lora_rank=c["kv_lora_rank"],
        qk_nope_dim=c["qk_nope_head_dim"], qk_rope_dim=c["qk_rope_head_dim"], v_head_dim=c["v_head_dim"],
        num_experts=c["n_routed_experts"], moe_intermediate=c["moe_intermediate_size"],
        top_k=c["num_experts_per_tok"], num_shared_experts=c.get("n_shared_experts", 0) or 0,
        router=c.get("scoring_func", "softmax"), n_group=c.get("n_group", 1) or 1,
        topk_group=c.get("topk_group", 1) or 1, norm_topk_prob=bool(c.get("norm_topk_prob", True)),
        routed_scaling=float(c.get("routed_scaling_factor", 1.0)), swiglu_limit=c.get("swiglu_limit"),
        index_heads=c.get("index_n_heads", 0) or 0, index_head_dim=c.get("index_head_dim", 128) or 128,
        index_topk=c.get("index_topk", 2048) or 2048, num_mtp_layers=c.get("num_nextn_predict_layers", 0) or 0,
        rope_theta=float(c.get("rope_theta", 10000.0)), rms_eps=float(c.get("rms_norm_eps", 1e-6)),
        max_position=c.get("max_position_embeddings", 163840), dense_dtype=dense,
        hc_mult=int(c.get("hc_mult", 1) or 1), hc_sinkhorn_iters=int(c.get("hc_sinkhorn_iters", 20) or 20),
        hc_eps=float(c.get("hc_eps", 1e-6)))
    if c.get("q_lora_rank") is None:
        raise NotImplementedError("checkpoints without q_lora_rank (no low-rank q) are not supported")
    kw.update(overrides)
    return ModelConfig(**kw)


# ------------------------------------------------------------------ tensors
class CheckpointReader:
    """Lazy tensor access over a checkpoint's safetensors shards."""

    def __init__(self, path: str):
        from safetensors import safe_open
        self.path = path
        idx = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                wm = json.load(f)["weight_map"]
            files = sorted(set(wm.values()))
        else:
            files = sorted(n for n in os.listdir(path) if n.endswith(".safetensors"))
            wm = None
        self.handles = {fn: safe_open(os.path.join(path, fn), framework="pt") for fn in files}
        self.where: Dict[str, str] = dict(wm) if wm else {k: fn for fn, h in self.handles.items() for k in h.keys()}

    def has(self, name: str) -> bool:
        return name in self.where

    def get(self, name: str) -> torch.Tensor:
        if name not in self.where:
            raise KeyError(f"tensor {name!r} not in checkpoint {self.path}")
        return self.handles[self.where[name]].get_tensor(name)

    def dense64(self, prefix: str) -> torch.Tensor:
        """`prefix`.weight dequantised to exact float64 (bf16 / f32 / FP8 + weight_scale_inv / NVFP4)."""
        w = self.get(prefix + ".weight")
        if self.has(prefix + ".weight_scale_inv"):                          # FP8 e4m3, 128x128 blocks
            s = self.get(prefix + ".weight_scale_inv").double()
            N, K = w.shape
            full = s.repeat_interleave(128, 0)[:N].repeat_interleave(128, 1)[:, :K]
            return w.to(torch.float32).double() * full
        if w.dtype == torch.uint8 and self.has(prefix + ".weight_scale"):  # NVFP4: e2m1 pairs, e4m3 block-16
            sb = self.get(prefix + ".weight_scale").float()
            s2 = self.get(prefix + ".weight_scale_2").double() if self.has(prefix + ".weight_scale_2") \
                else torch.ones((), dtype=torch.float64)
            vals = codebook.E2M1_VALUES[codebook.split_packed_e2m1(w).long()]
            vals = vals * sb.double().repeat_interleave(16, dim=1)
            return vals * (s2.reshape(()) if s2.numel() == 1 else s2.reshape(-1, 1))
        return w.double()

    def linear(self, prefix: str, dtype: str, rows=None, cols=None):
        """A dense linear, optionally sliced (rows / cols = (lo, hi)).  NVFP4 tensors stay
        NVFP4 (bit-exact) when the model's dense format is nvfp4 and nothing is sliced."""
        if dtype == "nvfp4" and rows is None and cols is None and self.has(prefix + ".weight_scale") \
                and self.get(prefix + ".weight").dtype == torch.uint8:
            from .weights import Nvfp4Linear
            s2 = self.get(prefix + ".weight_scale_2") if self.has(prefix + ".weight_scale_2") else torch.tensor(1.0)
            return Nvfp4Linear(self.get(prefix + ".weight").contiguous(), self.get(prefix + ".weight_scale"),
                               s2.float().reshape(()))
        if dtype == "fp8" and rows is None and cols is None and self.has(prefix + ".weight_scale_inv"):
            s = self.get(prefix + ".weight_scale_inv").float()
            e = torch.log2(s)
            if torch.equal(e, torch.round(e)) and bool(((e >= -127) & (e <= 127)).all()):   # UE8M0: keep bytes
                w = self.get(prefix + ".weight")
                return Fp8Linear(w.view(torch.uint8).contiguous(), (e + 127).to(torch.uint8).contiguous())
        w = self.dense64(prefix)
        if rows is not None:
            w = w[rows[0]:rows[1]]
        if cols is not None:
            w = w[:, cols[0]:cols[1]]
        return make_linear(w.float().contiguous(), dtype)

    def vector(self, name: str, default=None) -> Optional[torch.Tensor]:
        return self.get(name) if self.has(name) else default


# ------------------------------------------------------------------ layers
def _pack_expert(w13: torch.Tensor, w2: torch.Tensor, layout: ExpertLayout, slot: torch.Tensor):
    for mat, oc, osc in ((w13, layout.off_codes13, layout.off_sc13), (w2, layout.off_codes2, layout.off_sc2)):
        N, K = mat.shape
        codes, sc, _ = codebook.f64_to_codes_scales(mat.double())
        slot[oc:oc + N * K // 4] = planes.pack_codes(codes).to(slot.device)
        slot[osc:osc + N * K // 32] = planes.pack_scales(sc).to(slot.device)


def _layer(rd: CheckpointReader, cfg: ModelConfig, li: int, dev, moe: bool, tp_rank: int, tp_size: int,
           ep: bool, expert_source=None) -> LayerWeights:
    P = f"model.layers.{li}."
    dt = cfg.dense_dtype
    H, nh = cfg.hidden, cfg.num_heads
    if nh % tp_size:
        raise ValueError("num_heads must divide by the TP size")
    Hh = nh // tp_size
    qk, nope_v, vd = cfg.qk_head_dim, cfg.qk_nope_dim + cfg.v_head_dim, cfg.v_head_dim
    h0, h1 = tp_rank * Hh, (tp_rank + 1) * Hh
    sl = (lambda a, b: (a, b)) if tp_size > 1 else (lambda a, b: None)

    def bf(name, n):
        v = rd.vector(name)
        return (v if v is not None else torch.ones(n)).to(torch.bfloat16).to(dev)
    # q_a and kv_a are replicated across TP ranks and fused row-wise: exact FP8 bytes when
    # both halves have UE8M0 block scales and q_lora starts a new 128-row block
    a = rd.linear(P + "self_attn.q_a_proj", dt)
    b = rd.linear(P + "self_attn.kv_a_proj_with_mqa", dt)
    if isinstance(a, Fp8Linear) and isinstance(b, Fp8Linear) and cfg.q_lora_rank % 128 == 0:
        qkv_a = Fp8Linear(torch.cat([a.w, b.w], 0), torch.cat([a.s, b.s], 0))
    else:
        qkv_a = make_linear(torch.cat([rd.dense64(P + "self_attn.q_a_proj"),
                                       rd.dense64(P + "self_attn.kv_a_proj_with_mqa")], 0).float(), dt)
    lw = LayerWeights(
        attn_norm=bf(P + "input_layernorm.weight", H),
        qkv_a=qkv_a,
        q_a_norm=bf(P + "self_attn.q_a_layernorm.weight", cfg.q_lora_rank),
        kv_a_norm=bf(P + "self_attn.kv_a_layernorm.weight", cfg.kv_lora_rank),
        q_b=rd.linear(P + "self_attn.q_b_proj", dt, rows=sl(h0 * qk, h1 * qk)),
        kv_b=rd.linear(P + "self_attn.kv_b_proj", dt, rows=sl(h0 * nope_v, h1 * nope_v)),
        o=rd.linear(P + "self_attn.o_proj", dt, cols=sl(h0 * vd, h1 * vd)),
        ffn_norm=bf(P + "post_attention_layernorm.weight", H),
    )
    if isinstance(lw.kv_b, Fp8Linear):
        lw.w_uk_t, lw.w_uv = _derive_absorb(lw.kv_b, cfg, Hh)
    if cfg.index_heads:
        if rd.has(P + "self_attn.indexer.k_norm.weight"):
            raise NotImplementedError("indexer with a key LayerNorm (DeepSeek-V3.2 layout): this engine's DSA "
                                      "indexer has no key norm or indexer rope, so the checkpoint would be "
                                      "served as a different model")
        lw.idx_wq = rd.linear(P + "self_attn.indexer.wq_b", dt)
        lw.idx_wk = rd.linear(P + "self_attn.indexer.wk", dt)
        lw.idx_ww = rd.linear(P + "self_attn.indexer.weights_proj", dt)
    if not moe:
        I = cfg.dense_intermediate
        Ip = tp_ffn_shard(I, tp_size, dt) if tp_size > 1 else I
        gu = torch.cat([rd.dense64(P + "mlp.gate_proj"), rd.dense64(P + "mlp.up_proj")], 0).float()
        gu, dn = _shard_ffn(gu, rd.dense64(P + "mlp.down_proj").float(), I, tp_rank, tp_size, Ip)
        lw.gate_up, lw.down = make_linear(gu.contiguous(), dt), make_linear(dn.contiguous(), dt)
        return lw
    E, Ifull = cfg.num_experts, cfg.moe_intermediate
    if ep:
        if E % tp_size:
            raise ValueError("num_experts must divide by the EP size")
        I, e_lo, n_loc = Ifull, tp_rank * (E // tp_size), E // tp_size
    else:
        if Ifull % tp_size or (Ifull // tp_size) % 64:
            raise ValueError("expert intermediate / tp must be a multiple of 64")
        I, e_lo, n_loc = Ifull // tp_size, 0, E
    lw.router_w = rd.get(P + "mlp.gate.weight").float().to(dev)
    bias = rd.vector(P + "mlp.gate.e_score_correction_bias")
    lw.router_bias = (bias.float() if bias is not None else torch.zeros(E)).to(dev)
    if cfg.num_shared_experts:
        Is = Ifull * cfg.num_shared_experts
        Isp = tp_ffn_shard(Is, tp_size, dt) if tp_size > 1 else Is
        gu = torch.cat([rd.dense64(P + "mlp.shared_experts.gate_proj"),
                        rd.dense64(P + "mlp.shared_experts.up_proj")], 0).float()
        gu, dn = _shard_ffn(gu, rd.dense64(P + "mlp.shared_experts.down_proj").float(), Is, tp_rank, tp_size, Isp)
        lw.shared_gate_up, lw.shared_down = make_linear(gu.contiguous(), dt), make_linear(dn.contiguous(), dt)
    layout = ExpertLayout(H=H, I=I)
    lo = 0 if ep else tp_rank * I
    pool = torch.empty(n_loc, layout.slot_bytes, dtype=torch.uint8, device=dev)
    cached = expert_source.load(li, n_loc, layout.slot_bytes) if expert_source is not None else None
    if cached is not None:
        pool.copy_(cached.view(n_loc, layout.slot_bytes))
    else:
        for j in range(n_loc):
            e = e_lo + j
            EP = P + f"mlp.experts.{e}."
            g, u = rd.dense64(EP + "gate_proj"), rd.dense64(EP + "up_proj")
            d = rd.dense64(EP + "down_proj")
            w13 = torch.cat([g[lo:lo + I], u[lo:lo + I]], 0)
            w2 = d[:, lo:lo + I]
            slot = torch.empty(layout.slot_bytes, dtype=torch.uint8)
            _pack_expert(w13, w2, layout, slot)
            pool[j].copy_(slot)
        if expert_source is not None:
            expert_source.store(li, pool)
    lw.experts = ExpertPool(layout, pool, torch.arange(n_loc, dtype=torch.int32, device=dev), e_lo=e_lo,
                            n_local=n_loc if ep else None)
    return lw


def load_weights(path: str, cfg: Optional[ModelConfig] = None, device="cpu", tp_rank: int = 0, tp_size: int = 1,
                 with_mtp: bool = True, num_layers: Optional[int] = None, pp_rank: int = 0, pp_size: int = 1,
                 expert_parallel: bool = False, expert_source=None) -> ModelWeights:
    """The checkpoint at `path` as ModelWeights (TP / EP / PP slices as the synthetic builder)."""
    cfg = cfg or hf_config(path)
    if cfg.expert_scale != "ue8m0":
        cfg = cfg.replace(expert_scale="ue8m0")
    dev = torch.device(device)
    rd = CheckpointReader(path)
    has_hc = any(".hc_" in n or n.startswith("hc_") for n in rd.where)
    if has_hc != (cfg.hc_mult > 1):
        raise ValueError(f"config hc_mult={cfg.hc_mult} but the checkpoint "
                         f"{'has' if has_hc else 'has no'} hyper-connection (hc_*) tensors")
    H = cfg.hidden
    L = cfg.num_layers if num_layers is None else num_layers
    l0, l1 = pp_layer_range(L, pp_rank, pp_size)
    first, last = pp_rank == 0, pp_rank == pp_size - 1
    embed = rd.get("model.embed_tokens.weight").to(torch.bfloat16).to(dev) if first else None
    layers = [_layer(rd, cfg, i, dev, cfg.is_moe_layer(i), tp_rank, tp_size, expert_parallel, expert_source)
              for i in range(l0, l1)]
    head = final_norm = None
    if last:
        hw = rd.dense64("lm_head").float()
        head = make_linear(_vocab_shard(hw, tp_rank, tp_size), cfg.dense_dtype)
        final_norm = rd.get("model.norm.weight").to(torch.bfloat16).to(dev)
    mw = ModelWeights(cfg=cfg, embed=embed, layers=layers,
                      final_norm=final_norm if final_norm is not None else torch.ones(H, dtype=torch.bfloat16,
                                                                                      device=dev),
                      lm_head=head, tp_rank=tp_rank, tp_size=tp_size)
    mw.extra.update(layer_range=(l0, l1), pp_rank=pp_rank, pp_size=pp_size, checkpoint=path)
    N = cfg.num_layers
    split_eh = rd.has(f"model.layers.{N}.e_proj.weight") and rd.has(f"model.layers.{N}.h_proj.weight")
    if with_mtp and cfg.num_mtp_layers and last and (rd.has(f"model.layers.{N}.eh_proj.weight") or split_eh):
        P = f"model.layers.{N}."
        if mw.embed is None:
            src = P + "embed_tokens.weight" if rd.has(P + "embed_tokens.weight") else "model.embed_tokens.weight"
            mw.extra["mtp_embed"] = rd.get(src).to(torch.bfloat16).to(dev)
        mw.mtp = MTPWeights(
            enorm=rd.get(P + "enorm.weight").to(torch.bfloat16).to(dev),
            hnorm=rd.get(P + "hnorm.weight").to(torch.bfloat16).to(dev),
            # DeepSeek-V4 stores the projection as separate embedding / hidden halves
            eh_proj=(make_linear(torch.cat([rd.dense64(P + "e_proj"), rd.dense64(P + "h_proj")], 1).float(),
                                 cfg.dense_dtype) if split_eh else rd.linear(P + "eh_proj", cfg.dense_dtype)),
            layer=_layer(rd, cfg, N, dev, True, tp_rank, tp_size, expert_parallel, expert_source),
            head_norm=rd.get(P + "shared_head.norm.weight").to(torch.bfloat16).to(dev))
    if cfg.hc_mult > 1:
        for i, lw in zip(range(l0, l1), mw.layers):
            lw.hc_attn, lw.hc_ffn = _hc_site(rd, f"model.layers.{i}.hc_attn", dev), \
                _hc_site(rd, f"model.layers.{i}.hc_ffn", dev)
        if last:
            mw.extra["hc_head"] = _hc_site(rd, "model.hc_head", dev)
        if mw.mtp is not None:
            P = f"model.layers.{N}."
            mw.mtp.layer.hc_attn, mw.mtp.layer.hc_ffn = _hc_site(rd, P + "hc_attn", dev), _hc_site(rd, P + "hc_ffn", dev)
            mw.mtp.hc_head = _hc_site(rd, P + "hc_head", dev)
    for lw in mw.layers + ([mw.mtp.layer] if mw.mtp is not None else []):
        for name in ("qkv_a", "q_b", "kv_b", "o", "gate_up", "down", "shared_gate_up", "shared_down", "w_uk_t",
                     "w_uv", "idx_wq", "idx_wk", "idx_ww"):
            v = getattr(lw, name)
            if v is not None and hasattr(v, "to"):
                setattr(lw, name, v.to(dev))
    if mw.lm_head is not None:
        mw.lm_head = mw.lm_head.to(dev)
    if mw.mtp is not None:
        mw.mtp.eh_proj = mw.mtp.eh_proj.to(dev)
    return mw


def _hc_site(rd: CheckpointReader, prefix: str, dev) -> HyperConn:
    """`prefix`_fn / _base / _scale (f32, replicated on every TP rank)."""
    return HyperConn(*(rd.get(f"{prefix}_{k}").float().to(dev) for k in ("fn", "base", "scale")))


def is_checkpoint_dir(path) -> bool:
    return isinstance(path, str) and os.path.isdir(path) and os.path.exists(os.path.join(path, "config.json"))
