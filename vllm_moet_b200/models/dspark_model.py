"""DSpark draft model: a parallel block drafter that attends to the target's context.

Architecture (the DeepSeek-V4 DSpark draft, reference ``dspark.py`` P:14478-14971 and
``qwen3_dspark.py`` P:14211-14436):

* context: the target's residual stream after a few chosen layers (aux hidden states)
  is concatenated and projected, ``main_x = rms_norm(main_proj(concat aux))``.  Every
  draft layer derives its own context K/V from ``main_x`` through its MLA key/value
  path (kv_a -> norm -> kv_b, RoPE on the shared key) and keeps the last ``window``
  positions (sliding-window context);
* block: the pending token followed by L - 1 mask tokens at positions p .. p + L - 1
  runs through the draft layers (the target's decoder-layer architecture, hyper-
  connections included) with non-causal attention: every block query sees the
  context window and the whole block, future block positions included; the block's
  own K/V are not kept;
* heads: the block's hidden states go through the stream reduction (hyper-
  connections), the final norm and the target's shared lm_head (base logits); a
  sequential low-rank Markov head then walks the block left to right, adding
  ``markov_w2 @ markov_w1[previous token]`` to each position's base logits; the
  confidence head scores ``w . [h_j ; markov_w1[previous token]] + b`` and its
  sigmoid, multiplied along the block, is the survival curve the scheduler reads.

The drafter's weights ship with the target (layers after the MTP module); here they are
random-init of that architecture.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import reference as ref
from .weights import HyperConn, LayerWeights, ModelWeights, _make_layer, _Rng, make_linear


@dataclass
class DSparkWeights:
    target_layers: Tuple[int, ...]
    main_proj: object                  # [H, H * len(target_layers)]
    main_norm: torch.Tensor
    layers: List[LayerWeights]
    norm: torch.Tensor
    markov_w1: torch.Tensor            # [V, r]
    markov_w2: torch.Tensor            # [V, r]
    conf_w: torch.Tensor               # [H + r]
    conf_b: float
    mask_token: int
    window: int
    hc_head: Optional[HyperConn] = None


def random_dspark_weights(mw: ModelWeights, num_layers: int = 2, rank: int = 32,
                          target_layers: Optional[Sequence[int]] = None, window: int = 128,
                          mask_token: Optional[int] = None, seed: int = 0) -> DSparkWeights:
    cfg = mw.cfg
    H, V = cfg.hidden, cfg.vocab
    L = len(mw.layers)
    tl = tuple(target_layers) if target_layers is not None else tuple(sorted({0, L // 2, L - 1}))
    dev = mw.final_norm.device
    rng = _Rng(seed + 7717, dev)
    layers = [_make_layer(cfg, rng, 1000 + i, dev, cfg.is_moe_layer(cfg.num_layers - 1)) for i in range(num_layers)]
    g = torch.Generator().manual_seed(seed + 7718)
    hc_head = None
    if cfg.hc_mult > 1:
        n = cfg.hc_mult

        def site(rows):
            return HyperConn((torch.randn(rows, n * H, generator=g) * 0.02).to(dev),
                             (torch.randn(rows, generator=g) * 0.5).to(dev),
                             (0.5 + torch.rand(3 if rows > n else 1, generator=g)).to(dev))
        for lw in layers:
            lw.hc_attn, lw.hc_ffn = site((2 + n) * n), site((2 + n) * n)
        hc_head = site(n)
    return DSparkWeights(
        target_layers=tl,
        main_proj=make_linear(torch.randn(H, H * len(tl), generator=g) / math.sqrt(H * len(tl)), "bf16"),
        main_norm=torch.ones(H, dtype=torch.bfloat16, device=dev), layers=layers,
        norm=torch.ones(H, dtype=torch.bfloat16, device=dev),
        markov_w1=(torch.randn(V, rank, generator=g) * 0.02).to(dev),
        markov_w2=(torch.randn(V, rank, generator=g) * 0.02).to(dev),
        conf_w=(torch.randn(H + rank, generator=g) * 0.02).to(dev), conf_b=1.5,
        mask_token=V - 1 if mask_token is None else mask_token, window=window, hc_head=hc_head)


# ------------------------------------------------------------------ MLA pieces
def _heads(cfg, lw) -> int:
    return lw.q_b.shape[0] // cfg.qk_head_dim


def mla_kv(cfg, lw, x: torch.Tensor, positions: torch.Tensor, cs: torch.Tensor):
    """x [T, H] -> (k [Hh, T, qk], v [Hh, T, vd]) through the layer's key/value path."""
    Hh, T = _heads(cfg, lw), x.shape[0]
    nope, lat = cfg.qk_nope_dim, cfg.kv_lora_rank
    qkva = x.float() @ lw.qkv_a.dequant().t()
    c = ref.rms_norm(qkva[:, cfg.q_lora_rank: cfg.q_lora_rank + lat], lw.kv_a_norm, cfg.rms_eps)
    kr = ref.apply_rope(qkva[:, cfg.q_lora_rank + lat:], cs[positions])
    kvb = (c @ lw.kv_b.dequant().t()).view(T, Hh, nope + cfg.v_head_dim)
    k = torch.cat([kvb[..., :nope], kr[:, None, :].expand(T, Hh, cfg.qk_rope_dim)], dim=-1).transpose(0, 1)
    return k, kvb[..., nope:].transpose(0, 1)


def block_attention(cfg, lw, x: torch.Tensor, positions: torch.Tensor, cs: torch.Tensor,
                    ctx_k: Optional[torch.Tensor], ctx_v: Optional[torch.Tensor]) -> torch.Tensor:
    """Non-causal attention of a block x [T, H] (normed) over the context K/V and the
    whole block -> [T, H]."""
    Hh, T = _heads(cfg, lw), x.shape[0]
    nope = cfg.qk_nope_dim
    qkva = x.float() @ lw.qkv_a.dequant().t()
    qa = ref.rms_norm(qkva[:, : cfg.q_lora_rank], lw.q_a_norm, cfg.rms_eps)
    q = (qa @ lw.q_b.dequant().t()).view(T, Hh, cfg.qk_head_dim)
    q_pe = ref.apply_rope(q[..., nope:].transpose(0, 1), cs[positions]).transpose(0, 1)
    qf = torch.cat([q[..., :nope], q_pe], dim=-1).transpose(0, 1)
    k, v = mla_kv(cfg, lw, x, positions, cs)
    if ctx_k is not None and ctx_k.shape[1]:
        k, v = torch.cat([ctx_k, k], 1), torch.cat([ctx_v, v], 1)
    s = (qf @ k.transpose(1, 2)) / math.sqrt(cfg.qk_head_dim)
    o = torch.softmax(s, dim=-1) @ v
    return o.transpose(0, 1).reshape(T, Hh * cfg.v_head_dim) @ lw.o.dequant().t()


def _draft_layer(cfg, lw, x, positions, cs, ctx):
    ck, cv = ctx

    def attn(h):
        return block_attention(cfg, lw, ref.rms_norm(h, lw.attn_norm, cfg.rms_eps), positions, cs, ck, cv)

    def ffn(h):
        h = ref.rms_norm(h, lw.ffn_norm, cfg.rms_eps)
        return ref.moe_block(cfg, lw, h) if lw.is_moe else ref.dense_ffn(cfg, lw, h)
    if lw.hc_attn is not None:
        h, post, comb = ref.hc_pre(cfg, lw.hc_attn, x)
        x = ref.hc_post(attn(h), x, post, comb)
        h, post, comb = ref.hc_pre(cfg, lw.hc_ffn, x)
        return ref.hc_post(ffn(h), x, post, comb)
    x = x + attn(x)
    return x + ffn(x)


# ------------------------------------------------------------------ drafter
@dataclass
class DSparkContext:
    """Per-sequence sliding-window context K/V of every draft layer."""
    k: List[Optional[torch.Tensor]] = field(default_factory=list)
    v: List[Optional[torch.Tensor]] = field(default_factory=list)
    end: int = 0                     # positions [end - window, end) are held


class DSparkModelDrafter:
    """The drafter the engine calls: `extend` the context with verified positions'
    aux hidden states, `propose` a block per sequence."""

    def __init__(self, mw: ModelWeights, dw: DSparkWeights, block: int, cs: torch.Tensor, markov: bool = True):
        """markov=False: DFlash -- the block's base logits alone, survival 1 everywhere."""
        self.mw, self.dw, self.block, self.cs, self.markov = mw, dw, block, cs, markov
        self.cfg = mw.cfg

    def aux_request(self) -> Dict[int, None]:
        return {li: None for li in self.dw.target_layers}

    def new_context(self) -> DSparkContext:
        n = len(self.dw.layers)
        return DSparkContext([None] * n, [None] * n, 0)

    @torch.no_grad()
    def extend(self, ctx: DSparkContext, aux: Dict[int, torch.Tensor], start: int, count: int) -> None:
        """Append positions [start, start + count) (rows [0, count) of each aux tensor)."""
        if count <= 0:
            return
        assert start == ctx.end, "context positions must arrive in order"
        dw, cfg = self.dw, self.cfg
        a = torch.cat([aux[li][:count].float() for li in dw.target_layers], dim=-1)
        main_x = ref.rms_norm(a @ dw.main_proj.dequant().t(), dw.main_norm, cfg.rms_eps)
        pos = torch.arange(start, start + count, device=main_x.device)
        for i, lw in enumerate(dw.layers):
            k, v = mla_kv(cfg, lw, main_x, pos, self.cs)
            if ctx.k[i] is not None:
                k, v = torch.cat([ctx.k[i], k], 1), torch.cat([ctx.v[i], v], 1)
            ctx.k[i], ctx.v[i] = k[:, -dw.window:], v[:, -dw.window:]
        ctx.end = start + count

    @torch.no_grad()
    def propose_one(self, ctx: DSparkContext, pending: int, pos: int):
        """-> (drafts [L], base logits [L, V], survival [L]) for one sequence whose
        pending token sits at position `pos` (== ctx.end)."""
        cfg, dw, mw, L = self.cfg, self.dw, self.mw, self.block
        ids = torch.tensor([pending] + [dw.mask_token] * (L - 1), device=mw.embed.device)
        positions = torch.arange(pos, pos + L, device=ids.device)
        x = mw.embed[ids].float()
        if cfg.hc_mult > 1:
            x = x[:, None, :].expand(-1, cfg.hc_mult, -1)
        for i, lw in enumerate(dw.layers):
            x = _draft_layer(cfg, lw, x, positions, self.cs, (ctx.k[i], ctx.v[i]))
        if cfg.hc_mult > 1:
            x = ref.hc_head(cfg, dw.hc_head, x)
        h = ref.rms_norm(x, dw.norm, cfg.rms_eps)
        base = h @ mw.lm_head.dequant().t()
        if not self.markov:
            return base.argmax(-1).cpu(), base, torch.ones(L, device=base.device)
        prev, drafts, conf = pending, [], []
        for j in range(L):                            # the sequential Markov walk
            e = dw.markov_w1[prev]
            lg = base[j] + dw.markov_w2 @ e
            conf.append(torch.sigmoid(torch.dot(dw.conf_w, torch.cat([h[j], e])) + dw.conf_b))
            prev = int(lg.argmax())
            drafts.append(prev)
        return torch.tensor(drafts), base, torch.cumprod(torch.stack(conf), 0)
