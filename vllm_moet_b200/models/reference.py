"""Pure-PyTorch fp32 reference of the MLA + MoE (+ MTP) model.

This is the oracle every native kernel and the whole GPU engine are checked
against, and the executor of the CPU engine path (BASELINE config 1 runs
without a GPU).  Weights are used dequantized (FP8 blocks and 2-bit experts
expanded to fp32); activations stay fp32.  Semantics:

* MLA (DeepSeek-V2/V3 form): q = W_qb RMSNorm(W_qa x), kv = W_kva x split
  into latent c (RMSNorm) and a shared rope key; k_nope/v = W_kvb c;
  rotate-half RoPE on the rope dims; softmax scale 1/sqrt(nope + rope).
* MoE: sigmoid scores + selection bias (optionally group-limited) or
  softmax; top-k; weights renormalised and scaled; SwiGLU experts with an
  optional clamp (gate <= L, |up| <= L, DeepSeek-V4 semantics P:6105-6151);
  shared expert added.
* MTP: h' = W_eh [RMSNorm(emb(next)); RMSNorm(h)], one decoder layer, head
  RMSNorm, shared lm_head (DeepSeek-V3 MTP module).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from ..config import ModelConfig
from .weights import LayerWeights, ModelWeights


_TP_GROUP = None


class tp_context:
    """Run the oracle as one rank of a tensor-parallel group (weights from
    ``random_weights(..., tp_rank, tp_size)``): partial outputs of the o and
    down projections are all-reduced and vocab-sharded logits all-gathered."""

    def __init__(self, group):
        self.group = group

    def __enter__(self):
        global _TP_GROUP
        self.prev, _TP_GROUP = _TP_GROUP, self.group
        return self

    def __exit__(self, *a):
        global _TP_GROUP
        _TP_GROUP = self.prev


_ATTN_IMPL = None


class attention_context:
    """Run every decoder layer's attention through `fn` (same signature as
    :func:`attention`), e.g. decode-context-parallel attention over a sharded KV."""

    def __init__(self, fn):
        self.fn = fn

    def __enter__(self):
        global _ATTN_IMPL
        self.prev, _ATTN_IMPL = _ATTN_IMPL, self.fn
        return self

    def __exit__(self, *a):
        global _ATTN_IMPL
        _ATTN_IMPL = self.prev


_MOE_IMPL = None


class moe_context:
    """Run every MoE block through `fn(cfg, lw, h)` (e.g. expert parallelism with
    all-to-all dispatch / combine over data-parallel tokens)."""

    def __init__(self, fn):
        self.fn = fn

    def __enter__(self):
        global _MOE_IMPL
        self.prev, _MOE_IMPL = _MOE_IMPL, self.fn
        return self

    def __exit__(self, *a):
        global _MOE_IMPL
        _MOE_IMPL = self.prev


def _allreduce(x: torch.Tensor) -> torch.Tensor:
    if _TP_GROUP is not None:
        import torch.distributed as dist
        x = x.contiguous()
        dist.all_reduce(x, group=_TP_GROUP)
    return x


def _gather_vocab(logits: torch.Tensor) -> torch.Tensor:
    if _TP_GROUP is None:
        return logits
    import torch.distributed as dist
    n = dist.get_world_size(_TP_GROUP)
    parts = [torch.empty_like(logits) for _ in range(n)]
    dist.all_gather(parts, logits.contiguous(), group=_TP_GROUP)
    return torch.cat(parts, dim=-1)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def rope_cos_sin(cfg: ModelConfig, max_pos: int, device="cpu") -> torch.Tensor:
    """[max_pos, rope] f32 = [cos(half) | sin(half)] for rotate-half RoPE."""
    half = cfg.qk_rope_dim // 2
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, half, dtype=torch.float64) * 2 / cfg.qk_rope_dim))
    ang = torch.arange(max_pos, dtype=torch.float64)[:, None] * inv[None, :]
    return torch.cat([ang.cos(), ang.sin()], dim=1).float().to(device)


def apply_rope(x: torch.Tensor, cs: torch.Tensor) -> torch.Tensor:
    """x [..., T, rope] with cs [T, rope]."""
    half = x.shape[-1] // 2
    c, s = cs[..., :half], cs[..., half:]
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def swiglu(gu: torch.Tensor, limit: Optional[float]) -> torch.Tensor:
    I = gu.shape[-1] // 2
    g, u = gu[..., :I], gu[..., I:]
    if limit:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    return F.silu(g) * u


def route(cfg: ModelConfig, lw: LayerWeights, x: torch.Tensor):
    """x [T, H] -> (ids [T, k] long, weights [T, k] f32)."""
    logits = x.float() @ lw.router_w.float().t()
    if cfg.router == "sigmoid":
        scores = torch.sigmoid(logits)
        sel = scores + (lw.router_bias.float() if lw.router_bias is not None else 0.0)
        if cfg.n_group > 1 and cfg.topk_group < cfg.n_group:
            T, E = sel.shape
            gs = sel.view(T, cfg.n_group, E // cfg.n_group)
            gscore = gs.topk(min(2, E // cfg.n_group), dim=-1).values.sum(-1)
            keep = torch.zeros_like(gscore, dtype=torch.bool)
            keep.scatter_(1, _stable_topk(gscore, cfg.topk_group), True)
            sel = sel.masked_fill(~keep.repeat_interleave(E // cfg.n_group, dim=1), float("-inf"))
    else:
        scores = torch.softmax(logits, dim=-1)
        sel = scores
    ids = _stable_topk(sel, cfg.top_k)
    w = scores.gather(1, ids)
    if cfg.norm_topk_prob:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return ids, w * cfg.routed_scaling


def _stable_topk(x: torch.Tensor, k: int) -> torch.Tensor:
    """Top-k indices, ties broken toward the lower index (matches the kernel)."""
    # stable sort on -value keeps index order among ties
    _, perm = torch.sort(-x, dim=1, stable=True)
    return perm[:, :k]


_TOPP = (0.0, 1)


def set_topp(p: float, min_keep: int = 1):
    """Expert top-p pruning in the oracle (mirrors MoetConfig.topp)."""
    global _TOPP
    _TOPP = (p, min_keep)


def moe_block(cfg: ModelConfig, lw: LayerWeights, h: torch.Tensor) -> torch.Tensor:
    ids, w = route(cfg, lw, h)
    if _TOPP[0] > 0:
        from .moe_policy import apply_topp
        ids, w = apply_topp(ids, w, *_TOPP)
    out = torch.zeros_like(h, dtype=torch.float32)
    ex = lw.experts
    lo, n_loc = ex.e_lo, ex.n_local
    for e in torch.unique(ids).tolist():
        if n_loc is not None and not lo <= e < lo + n_loc:
            continue            # expert parallelism: another rank owns this expert
        rows, slot = (ids == e).nonzero(as_tuple=True)
        w13, w2 = ex.dequant_expert(e - lo)
        y = swiglu(h[rows].float() @ w13.float().t(), cfg.swiglu_limit) @ w2.float().t()
        out.index_add_(0, rows, y * w[rows, slot, None])
    if lw.shared_gate_up is not None:
        out = out + swiglu(h.float() @ lw.shared_gate_up.dequant().t(), cfg.swiglu_limit) @ lw.shared_down.dequant().t()
    return out


def dense_ffn(cfg: ModelConfig, lw: LayerWeights, h: torch.Tensor) -> torch.Tensor:
    return swiglu(h.float() @ lw.gate_up.dequant().t(), None) @ lw.down.dequant().t()


class RefKV:
    """Per-sequence, per-layer cache of (k [Hh, L, qk], v [Hh, L, v]) in fp32, and of the
    DSA indexer keys [L, D] of layers with an indexer."""

    def __init__(self, n_layers: int):
        self.k = [None] * n_layers
        self.v = [None] * n_layers
        self.idx = [None] * n_layers

    def truncate(self, length: int):
        for i in range(len(self.k)):
            if self.k[i] is not None:
                self.k[i] = self.k[i][:, :length]
                self.v[i] = self.v[i][:, :length]
            if self.idx[i] is not None:
                self.idx[i] = self.idx[i][:length]


def dsa_select(cfg: ModelConfig, lw: LayerWeights, x: torch.Tensor, qa: torch.Tensor, qpos: torch.Tensor,
               cache: Optional[RefKV] = None, li: int = 0) -> Optional[torch.Tensor]:
    """DeepSeek sparse attention ("lightning indexer"): with the normed hidden x [T, H] and
    normed q_a [T, q_lora], keys k_s = W_k x_s (cached), queries q_t,h = W_q q_a and head
    weights w_t = W_w x_t give score(t, s) = sum_h w_t,h relu(q_t,h . k_s) over s <= pos(t);
    each query keeps the index_topk highest (lowest position first among ties).  Returns
    the [T, L] keep mask, or None while the context fits in index_topk (every key kept)."""
    if lw.idx_wq is None or not cfg.index_heads:
        return None
    T = x.shape[0]
    Hi, Di = cfg.index_heads, cfg.index_head_dim
    ki = x.float() @ lw.idx_wk.dequant().t()
    if cache is not None:
        if cache.idx[li] is not None:
            ki = torch.cat([cache.idx[li], ki], dim=0)
        cache.idx[li] = ki
    L = ki.shape[0]
    if L <= cfg.index_topk:
        return None
    qi = (qa.float() @ lw.idx_wq.dequant().t()).view(T, Hi, Di)
    wi = x.float() @ lw.idx_ww.dequant().t()
    sc = (torch.relu(torch.einsum("thd,sd->ths", qi, ki)) * wi[..., None]).sum(1)      # [T, L]
    kpos = torch.arange(L, device=x.device)
    sc = sc.masked_fill(kpos[None, :] > qpos[:, None], float("-inf"))
    top = _stable_topk(sc, cfg.index_topk)
    keep = torch.zeros(T, L, dtype=torch.bool, device=x.device)
    keep.scatter_(1, top, True)
    return keep


def attention(cfg: ModelConfig, lw: LayerWeights, x: torch.Tensor, positions: torch.Tensor, cs: torch.Tensor,
              cache: Optional[RefKV] = None, li: int = 0, heads: Optional[int] = None) -> torch.Tensor:
    """x [T, H] (normed), positions [T] (contiguous, appended after the cache) -> [T, H]."""
    Hh = heads or lw.q_b.shape[0] // cfg.qk_head_dim
    T = x.shape[0]
    nope, rope, vd, lat = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
    qkva = x.float() @ lw.qkv_a.dequant().t()
    qa = rms_norm(qkva[:, : cfg.q_lora_rank], lw.q_a_norm, cfg.rms_eps)
    c = rms_norm(qkva[:, cfg.q_lora_rank: cfg.q_lora_rank + lat], lw.kv_a_norm, cfg.rms_eps)
    kr = qkva[:, cfg.q_lora_rank + lat:]
    q = (qa @ lw.q_b.dequant().t()).view(T, Hh, nope + rope)
    pcs = cs[positions]
    q_nope, q_pe = q[..., :nope], apply_rope(q[..., nope:].transpose(0, 1), pcs).transpose(0, 1)
    kr = apply_rope(kr, pcs)
    kvb = (c @ lw.kv_b.dequant().t()).view(T, Hh, nope + vd)
    k = torch.cat([kvb[..., :nope], kr[:, None, :].expand(T, Hh, rope)], dim=-1).transpose(0, 1)  # [Hh,T,qk]
    v = kvb[..., nope:].transpose(0, 1)
    qf = torch.cat([q_nope, q_pe], dim=-1).transpose(0, 1)  # [Hh, T, qk]
    if cache is not None:
        if cache.k[li] is not None:
            k = torch.cat([cache.k[li], k], dim=1)
            v = torch.cat([cache.v[li], v], dim=1)
        cache.k[li], cache.v[li] = k, v
    L = k.shape[1]
    scale = 1.0 / math.sqrt(nope + rope)
    s = (qf @ k.transpose(1, 2)) * scale                   # [Hh, T, L]
    kpos = torch.arange(L, device=x.device)
    qpos = (L - T) + torch.arange(T, device=x.device)
    s = s.masked_fill(kpos[None, None, :] > qpos[None, :, None], float("-inf"))
    keep = dsa_select(cfg, lw, x, qa, qpos, cache, li)
    if keep is not None:
        s = s.masked_fill(~keep[None], float("-inf"))
    o = torch.softmax(s, dim=-1) @ v                       # [Hh, T, vd]
    return o.transpose(0, 1).reshape(T, Hh * vd) @ lw.o.dequant().t()


# ------------------------------------------------------------------ hyper-connections (mHC)
# The residual is n = hc_mult streams per token, x [T, n, H].  Around each block one
# set of mixes is computed from the RMS-scaled flattened streams (DeepSeek-V4's mHC;
# reference model: the upstream DeepSeek-V4 decoder layer, ``hc_pre`` / ``hc_post``):
#   pre  = sigmoid(m[:n] s0 + b[:n]) + eps           block input = sum_i pre_i x_i
#   post = 2 sigmoid(m[n:2n] s1 + b[n:2n])            weight of the block output per stream
#   comb = softmax_j(m[2n:] s2 + b[2n:]) made doubly stochastic by Sinkhorn iterations
#   x'_j = sum_i comb_ij x_i + post_j * block(...)
def _hc_mixes(cfg, hc, x):
    T, n, H = x.shape
    flat = x.reshape(T, n * H).float()
    return (flat @ hc.fn.float().t()) * torch.rsqrt(flat.square().mean(-1, keepdim=True) + cfg.rms_eps)


def hc_pre(cfg, hc, x):
    """x [T, n, H] -> (block input [T, H], post [T, n], comb [T, n, n])."""
    T, n, _ = x.shape
    m = _hc_mixes(cfg, hc, x)
    b, s, eps = hc.base.float(), hc.scale.float(), cfg.hc_eps
    pre = torch.sigmoid(m[:, :n] * s[0] + b[:n]) + eps
    post = 2.0 * torch.sigmoid(m[:, n:2 * n] * s[1] + b[n:2 * n])
    comb = torch.softmax(m[:, 2 * n:].view(T, n, n) * s[2] + b[2 * n:].view(n, n), dim=-1) + eps
    comb = comb / (comb.sum(-2, keepdim=True) + eps)
    for _ in range(cfg.hc_sinkhorn_iters - 1):
        comb = comb / (comb.sum(-1, keepdim=True) + eps)
        comb = comb / (comb.sum(-2, keepdim=True) + eps)
    return (pre[..., None] * x.float()).sum(1), post, comb


def hc_post(out, x, post, comb):
    """Block output [T, H] back into the streams: x'_j = sum_i comb_ij x_i + post_j out."""
    return torch.einsum("tij,tih->tjh", comb, x.float()) + post[..., None] * out.float()[:, None, :]


def hc_head(cfg, hc, x):
    """Collapse the streams before the final norm: sum_i gate_i x_i with
    gate = sigmoid(m s + b) + eps over the RMS-scaled flattened streams."""
    gate = torch.sigmoid(_hc_mixes(cfg, hc, x) * hc.scale.float()[0] + hc.base.float()) + cfg.hc_eps
    return (gate[..., None] * x.float()).sum(1)


def decoder_layer(cfg, lw, x, positions, cs, cache=None, li=0):
    """x [T, H], or [T, n, H] residual streams when the layer has hyper-connections."""
    if lw.hc_attn is not None:
        h, post, comb = hc_pre(cfg, lw.hc_attn, x)
        a = (_ATTN_IMPL or attention)(cfg, lw, rms_norm(h, lw.attn_norm, cfg.rms_eps), positions, cs, cache, li)
        a = _allreduce(a) if lw.attn_tp else a        # replicated attention: the whole output on every rank
        x = hc_post(a, x, post, comb)
        h, post, comb = hc_pre(cfg, lw.hc_ffn, x)
        h = rms_norm(h, lw.ffn_norm, cfg.rms_eps)
        f = _allreduce((_MOE_IMPL or moe_block)(cfg, lw, h) if lw.is_moe else dense_ffn(cfg, lw, h))
        return hc_post(f, x, post, comb)
    h = rms_norm(x, lw.attn_norm, cfg.rms_eps)
    a = (_ATTN_IMPL or attention)(cfg, lw, h, positions, cs, cache, li)
    x = x + (_allreduce(a) if lw.attn_tp else a)    # replicated attention: the whole output on every rank
    h = rms_norm(x, lw.ffn_norm, cfg.rms_eps)
    return x + _allreduce((_MOE_IMPL or moe_block)(cfg, lw, h) if lw.is_moe else dense_ffn(cfg, lw, h))


def forward(mw: ModelWeights, tokens: torch.Tensor, positions: torch.Tensor, cs: torch.Tensor,
            cache: Optional[RefKV] = None, aux: Optional[dict] = None):
    """-> (logits [T, V] f32, the hidden state the MTP module reads: the final normed
    hidden [T, H] f32, or with hyper-connections the streams before the head [T, n H]).
    `aux` {layer index: None}: filled with the residual after each listed layer [T, H]
    (hyper-connections: the mean of the streams) -- the aux hidden states a DSpark
    drafter reads."""
    cfg = mw.cfg
    eagle = mw.extra.get("eagle3")
    if eagle is not None:                       # EAGLE-3 drafts from the concatenated aux states
        aux = {} if aux is None else aux
        for li in eagle.target_layers:
            aux.setdefault(li, None)
    x = mw.embed[tokens].float()
    if cfg.hc_mult > 1:
        x = x[:, None, :].expand(-1, cfg.hc_mult, -1)
    for li, lw in enumerate(mw.layers):
        x = decoder_layer(cfg, lw, x, positions, cs, cache, li)
        if aux is not None and li in aux:
            aux[li] = x.mean(1) if x.dim() == 3 else x
    if eagle is not None:
        logits, _ = _head(mw, x)
        return logits, torch.cat([aux[li] for li in eagle.target_layers], -1)
    return _head(mw, x)


def _head(mw: ModelWeights, x: torch.Tensor):
    cfg = mw.cfg
    if cfg.hc_mult > 1:
        h = rms_norm(hc_head(cfg, mw.extra["hc_head"], x), mw.final_norm, cfg.rms_eps)
        return _gather_vocab(h @ mw.lm_head.dequant().t()), x.reshape(x.shape[0], -1)
    h = rms_norm(x, mw.final_norm, cfg.rms_eps)
    return _gather_vocab(h @ mw.lm_head.dequant().t()), h


def mtp_forward(mw: ModelWeights, hidden: torch.Tensor, next_tokens: torch.Tensor, positions: torch.Tensor,
                cs: torch.Tensor, cache: Optional[RefKV] = None):
    """MTP module: (h_i, token_{i+1}) at position i -> logits for token_{i+2}; returns (logits, hidden)."""
    cfg, m = mw.cfg, mw.mtp
    if mw.extra.get("eagle3") is not None:
        from .eagle3_model import eagle3_forward
        return eagle3_forward(mw, hidden, next_tokens, positions, cs, cache)
    if cfg.hc_mult > 1:
        return _mtp_forward_hc(mw, hidden, next_tokens, positions, cs, cache)
    e = rms_norm(mw.embed[next_tokens].float(), m.enorm, cfg.rms_eps)
    hn = rms_norm(hidden, m.hnorm, cfg.rms_eps)
    x = torch.cat([e, hn], dim=-1) @ m.eh_proj.dequant().t()
    x = decoder_layer(cfg, m.layer, x, positions, cs, cache, 0)
    h = rms_norm(x, m.head_norm, cfg.rms_eps)
    return _gather_vocab(h @ mw.lm_head.dequant().t()), h


def _mtp_forward_hc(mw, hidden, next_tokens, positions, cs, cache):
    """The MTP module over residual streams: `hidden` [T, n H] is the main model's (or
    the previous draft's) pre-head streams.  Each stream is normed and projected by the
    hidden half of eh_proj, the normed next-token embedding by its embedding half is
    added to every stream (the embedding is zero at position 0, as DeepSeek-V4's MTP
    masks it), then the MTP layer runs on the streams; logits come from the module's own
    stream reduction, its head norm and the shared head.  -> (logits, streams [T, n H])."""
    cfg, m = mw.cfg, mw.mtp
    n, H = cfg.hc_mult, cfg.hidden
    T = hidden.shape[0]
    emb = mw.embed[next_tokens].float() * (positions != 0).float()[:, None]
    e = rms_norm(emb, m.enorm, cfg.rms_eps)
    hn = rms_norm(hidden.float().view(T, n, H), m.hnorm, cfg.rms_eps)
    w = m.eh_proj.dequant().float()
    x = hn @ w[:, H:].t() + (e @ w[:, :H].t())[:, None, :]
    x = decoder_layer(cfg, m.layer, x, positions, cs, cache, 0)
    h = rms_norm(hc_head(cfg, m.hc_head, x), m.head_norm, cfg.rms_eps)
    return _gather_vocab(h @ mw.lm_head.dequant().t()), x.reshape(T, n * H)


def greedy_generate(mw: ModelWeights, prompt: list, max_tokens: int) -> list:
    """Full-recompute greedy decoding (no cache): the end-to-end oracle."""
    cs = rope_cos_sin(mw.cfg, len(prompt) + max_tokens + 8, device=mw.embed.device)
    toks = list(prompt)
    out = []
    for _ in range(max_tokens):
        t = torch.tensor(toks, device=mw.embed.device)
        logits, _ = forward(mw, t, torch.arange(len(toks), device=t.device), cs)
        nxt = int(logits[-1].argmax())
        out.append(nxt)
        toks.append(nxt)
    return out
