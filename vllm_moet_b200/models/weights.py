"""Model weights: containers, expert slot layout, and synthetic random init.

Dense stack: FP8 e4m3 with UE8M0 128x128 block scales (:class:`Fp8Linear`),
NVFP4 (:class:`Nvfp4Linear`, the GLM dense format; the GPU runner serves it as FP8),
or plain float for the CPU tiny model.  Routed experts: one slot per expert
holding ``[codes13 | sc13 | codes2 | sc2]`` -- the fragment-major 2-bit
planes of the fused gate/up matrix [2I, H] and of the down matrix [H, I]
with their UE8M0 scale planes (the pack-row section order of the
reference's base tier, P:12830-12869).  A layer's experts live in one pool
tensor [E, slot_bytes] addressed through an expert -> slot table, so the
residency tiers can swap the pool for a cache without touching kernels.

Random init follows the benchmark configs: N(0, 0.02) weights; experts go
through NVFP4 (e2m1 + e4m3 block-16 + f32 tensor scale) and are then
re-quantised to the 2-bit codebook (GPU kernels on CUDA, the golden torch
pipeline on CPU).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import torch

from ..config import ModelConfig
from ..formats import codebook, fp8, planes


# --------------------------------------------------------------------------
@dataclass
class Fp8Linear:
    """y = x W^T with W [N, K] in e4m3 (uint8 storage) + UE8M0 [ceil(N/128), ceil(K/128)]."""
    w: torch.Tensor
    s: torch.Tensor

    @property
    def shape(self):
        return tuple(self.w.shape)

    @classmethod
    def from_float(cls, w: torch.Tensor) -> "Fp8Linear":
        q, s = fp8.quant_weight_fp8(w)
        return cls(q.view(torch.uint8), s)

    def dequant(self) -> torch.Tensor:
        return fp8.dequant_weight_fp8(self.w.view(torch.float8_e4m3fn), self.s)

    def to(self, device) -> "Fp8Linear":
        return Fp8Linear(self.w.to(device), self.s.to(device))


@dataclass
class FloatLinear:
    w: torch.Tensor

    @property
    def shape(self):
        return tuple(self.w.shape)

    def dequant(self) -> torch.Tensor:
        return self.w.float()

    def to(self, device) -> "FloatLinear":
        return FloatLinear(self.w.to(device))


@dataclass
class Nvfp4Linear:
    """y = x W^T with W [N, K] in NVFP4: packed e2m1 pairs [N, K/2] (low nibble = even k),
    e4m3 block-16 scales [N, K/16] and an f32 tensor scale (the GLM dense format)."""
    w: torch.Tensor
    s: torch.Tensor
    s2: torch.Tensor

    @property
    def shape(self):
        return (self.w.shape[0], self.w.shape[1] * 2)

    @classmethod
    def from_float(cls, w: torch.Tensor) -> "Nvfp4Linear":
        packed, sf, t2 = codebook.f32_to_nvfp4(w.float().cpu())
        return cls(packed.to(w.device), sf.to(w.device), t2.to(w.device))

    def dequant(self) -> torch.Tensor:
        vals = codebook.E2M1_VALUES.to(self.w.device)[codebook.split_packed_e2m1(self.w).long()].float()
        return vals * self.s.float().repeat_interleave(16, dim=1) * self.s2.float()

    def to(self, device) -> "Nvfp4Linear":
        return Nvfp4Linear(self.w.to(device), self.s.to(device), self.s2.to(device))


def make_linear(w: torch.Tensor, dtype: str):
    if dtype == "fp8":
        return Fp8Linear.from_float(w)
    if dtype == "nvfp4" and w.shape[-1] % 16 == 0:
        return Nvfp4Linear.from_float(w)
    return FloatLinear(w.float())


# --------------------------------------------------------------------------
@dataclass
class ExpertLayout:
    """Byte layout of one expert slot [codes13 | sc13 | codes2 | sc2]."""
    H: int
    I: int

    @property
    def codes13(self) -> int:
        return planes.codes_plane_bytes(2 * self.I, self.H)

    @property
    def sc13(self) -> int:
        return planes.scale_plane_bytes(2 * self.I, self.H)

    @property
    def codes2(self) -> int:
        return planes.codes_plane_bytes(self.H, self.I)

    @property
    def sc2(self) -> int:
        return planes.scale_plane_bytes(self.H, self.I)

    @property
    def off_codes13(self) -> int:
        return 0

    @property
    def off_sc13(self) -> int:
        return self.codes13

    @property
    def off_codes2(self) -> int:
        return self.codes13 + self.sc13

    @property
    def off_sc2(self) -> int:
        return self.codes13 + self.sc13 + self.codes2

    @property
    def slot_bytes(self) -> int:
        return self.codes13 + self.sc13 + self.codes2 + self.sc2

    def split(self, slot: torch.Tensor):
        o = [0, self.codes13, self.sc13, self.codes2, self.sc2]
        c = [sum(o[: i + 1]) for i in range(5)]
        return tuple(slot[..., c[i]:c[i + 1]] for i in range(4))


@dataclass
class ExpertPool:
    """All routed experts of one layer: pool [E, slot_bytes] + slot table [E]."""
    layout: ExpertLayout
    pool: torch.Tensor
    slot_table: torch.Tensor
    # CPU tiny config with fp16 group scales keeps dequantized matrices instead
    dense_w13: Optional[torch.Tensor] = None
    dense_w2: Optional[torch.Tensor] = None
    e_lo: int = 0                  # expert parallelism: this rank holds experts [e_lo, e_lo + n_local)
    n_local: Optional[int] = None
    delta_rows: Optional[torch.Tensor] = None     # [E, delta slot bytes] FP4 delta-tier rows (host)

    def dequant_expert(self, e: int):
        """-> (w13 [2I, H], w2 [H, I]) float32."""
        if self.dense_w13 is not None:
            return self.dense_w13[e], self.dense_w2[e]
        L = self.layout
        c13, s13, c2, s2 = L.split(self.pool[int(self.slot_table[e])])
        w13 = planes.dequant_plane(c13.cpu(), s13.cpu(), 2 * L.I, L.H)
        w2 = planes.dequant_plane(c2.cpu(), s2.cpu(), L.H, L.I)
        return w13.to(self.pool.device), w2.to(self.pool.device)


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    qkv_a: object                  # [q_lora + kv_lora + rope, H]
    q_a_norm: torch.Tensor
    kv_a_norm: torch.Tensor
    q_b: object                    # [Hh*(nope+rope), q_lora]
    kv_b: object                   # [Hh*(nope+v), kv_lora]
    o: object                      # [H, Hh*v]
    ffn_norm: torch.Tensor
    # dense FFN
    gate_up: object = None         # [2I, H]
    down: object = None            # [H, I]
    # MoE
    router_w: Optional[torch.Tensor] = None     # [E, H] f32
    router_bias: Optional[torch.Tensor] = None  # [E] f32
    experts: Optional[ExpertPool] = None
    shared_gate_up: object = None
    shared_down: object = None
    # absorbed MLA decode weights (derived from kv_b)
    w_uk_t: Optional[Fp8Linear] = None          # [Hh, kv_lora, nope]
    w_uv: Optional[Fp8Linear] = None            # [Hh, v, kv_lora]
    # sparse indexer (GLM shape)
    idx_wq: object = None          # [Hi*D, q_lora] indexer queries (from the normed q_a)
    idx_wk: object = None          # [D, H] indexer key (from the normed hidden)
    idx_ww: object = None          # [Hi, H] per-head weights (softmax-free, scaled by 1/sqrt(Hi*D))
    # hyper-connections (cfg.hc_mult > 1)
    attn_tp: bool = True                        # False: attention weights whole on every TP rank
    hc_attn: Optional["HyperConn"] = None
    hc_ffn: Optional["HyperConn"] = None

    @property
    def is_moe(self) -> bool:
        return self.experts is not None


@dataclass
class HyperConn:
    """Mixing parameters of one hyper-connection site (f32).  Around a block: `fn`
    [(2 + n) n, n H] with `base` [(2 + n) n] and `scale` [3] give the pre / post /
    n x n residual mixes; at a head: `fn` [n, n H], `base` [n], `scale` [1]."""
    fn: torch.Tensor
    base: torch.Tensor
    scale: torch.Tensor


@dataclass
class MTPWeights:
    enorm: torch.Tensor
    hnorm: torch.Tensor
    eh_proj: object                # [H, 2H]
    layer: LayerWeights
    head_norm: torch.Tensor
    hc_head: Optional[HyperConn] = None


@dataclass
class ModelWeights:
    cfg: ModelConfig
    embed: torch.Tensor            # [V, H] bf16
    layers: list
    final_norm: torch.Tensor
    lm_head: object                # [V, H]
    mtp: Optional[MTPWeights] = None
    tp_rank: int = 0
    tp_size: int = 1
    extra: dict = field(default_factory=dict)


# --------------------------------------------------------------------------
def _derive_absorb(kv_b, cfg: ModelConfig, heads: int):
    """kv_b [Hh*(nope+v), kv_lora] -> W_uk^T [Hh, kv_lora, nope], W_uv [Hh, v, kv_lora] (FP8)."""
    w = kv_b.dequant().view(heads, cfg.qk_nope_dim + cfg.v_head_dim, cfg.kv_lora_rank)
    wuk_t = w[:, : cfg.qk_nope_dim, :].transpose(1, 2).contiguous()        # [Hh, 512, nope]
    wuv = w[:, cfg.qk_nope_dim:, :].contiguous()                           # [Hh, v, 512]
    qs = [Fp8Linear.from_float(wuk_t[h]) for h in range(heads)]
    vs = [Fp8Linear.from_float(wuv[h]) for h in range(heads)]
    return (Fp8Linear(torch.stack([q.w for q in qs]), torch.stack([q.s for q in qs])),
            Fp8Linear(torch.stack([v.w for v in vs]), torch.stack([v.s for v in vs])))


class _Rng:
    """Deterministic normal generator on a device (seeded per named tensor)."""

    def __init__(self, seed: int, device):
        self.seed = seed
        self.device = torch.device(device)
        self.gen = torch.Generator(device=self.device)
        self.counter = 0

    def normal(self, shape, std=0.02):
        self.counter += 1
        self.gen.manual_seed(self.seed * 1000003 + self.counter)
        return torch.randn(shape, generator=self.gen, device=self.device, dtype=torch.float32) * std


def quantize_experts_gpu(w13: torch.Tensor, w2: torch.Tensor, layout: ExpertLayout, out_pool: torch.Tensor,
                         zero_mode: str = "auto"):
    """Random-init float experts [n, 2I, H], [n, H, I] (cuda) -> 2-bit slots in out_pool [n, slot_bytes]
    via NVFP4 then the 2-bit requant+pack, all n experts per matrix in three kernel launches
    (per-expert tensor scales and the zero-sign "auto" rule stay on the device, no host sync)."""
    from ..ops import native
    C = native()
    n = w13.shape[0]
    if n == 0:
        return
    mode = {"sign": 0, "alt": 1, "auto": 2}[zero_mode]
    for mat, off_c, off_s in ((w13, layout.off_codes13, layout.off_sc13), (w2, layout.off_codes2, layout.off_sc2)):
        mat = mat.contiguous()
        _, N, K = mat.shape
        # the host rule float(max|w|) / (6 * 448), 1.0 for an all-zero matrix, in double
        amax = mat.abs().amax(dim=(1, 2)).double()
        ts = torch.where(amax > 0, amax / (6.0 * 448.0), torch.ones_like(amax))
        packed = torch.empty(n, N, K // 2, dtype=torch.uint8, device=mat.device)
        sf = torch.empty(n, N, K // 16, dtype=torch.uint8, device=mat.device)
        counters = torch.zeros(n, 2, dtype=torch.int64, device=mat.device)
        C.experts_quant_pack(mat, ts, packed, sf, counters, out_pool, off_c, off_s, mode)


def quantize_experts_cpu(w13: torch.Tensor, w2: torch.Tensor, layout: ExpertLayout, out_pool: torch.Tensor,
                         zero_mode: str = "auto", want_nibbles: bool = False):
    """Golden torch pipeline (NVFP4 -> f64 -> 2-bit) for CPU / tests.  With
    want_nibbles, also -> the e2m1 nibbles (w13, w2) of the last expert, the exact
    values the codes were taken from (the split-FP4 refinement source)."""
    nibs = None
    for e in range(w13.shape[0]):
        nibs = []
        for (mat, off_c, off_s) in ((w13[e], layout.off_codes13, layout.off_sc13),
                                    (w2[e], layout.off_codes2, layout.off_sc2)):
            N, K = mat.shape
            ts = float(mat.abs().max()) / (6.0 * 448.0) or 1.0
            packed, sf, t2 = codebook.f32_to_nvfp4(mat.float().cpu(), ts)
            codes, sc, nib = codebook.nvfp4_to_codes_scales(packed, sf, t2, mode=zero_mode, want_nibbles=want_nibbles)
            out_pool[e, off_c:off_c + N * K // 4] = planes.pack_codes(codes).to(out_pool.device)
            out_pool[e, off_s:off_s + N * K // 32] = planes.pack_scales(sc).to(out_pool.device)
            nibs.append(nib)
    return tuple(nibs) if want_nibbles else None


def _pad_to(n: int, m: int) -> int:
    return -(-n // m) * m


def tp_ffn_shard(I: int, tp_size: int, dtype: str) -> int:
    """Per-rank intermediate size of a TP-sharded dense FFN: I/tp rounded up to the
    128-row FP8 block (zero rows/columns pad the shard; silu(0) * 0 adds nothing)."""
    per = -(-I // tp_size)
    return _pad_to(per, 128) if dtype == "fp8" else per


def _shard_ffn(gu: torch.Tensor, down: torch.Tensor, I: int, tp_rank: int, tp_size: int, Ip: int):
    """Column-parallel gate/up [2I, H] and row-parallel down [H, I] -> this rank's
    [2Ip, H] and [H, Ip] (gate rows first, then up rows)."""
    if tp_size == 1 and Ip == I:
        return gu, down
    per = -(-I // tp_size)
    lo, hi = tp_rank * per, min(I, (tp_rank + 1) * per)
    n = max(0, hi - lo)
    H = gu.shape[1]
    g = gu.new_zeros((2 * Ip, H))
    d = down.new_zeros((down.shape[0], Ip))
    g[:n] = gu[lo:hi]
    g[Ip:Ip + n] = gu[I + lo:I + hi]
    d[:, :n] = down[:, lo:hi]
    return g, d


def _make_layer(cfg: ModelConfig, rng: _Rng, li: int, dev, moe: bool, tp_rank=0, tp_size=1,
                expert_chunk: int = 16, with_delta: bool = False, ep: bool = False,
                expert_source=None, attn_tp: bool = True) -> LayerWeights:
    """One decoder layer, sharded for rank `tp_rank` of a `tp_size` tensor-parallel
    group.  Full matrices are drawn first (the same draws for every TP size) and
    then sliced, so TP runs compute the same function as one GPU:
      * MLA: q_b / kv_b rows and o columns split by head (q_a / kv_a replicated);
      * dense FFN and shared expert: gate/up rows and down columns split, each
        shard zero-padded to the FP8 block;
      * routed experts: every expert's intermediate dimension split (w13 rows,
        w2 columns), so each rank streams 1/tp of every routed expert.
    With ``attn_tp=False`` the attention weights stay whole on every rank (replicated
    attention: its output needs no reduction); the FFN / experts are still sharded."""
    H, dt = cfg.hidden, cfg.dense_dtype
    rng.counter = 1000 * (li + 1)      # per-layer draw stream: a layer's weights do not depend on which
    nh = cfg.num_heads                 # other layers a (pipeline) stage builds
    assert nh % tp_size == 0, "num_heads must divide by the TP size"
    a_rank, a_size = (tp_rank, tp_size) if attn_tp else (0, 1)
    Hh = nh // a_size
    qk = cfg.qk_head_dim
    nope_v = cfg.qk_nope_dim + cfg.v_head_dim
    lin = lambda w: make_linear(w, dt)  # noqa: E731
    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
    q_lora = cfg.q_lora_rank
    h0, h1 = a_rank * Hh, (a_rank + 1) * Hh
    q_b = rng.normal((nh * qk, q_lora))[h0 * qk:h1 * qk]
    kv_b = rng.normal((nh * nope_v, cfg.kv_lora_rank))[h0 * nope_v:h1 * nope_v]
    o = rng.normal((H, nh * cfg.v_head_dim))[:, h0 * cfg.v_head_dim:h1 * cfg.v_head_dim]
    lw = LayerWeights(
        attn_norm=ones(H),
        qkv_a=lin(rng.normal((q_lora + cfg.kv_lora_rank + cfg.qk_rope_dim, H))),
        q_a_norm=ones(q_lora),
        kv_a_norm=ones(cfg.kv_lora_rank),
        q_b=lin(q_b.contiguous()),
        kv_b=lin(kv_b.contiguous()),
        o=lin(o.contiguous()),
        ffn_norm=ones(H),
        attn_tp=attn_tp or tp_size == 1,
    )
    if isinstance(lw.kv_b, Fp8Linear):
        lw.w_uk_t, lw.w_uv = _derive_absorb(lw.kv_b, cfg, Hh)
    if cfg.index_heads:     # DSA indexer (replicated across TP ranks); its own draw stream
        Hi, Di = cfg.index_heads, cfg.index_head_dim
        saved, rng.counter = rng.counter, 1000 * (li + 1) + 900
        lw.idx_wq = lin(rng.normal((Hi * Di, q_lora)))
        lw.idx_wk = lin(rng.normal((Di, H)))
        lw.idx_ww = lin(rng.normal((Hi, H)) / math.sqrt(Hi * Di))
        rng.counter = saved
    if not moe:
        I = cfg.dense_intermediate
        Ip = tp_ffn_shard(I, tp_size, dt) if tp_size > 1 else I
        gu, dn = _shard_ffn(rng.normal((2 * I, H)), rng.normal((H, I)), I, tp_rank, tp_size, Ip)
        lw.gate_up, lw.down = lin(gu.contiguous()), lin(dn.contiguous())
        return lw
    E, Ifull = cfg.num_experts, cfg.moe_intermediate
    if ep:      # expert parallelism: whole experts, E / tp of them per rank
        assert E % tp_size == 0, "num_experts must divide by the EP size"
        I = Ifull
        e_lo, n_loc = tp_rank * (E // tp_size), E // tp_size
    else:       # tensor parallelism: every expert's intermediate dimension split
        assert Ifull % tp_size == 0 and (Ifull // tp_size) % 64 == 0, "expert intermediate / tp must be a multiple of 64"
        I = Ifull // tp_size
        e_lo, n_loc = 0, E
    lw.router_w = rng.normal((E, H)).to(torch.bfloat16).float()   # bf16-valued gate weights
    lw.router_bias = torch.zeros(E, dtype=torch.float32, device=dev)
    if cfg.num_shared_experts:
        Is = cfg.moe_intermediate * cfg.num_shared_experts
        Isp = tp_ffn_shard(Is, tp_size, dt) if tp_size > 1 else Is
        gu, dn = _shard_ffn(rng.normal((2 * Is, H)), rng.normal((H, Is)), Is, tp_rank, tp_size, Isp)
        lw.shared_gate_up, lw.shared_down = lin(gu.contiguous()), lin(dn.contiguous())
    layout = ExpertLayout(H=H, I=I)
    lo = 0 if ep else tp_rank * I

    def shard13(w):   # [.., 2*Ifull, H] -> [.., 2I, H]
        return torch.cat([w[..., lo:lo + I, :], w[..., Ifull + lo:Ifull + lo + I, :]], dim=-2).contiguous()

    def shard2(w):    # [.., H, Ifull] -> [.., H, I]
        return w[..., lo:lo + I].contiguous()

    if cfg.expert_scale == "fp16_amax4":
        # CPU tiny config: fp16 group-32 scale = max|w|/4; keep the dequantized experts
        w13s, w2s = [], []
        for e in range(E):
            a = shard13(rng.normal((2 * Ifull, H))); b = shard2(rng.normal((H, Ifull)))
            c, s = codebook.f32_to_codes_fp16_amax4(a); w13s.append(codebook.dequant_codes_fp16(c, s))
            c, s = codebook.f32_to_codes_fp16_amax4(b); w2s.append(codebook.dequant_codes_fp16(c, s))
        pool = torch.zeros(E, 16, dtype=torch.uint8, device=dev)
        lw.experts = ExpertPool(layout, pool, torch.arange(E, dtype=torch.int32, device=dev),
                                dense_w13=torch.stack(w13s), dense_w2=torch.stack(w2s))
        if ep:
            lw.experts.dense_w13 = lw.experts.dense_w13[e_lo:e_lo + n_loc]
            lw.experts.dense_w2 = lw.experts.dense_w2[e_lo:e_lo + n_loc]
            lw.experts.e_lo, lw.experts.n_local = e_lo, n_loc
        return lw
    pool = torch.empty(n_loc, layout.slot_bytes, dtype=torch.uint8, device=dev)
    delta_rows = [] if with_delta else None
    # boot from a persistent cache (planes cache / pack): the quantised rows of this layer
    cached = expert_source.load(li, n_loc, layout.slot_bytes) if expert_source is not None and not with_delta else None
    if cached is not None:
        pool.copy_(cached.view(n_loc, layout.slot_bytes))
        rng.counter += 2 * ((E + expert_chunk - 1) // expert_chunk)   # keep later draws aligned
        lw.experts = ExpertPool(layout, pool, torch.arange(n_loc, dtype=torch.int32, device=dev), e_lo=e_lo,
                                n_local=n_loc if ep else None)
        return lw
    for e0 in range(0, E, expert_chunk):
        n = min(expert_chunk, E - e0)
        a, b = max(e0, e_lo), min(e0 + n, e_lo + n_loc)     # local experts of this chunk
        if a >= b:
            rng.counter += 2          # skip the chunk's two draws without generating them
            continue
        w13 = shard13(rng.normal((n, 2 * Ifull, H)))[a - e0:b - e0]
        w2 = shard2(rng.normal((n, H, Ifull)))[a - e0:b - e0]
        n, e0 = b - a, a - e_lo
        if with_delta == "split":        # base + refinement from one quantiser run (host side)
            from ..residency.delta import pack_split_slot
            for i in range(n):
                nibs = quantize_experts_cpu(w13[i:i + 1], w2[i:i + 1], layout, pool[e0 + i:e0 + i + 1],
                                            want_nibbles=True)
                delta_rows.append(pack_split_slot(*nibs))
        elif torch.device(dev).type == "cuda":
            quantize_experts_gpu(w13, w2, layout, pool[e0:e0 + n])
        else:
            quantize_experts_cpu(w13, w2, layout, pool[e0:e0 + n])
        if delta_rows is not None and with_delta != "split":   # FP4 delta-tier rows of the same experts
            from ..residency.delta import pack_delta_slot
            delta_rows += [pack_delta_slot(w13[i], w2[i]) for i in range(n)]
        del w13, w2
    lw.experts = ExpertPool(layout, pool, torch.arange(n_loc, dtype=torch.int32, device=dev), e_lo=e_lo,
                            n_local=n_loc if ep else None)
    if expert_source is not None:        # streaming first-boot build: persist the layer as soon as it exists
        expert_source.store(li, pool)
    if delta_rows is not None:
        lw.experts.delta_rows = torch.stack(delta_rows)
    return lw


def _vocab_shard(w: torch.Tensor, tp_rank: int, tp_size: int) -> torch.Tensor:
    """Rows [r*V/tp, (r+1)*V/tp) of a [V, H] head (vocab-parallel lm_head)."""
    if tp_size == 1:
        return w
    V = w.shape[0]
    assert V % tp_size == 0, "vocab must divide by the TP size"
    per = V // tp_size
    return w[tp_rank * per:(tp_rank + 1) * per].contiguous()


def pp_layer_range(num_layers: int, pp_rank: int, pp_size: int):
    """Contiguous, balanced layer range of a pipeline stage."""
    per, extra = divmod(num_layers, pp_size)
    l0 = pp_rank * per + min(pp_rank, extra)
    return l0, l0 + per + (1 if pp_rank < extra else 0)


def random_weights(cfg: ModelConfig, device="cpu", seed: int = 0, tp_rank: int = 0, tp_size: int = 1,
                   with_mtp: bool = True, num_layers: Optional[int] = None, pp_rank: int = 0,
                   pp_size: int = 1, with_delta: bool = False, expert_parallel: bool = False,
                   expert_source=None, attn_tp: bool = True) -> ModelWeights:
    """Synthetic random-init weights of the given architecture (N(0, 0.02)).
    With pp_size > 1 only the stage's layers are built; the first stage holds
    the embedding, the last the final norm, the head and the MTP module."""
    dev = torch.device(device)
    rng = _Rng(seed, dev)
    H = cfg.hidden
    L = cfg.num_layers if num_layers is None else num_layers
    l0, l1 = pp_layer_range(L, pp_rank, pp_size)
    first, last = pp_rank == 0, pp_rank == pp_size - 1
    rng.counter = 0
    embed = rng.normal((cfg.vocab, H)).to(torch.bfloat16) if first else None
    layers = [_make_layer(cfg, rng, i, dev, cfg.is_moe_layer(i), tp_rank, tp_size, with_delta=with_delta,
                          ep=expert_parallel, expert_source=expert_source, attn_tp=attn_tp) for i in range(l0, l1)]
    head = None
    if last:
        rng.counter = 1
        head = make_linear(_vocab_shard(rng.normal((cfg.vocab, H)), tp_rank, tp_size), cfg.dense_dtype)
    mw = ModelWeights(cfg=cfg, embed=embed, layers=layers,
                      final_norm=torch.ones(H, dtype=torch.bfloat16, device=dev),
                      lm_head=head, tp_rank=tp_rank, tp_size=tp_size)
    mw.extra.update(layer_range=(l0, l1), pp_rank=pp_rank, pp_size=pp_size)
    if with_mtp and cfg.num_mtp_layers and last:
        rng.counter = 2
        eh = make_linear(rng.normal((H, 2 * H)), cfg.dense_dtype)
        # the MTP module shares the head; its embedding copy lives on the last stage
        if mw.embed is None:
            rng.counter = 0
            mw.extra["mtp_embed"] = rng.normal((cfg.vocab, H)).to(torch.bfloat16)
        mw.mtp = MTPWeights(
            enorm=torch.ones(H, dtype=torch.bfloat16, device=dev),
            hnorm=torch.ones(H, dtype=torch.bfloat16, device=dev),
            eh_proj=eh,
            layer=_make_layer(cfg, rng, L, dev, True, tp_rank, tp_size, with_delta=with_delta, ep=expert_parallel,
                              expert_source=expert_source, attn_tp=attn_tp),
            head_norm=torch.ones(H, dtype=torch.bfloat16, device=dev))
    if cfg.hc_mult > 1:
        random_hyper_connections(mw, seed, L)
    return mw


def random_hyper_connections(mw: ModelWeights, seed: int = 0, num_layers: Optional[int] = None) -> None:
    """Random mHC parameters for every layer (and the MTP layer), plus the heads' reductions.
    Drawn from their own generator, so the other weights match the hc_mult = 1 model."""
    cfg = mw.cfg
    n, H = cfg.hc_mult, cfg.hidden
    dev = mw.final_norm.device
    g = torch.Generator().manual_seed(seed * 7919 + 17)

    def site(rows):
        fn = torch.randn(rows, n * H, generator=g) * 0.02
        base = torch.randn(rows, generator=g) * 0.5
        scale = 0.5 + torch.rand(3 if rows > n else 1, generator=g)
        return HyperConn(fn.to(dev), base.to(dev), scale.to(dev))
    L = cfg.num_layers if num_layers is None else num_layers
    l0 = mw.extra.get("layer_range", (0, len(mw.layers)))[0]
    for i in range(L + 1):                         # one draw order whatever the PP slice
        a, f = site((2 + n) * n), site((2 + n) * n)
        if l0 <= i < l0 + len(mw.layers):
            mw.layers[i - l0].hc_attn, mw.layers[i - l0].hc_ffn = a, f
        elif i == L and mw.mtp is not None:
            mw.mtp.layer.hc_attn, mw.mtp.layer.hc_ffn = a, f
    head, mtp_head = site(n), site(n)
    if mw.lm_head is not None:
        mw.extra["hc_head"] = head
    if mw.mtp is not None:
        mw.mtp.hc_head = mtp_head
