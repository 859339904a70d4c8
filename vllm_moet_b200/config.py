"""Typed model / engine configuration with validation at construction.

Model presets follow the five benchmark shapes this engine is measured on:
a CPU-sized tiny MoE, a DeepSeek-V4-Flash-shaped MoE (the headline), a
GLM-5.2-shaped MoE with a sparse indexer, and a Kimi-K2-shaped MoE.

The reference keeps these knobs in ~120 ``VLLM_MOE_W2_*`` environment
variables read at import (patch ``vllm/envs.py``, P:2907-2977); here one
dataclass per concern carries them, and :func:`MoetConfig.from_env` maps the
user-facing env names onto fields so recipes written for the reference keep
working.
"""
from __future__ import annotations

import dataclasses
import os
from dataclasses import dataclass, field
from typing import Optional


@dataclass(frozen=True)
class ModelConfig:
    name: str
    num_layers: int
    hidden: int
    vocab: int
    # dense FFN (first `num_dense_layers` layers)
    num_dense_layers: int
    dense_intermediate: int
    # MLA attention
    num_heads: int
    q_lora_rank: Optional[int]
    kv_lora_rank: int
    qk_nope_dim: int
    qk_rope_dim: int
    v_head_dim: int
    # MoE
    num_experts: int
    moe_intermediate: int
    top_k: int
    num_shared_experts: int
    router: str = "sigmoid"          # "sigmoid" (noaux bias) | "softmax"
    n_group: int = 1
    topk_group: int = 1
    norm_topk_prob: bool = True
    routed_scaling: float = 1.0
    swiglu_limit: Optional[float] = None
    # sparse indexer (DSA); 0 heads = dense MLA
    index_heads: int = 0
    index_head_dim: int = 128
    index_topk: int = 2048
    # MTP
    num_mtp_layers: int = 1
    # hyper-connections (mHC): hc_mult residual streams per token, mixed around every
    # attention / FFN block; 1 = a plain residual
    hc_mult: int = 1
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    rope_theta: float = 10000.0
    rms_eps: float = 1e-6
    max_position: int = 163840
    # precisions
    dense_dtype: str = "fp8"         # "fp8" (e4m3, UE8M0 block-128) | "bf16" | "nvfp4"
    expert_format: str = "w2"        # "w2" sign-symmetric 2-bit codebook
    expert_scale: str = "ue8m0"      # "ue8m0" block-32 | "fp16_amax4" (tiny CPU config)

    def __post_init__(self):
        if self.hidden % 128:
            raise ValueError("hidden must be a multiple of 128")
        if self.moe_intermediate % 64 or self.hidden % 64:
            raise ValueError("expert dims must be multiples of 64 (fragment-major planes)")
        if self.top_k > self.num_experts:
            raise ValueError("top_k > num_experts")
        if self.router not in ("sigmoid", "softmax"):
            raise ValueError(f"unknown router {self.router!r}")
        if self.num_experts % self.n_group:
            raise ValueError("num_experts must divide into n_group groups")
        if self.hc_mult < 1 or self.hc_sinkhorn_iters < 1:
            raise ValueError("hc_mult and hc_sinkhorn_iters must be >= 1")

    @property
    def qk_head_dim(self) -> int:
        return self.qk_nope_dim + self.qk_rope_dim

    @property
    def kv_dim(self) -> int:
        """Latent KV row width: compressed latent + shared rope key."""
        return self.kv_lora_rank + self.qk_rope_dim

    def is_moe_layer(self, i: int) -> bool:
        return i >= self.num_dense_layers

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def expert_param_count(self) -> int:
        return 3 * self.hidden * self.moe_intermediate


def tiny_config(**kw) -> ModelConfig:
    """CPU tiny MoE (2 layers, hidden 256, vocab 1024)."""
    base = dict(
        name="tiny-moe", num_layers=2, hidden=256, vocab=1024,
        num_dense_layers=0, dense_intermediate=512,
        num_heads=4, q_lora_rank=128, kv_lora_rank=64, qk_nope_dim=32,
        qk_rope_dim=16, v_head_dim=32,
        num_experts=8, moe_intermediate=128, top_k=2, num_shared_experts=1,
        router="softmax", norm_topk_prob=False, routed_scaling=1.0,
        dense_dtype="bf16", expert_scale="fp16_amax4", max_position=4096)
    base.update(kw)
    return ModelConfig(**base)


def ds4_flash_config(**kw) -> ModelConfig:
    """DeepSeek-V4-Flash-shaped MoE (~155B)."""
    base = dict(
        name="ds4-flash-shape", num_layers=32, hidden=4096, vocab=129280,
        num_dense_layers=1, dense_intermediate=11008,
        num_heads=32, q_lora_rank=1024, kv_lora_rank=512, qk_nope_dim=128,
        qk_rope_dim=64, v_head_dim=128,
        num_experts=256, moe_intermediate=1536, top_k=8, num_shared_experts=1,
        router="sigmoid", n_group=1, topk_group=1, norm_topk_prob=True,
        routed_scaling=2.5, swiglu_limit=10.0, dense_dtype="fp8")
    base.update(kw)
    return ModelConfig(**base)


def glm52_config(**kw) -> ModelConfig:
    """GLM-5.2-shaped MoE (~750B) with a DSA indexer."""
    base = dict(
        name="glm-5.2-shape", num_layers=78, hidden=6144, vocab=154880,
        num_dense_layers=3, dense_intermediate=16384,
        num_heads=64, q_lora_rank=2048, kv_lora_rank=512, qk_nope_dim=192,
        qk_rope_dim=64, v_head_dim=256,
        num_experts=256, moe_intermediate=2048, top_k=8, num_shared_experts=1,
        router="sigmoid", n_group=1, topk_group=1, routed_scaling=2.5,
        index_heads=32, index_head_dim=128, index_topk=2048,
        dense_dtype="nvfp4")
    base.update(kw)
    return ModelConfig(**base)


def kimi_k2_config(**kw) -> ModelConfig:
    """Kimi-K2-shaped MoE (~1T)."""
    base = dict(
        name="kimi-k2-shape", num_layers=61, hidden=7168, vocab=163840,
        num_dense_layers=1, dense_intermediate=18432,
        num_heads=64, q_lora_rank=1536, kv_lora_rank=512, qk_nope_dim=128,
        qk_rope_dim=64, v_head_dim=128,
        num_experts=384, moe_intermediate=2048, top_k=8, num_shared_experts=1,
        router="sigmoid", n_group=1, topk_group=1, routed_scaling=2.827,
        dense_dtype="fp8")
    base.update(kw)
    return ModelConfig(**base)


PRESETS = {
    "tiny-moe": tiny_config,
    "ds4-flash-shape": ds4_flash_config,
    "glm-5.2-shape": glm52_config,
    "kimi-k2-shape": kimi_k2_config,
}


def get_preset(name: str, **kw) -> ModelConfig:
    try:
        return PRESETS[name](**kw)
    except KeyError:
        raise ValueError(f"unknown model preset {name!r}; have {sorted(PRESETS)}") from None


def _env_bool(name: str, default: bool) -> bool:
    v = os.getenv(name)
    if v is None:
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")


def _env_float(name: str, default):
    v = os.getenv(name)
    return default if v is None or v == "" else float(v)


def _env_int(name: str, default):
    v = os.getenv(name)
    return default if v is None or v == "" else int(v)


@dataclass
class MoetConfig:
    """Runtime knobs of the 2-bit expert stack and its residency tiers.

    Field <-> reference env-name aliases are listed in ``ENV_ALIASES``; the
    reference reads them at import time (P:4113-4233, P:7903-8055,
    P:9871-10029, P:11321-11391).
    """
    prefill_t: int = 96                 # decode/prefill split (tokens)
    swiglu_clamp: bool = True
    topp: float = 0.0                   # expert top-p pruning (0 = off)
    topp_min: int = 1
    zero_mode: str = "auto"             # auto | sign | alt
    # FP4 delta tier
    delta: bool = False
    delta_gb: str = "0"                 # "N" GiB or "auto"
    delta_reserve_gb: float = 3.0       # auto: HBM left free beside the delta pool
    delta_max_gb: float = 0.0           # auto: cap of the pool (0 = none)
    delta_promote: int = 64             # background promotions per tick (the reference defaults to 8)
    delta_policy: str = "freq"          # freq | need | lru
    delta_split: bool = False
    delta_tick_ms: float = 50.0
    prefill_fp4: str = "1"              # "1": prefill serves delta-slot experts at FP4 too; "0": base only;
                                        # "ensure": each eager prefill chunk first makes its experts FP4-resident
    delta_decay: float = 0.98
    delta_rank: str = "need"            # capped gate fires: "need" (decayed rank) | "step_w" (step's routing weight)
    promo_hyst: float = 0.0             # > 1: background promotions into a full pool need freq > h x victim + 4
    # base cache (GPU as expert cache)
    base_cache_gb: float = 0.0
    base_miss_tol: int = 0
    fp_max: int = 32
    replay_mode: str = "strict"         # strict | approximate
    kpi_every: int = 500
    force_pool: bool = False
    force_resident: bool = False
    # confidence gate
    gate: bool = False
    gate_tau: float = 0.6
    gate_signal: str = "maxprob"        # maxprob | margin
    gate_agg: str = "min"               # min | q<frac>
    gate_fp_max: int = 3
    gate_max_promote: int = 64
    gate_spec_mask: bool = False        # score only the verify rows the step emits (skip rows past a rejection)
    gate_trace: bool = False            # log every fire / re-forward
    gate_audit: float = 0.0             # probability of an audit fire on a confident step (unbiased labels)
    gate_reforward: bool = True         # False: a fire promotes for later steps but does not replay this one
    gate_capture: bool = False          # measurement only: score and log, never promote or replay
    gate_hcap_dir: Optional[str] = None  # with the gate dump: hidden states of fired / audited steps
    gate_hcap_flush: int = 256
    # runtime-tunable knobs: a one-line file re-read when it changes (path or None)
    gate_tau_file: Optional[str] = None
    gate_max_promote_file: Optional[str] = None
    base_miss_tol_file: Optional[str] = None
    fp_thresh: int = 0                  # approximate replay: chase second-order misses while <= this many
    fp_thresh_file: Optional[str] = None
    # stores
    store_dir: Optional[str] = None
    base_ram_gb: Optional[str] = None
    tier_direct: bool = False
    store_threads: int = 8
    planes_cache: Optional[str] = None
    ckpt_id: Optional[str] = None
    pool_heat: bool = True              # dump the expert cache's heat at shutdown, preload it at boot
    tier_preheat: bool = True           # tiered store: refill the arena from its heat file at boot
    tier_scan: bool = True              # tiered store: one-shot sweeps bypass the arena
    # tracing and dumps
    prefill_timers_flush: int = 0       # CUDA-event spans of prefill, resolved every N spans (0 = off)
    delta_trace: int = 0                # 1: delta coverage / hit-rate line; 2: + per-layer FP4 histogram
    delta_dump: Optional[str] = None    # atomic JSON precision map (which expert sits in which tier)
    delta_capture: Optional[str] = None  # .npy of per-step routed expert ids
    gate_fire_timing: bool = False      # promote / replay milliseconds per gate iteration
    gate_dump: Optional[str] = None     # JSONL: one row per gate evaluation
    # spec guard (drafting latched off while the base pool replays) and draft-affinity prefetch
    spec_guard: float = 60.0            # replay-EMA percent that suppresses drafting (0 = off)
    spec_guard_ema: float = 0.02
    prefetch: bool = False              # prefetch the experts the next step's drafts routed to before
    # router lookahead: layer L+1's router applied in-graph to layer L's MoE input predicts
    # L+1's experts; LOOKA scores the predictions (recall counters), PILOT prefetches them
    looka: bool = False
    pilot: bool = False
    pilot_k: int = 8                    # experts predicted per row
    pilot_cap: int = 32                 # prefetches per step
    pilot_min_replay: float = 30.0      # replay-EMA percent below which the pool counts as warm
    # bf12: lossless 12-bit container for dense BF16 linears, converted after load
    bf12: bool = False
    bf12_min_numel: int = 1 << 20
    bf12_verify: bool = True
    bf12_exclude: str = ""              # comma-separated name substrings kept in BF16

    ENV_ALIASES = {
        "prefill_t": "VLLM_MOE_W2_PREFILL_T",
        "swiglu_clamp": "VLLM_MOE_W2_SWIGLU_CLAMP",
        "topp": "VLLM_MOE_W2_TOPP",
        "topp_min": "VLLM_MOE_W2_TOPP_MIN",
        "zero_mode": "VLLM_MOE_W2_ZERO_MODE",
        "delta": "VLLM_MOE_W2_DELTA",
        "delta_gb": "VLLM_MOE_W2_DELTA_GB",
        "delta_reserve_gb": "VLLM_MOE_W2_DELTA_RESERVE_GB",
        "delta_max_gb": "VLLM_MOE_W2_DELTA_MAX_GB",
        "delta_promote": "VLLM_MOE_W2_DELTA_PROMOTE",
        "delta_policy": "VLLM_MOE_W2_DELTA_POLICY",
        "delta_split": "VLLM_MOE_W2_DELTA_SPLIT",
        "delta_tick_ms": "VLLM_MOE_W2_DELTA_TICK_MS",
        "prefill_fp4": "VLLM_MOE_W2_PREFILL_FP4",
        "delta_decay": "VLLM_MOE_W2_DELTA_DECAY",
        "promo_hyst": "VLLM_MOE_W2_PROMO_HYST",
        "delta_rank": "VLLM_MOE_W2_DELTA_RANK",
        "gate_spec_mask": "VLLM_MOE_W2_GATE_SPEC_MASK",
        "gate_trace": "VLLM_MOE_W2_GATE_TRACE",
        "gate_audit": "VLLM_MOE_W2_GATE_AUDIT",
        "gate_reforward": "VLLM_MOE_W2_GATE_REFORWARD",
        "gate_capture": "VLLM_MOE_W2_GATE_CAPTURE",
        "gate_hcap_dir": "VLLM_MOE_W2_GATE_HCAP_DIR",
        "gate_hcap_flush": "VLLM_MOE_W2_GATE_HCAP_FLUSH",
        "base_cache_gb": "VLLM_MOE_W2_BASE_CACHE_GB",
        "base_miss_tol": "VLLM_MOE_W2_BASE_MISS_TOL",
        "base_miss_tol_file": "VLLM_MOE_W2_BASE_MISS_TOL_FILE",
        "fp_thresh": "VLLM_MOE_W2_FP_THRESH",
        "pool_heat": "VLLM_MOE_W2_POOL_HEAT",
        "tier_preheat": "VLLM_MOE_W2_TIER_PREHEAT",
        "tier_scan": "VLLM_MOE_W2_TIER_SCAN",
        "fp_thresh_file": "VLLM_MOE_W2_FP_THRESH_FILE",
        "gate_tau_file": "VLLM_MOE_W2_GATE_TAU_FILE",
        "gate_max_promote_file": "VLLM_MOE_W2_GATE_MAX_PROMOTE_FILE",
        "fp_max": "VLLM_MOE_W2_FP_MAX",
        "replay_mode": "VLLM_MOE_W2_REPLAY_MODE",
        "kpi_every": "VLLM_MOE_W2_KPI_EVERY",
        "force_pool": "VLLM_MOE_W2_FORCE_POOL",
        "force_resident": "VLLM_MOE_W2_FORCE_RESIDENT",
        "gate": "VLLM_MOE_W2_GATE",
        "gate_tau": "VLLM_MOE_W2_GATE_TAU",
        "gate_signal": "VLLM_MOE_W2_GATE_SIGNAL",
        "gate_agg": "VLLM_MOE_W2_GATE_AGG",
        "gate_fp_max": "VLLM_MOE_W2_GATE_FP_MAX",
        "gate_max_promote": "VLLM_MOE_W2_GATE_MAX_PROMOTE",
        "store_dir": "VLLM_MOE_W2_STORE_DIR",
        "base_ram_gb": "VLLM_MOE_W2_BASE_RAM_GB",
        "tier_direct": "VLLM_MOE_W2_TIER_DIRECT",
        "store_threads": "VLLM_MOE_W2_STORE_THREADS",
        "planes_cache": "VLLM_MOE_W2_PLANES_CACHE",
        "ckpt_id": "VLLM_MOE_W2_CKPT_ID",
        "prefill_timers_flush": "VLLM_PREFILL_TIMERS_FLUSH",
        "delta_trace": "VLLM_MOE_W2_DELTA_TRACE",
        "delta_dump": "VLLM_MOE_W2_DELTA_DUMP",
        "delta_capture": "VLLM_MOE_W2_DELTA_CAPTURE",
        "gate_fire_timing": "VLLM_MOE_W2_GATE_FIRE_TIMING",
        "gate_dump": "VLLM_MOE_W2_GATE_DUMP",
        "spec_guard": "VLLM_MOE_W2_SPEC_GUARD",
        "spec_guard_ema": "VLLM_MOE_W2_SPEC_GUARD_EMA",
        "prefetch": "VLLM_MOE_W2_PREFETCH",
        "looka": "VLLM_MOE_W2_LOOKA",
        "pilot": "VLLM_MOE_W2_PILOT",
        "pilot_k": "VLLM_MOE_W2_PILOT_K",
        "pilot_cap": "VLLM_MOE_W2_PILOT_CAP",
        "pilot_min_replay": "VLLM_MOE_W2_PILOT_MIN_REPLAY",
        "bf12": "VLLM_MOE_W2_BF12",
        "bf12_min_numel": "VLLM_MOE_W2_BF12_MIN_NUMEL",
        "bf12_verify": "VLLM_MOE_W2_BF12_VERIFY",
        "bf12_exclude": "VLLM_MOE_W2_BF12_EXCLUDE",
    }

    def __post_init__(self):
        self.validate()

    def validate(self):
        if not 1 <= int(self.pilot_k) <= 32:
            raise ValueError("pilot_k (VLLM_MOE_W2_PILOT_K) must be in [1, 32]")
        if self.zero_mode not in ("auto", "sign", "alt"):
            raise ValueError(
                f"VLLM_MOE_W2_ZERO_MODE must be one of auto|sign|alt, got {self.zero_mode!r}")
        if self.delta_policy not in ("freq", "need", "lru"):
            raise ValueError(f"delta_policy must be freq|need|lru, got {self.delta_policy!r}")
        if str(self.prefill_fp4) not in ("0", "1", "ensure", ""):
            raise ValueError(f"VLLM_MOE_W2_PREFILL_FP4 must be 0|1|ensure, got {self.prefill_fp4!r}")
        if self.delta_rank not in ("need", "step_w"):
            raise ValueError(f"VLLM_MOE_W2_DELTA_RANK must be need|step_w, got {self.delta_rank!r}")
        if self.replay_mode not in ("strict", "approximate"):
            raise ValueError(f"replay_mode must be strict|approximate, got {self.replay_mode!r}")
        if self.gate_signal not in ("maxprob", "margin"):
            raise ValueError(f"gate_signal must be maxprob|margin, got {self.gate_signal!r}")
        if not (self.gate_agg == "min" or (self.gate_agg.startswith("q")
                                           and 0 < float(self.gate_agg[1:]) <= 1)):
            raise ValueError(f"gate_agg must be 'min' or 'q<frac>', got {self.gate_agg!r}")
        if self.gate and not (self.delta or self.base_cache_gb > 0):
            raise ValueError("the confidence gate needs an FP4 delta tier or a base cache to promote into")
        if not 0.0 <= self.topp < 1.0:
            raise ValueError("topp must be in [0, 1)")
        if self.fp_max < 1 or self.gate_fp_max < 1:
            raise ValueError("fixed-point budgets must be >= 1")

    @classmethod
    def from_env(cls, **overrides) -> "MoetConfig":
        kw = {}
        for f in dataclasses.fields(cls):
            env = cls.ENV_ALIASES.get(f.name)
            if env is None or os.getenv(env) is None:
                continue
            default = f.default
            if isinstance(default, bool):
                kw[f.name] = _env_bool(env, default)
            elif isinstance(default, int):
                kw[f.name] = _env_int(env, default)
            elif isinstance(default, float):
                kw[f.name] = _env_float(env, default)
            else:
                kw[f.name] = os.getenv(env)
        kw.update(overrides)
        return cls(**kw)


@dataclass
class ParallelConfig:
    tp: int = 1
    pp: int = 1
    dp: int = 1
    ep: bool = False
    dcp: int = 1
    sp_prefill: bool = False
    fused_comm: bool = True     # fused peer-memory kernels (False = NCCL baseline)

    def __post_init__(self):
        for n in ("tp", "pp", "dp", "dcp"):
            v = getattr(self, n)
            if v < 1 or (v & (v - 1)):
                raise ValueError(f"{n} must be a power of two >= 1, got {v}")

    @property
    def world_size(self) -> int:
        return self.tp * self.pp * self.dp


@dataclass
class EngineConfig:
    model: ModelConfig
    moet: MoetConfig = field(default_factory=MoetConfig)
    parallel: ParallelConfig = field(default_factory=ParallelConfig)
    max_num_seqs: int = 32
    max_model_len: int = 16384
    kv_block_size: int = 64
    kv_cache_dtype: str = "bf16"      # bf16 | nvfp4
    num_speculative_tokens: int = 2   # MTP k
    cuda_graphs: bool = True
    max_prefill_chunk: int = 8192
    seed: int = 0
    device: str = "cuda"

    def __post_init__(self):
        if self.kv_cache_dtype not in ("bf16", "nvfp4"):
            raise ValueError(f"kv_cache_dtype must be bf16|nvfp4, got {self.kv_cache_dtype!r}")
        if self.kv_cache_dtype == "nvfp4" and (self.model.kv_lora_rank != 512 or self.model.qk_rope_dim != 64):
            raise ValueError("nvfp4 MLA KV needs kv_lora_rank 512 and rope 64 (352 B/token layout)")
        if self.num_speculative_tokens < 0 or self.num_speculative_tokens > 7:
            raise ValueError("num_speculative_tokens must be in [0, 7]")
        if self.num_speculative_tokens and self.model.num_mtp_layers < 1:
            raise ValueError("MTP speculation needs a model with an MTP layer")
