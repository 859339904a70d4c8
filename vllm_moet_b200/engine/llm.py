"""User-facing engine: ``LLM(model=...).generate(prompts, SamplingParams)``.

One engine object owns the model weights, the paged KV cache, the decode
state of a batch bucket and (on a GPU) the captured decode graph of that
bucket.  The loop is: admit waiting requests into free rows (reserve KV
blocks, batched prefill that also primes the MTP drafts), then replay the
decode step until some row finishes, refilling freed rows as it goes.  Per
step the host sends the row-activity vector (pinned H2D) and reads back the
emitted tokens and acceptance counts (pinned D2H).
"""
from __future__ import annotations

import contextlib
import itertools
import os
import time
from collections import deque
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Union

import torch

from ..config import EngineConfig, ModelConfig, MoetConfig, ParallelConfig, get_preset
from ..models.weights import ModelWeights, random_weights
from .kv_manager import BlockManager
from .sampling_params import CompletionOutput, RequestOutput, SamplingParams, cut_at_stop
from .tokenizer import ByteTokenizer, tokenizer_for


@dataclass
class _Req:
    rid: str
    prompt: List[int]
    params: SamplingParams
    out: List[int] = field(default_factory=list)
    row: int = -1
    finish: Optional[str] = None
    t_arrive: float = 0.0
    t_first: float = 0.0
    t_done: float = 0.0
    callback: Optional[object] = None     # callback(new_token_ids, finish_reason) for streaming
    text: Optional[str] = None            # final text when a stop string cut it
    logprobs: Optional[list] = None       # per emitted token {token: logprob} (when requested)
    prompt_logprobs: Optional[list] = None
    stop_reason: Optional[object] = None
    emits: int = 0                        # emit calls: the prefill's first token, then one per decode step


class LLM:
    def __init__(self, model: Union[str, ModelConfig] = "tiny-moe", *, device: Optional[str] = None,
                 num_speculative_tokens: int = 2, max_model_len: int = 4096, max_num_seqs: int = 8,
                 kv_cache_dtype: str = "bf16", seed: int = 0, weights: Optional[ModelWeights] = None,
                 num_layers: Optional[int] = None, cuda_graphs: bool = True, num_gpu_blocks: Optional[int] = None,
                 tensor_parallel_size: int = 1, tp_group=None, tp_rank: int = 0,
                 pipeline_parallel_size: int = 1, pp_group=None, pp_rank: int = 0, expert_cache_slots: int = 0,
                 delta_slots: int = 0, gate: Optional[bool] = None, expert_parallel: bool = False,
                 expert_store: str = "pinned", expert_store_dir: Optional[str] = None, sp_group=None,
                 dcp_group=None, dcp_interleave: int = 1, ep_group=None, speculative_method: str = "mtp",
                 dspark: Optional[dict] = None, enable_prefix_caching: bool = False,
                 prefix_block_size: int = 16, enable_chunked_prefill: bool = False,
                 max_num_batched_tokens: Optional[int] = None, tp_attention: Optional[str] = None,
                 trellis_pack: Optional[str] = None, **model_overrides):
        from ..models.loader import hf_config, is_checkpoint_dir, load_weights
        ckpt = model if is_checkpoint_dir(model) else None
        if ckpt is not None:
            cfg = hf_config(ckpt, **model_overrides)
        else:
            cfg = get_preset(model, **model_overrides) if isinstance(model, str) else model
        if (sp_group is not None or dcp_group is not None) and (tp_group is not None or pp_group is not None):
            raise ValueError("context parallelism here runs on replicated weights (no TP / PP group)")
        if sum(g is not None for g in (sp_group, dcp_group, ep_group)) > 1:
            raise ValueError("choose one of sp_group (SP prefill), dcp_group (DCP decode), ep_group (DP + EP)")
        if ep_group is not None and (tp_group is not None or pp_group is not None):
            raise ValueError("ep_group: data-parallel attention with expert-parallel MoE (no TP / PP group)")
        self._mtp_requested = num_speculative_tokens > 0
        if num_layers is not None:
            cfg = cfg.replace(num_layers=num_layers)
        if device is None:
            device = "cuda" if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        self._tp_group, self._pp_group = tp_group, pp_group
        # ranks that must draw the same sampling seeds (they emit the same tokens)
        self._seed_group = tp_group if tp_group is not None else dcp_group
        if self.device.type == "cuda" and dcp_group is not None and cfg.index_heads:
            raise NotImplementedError("GPU DCP decode: dense MLA attention (DSA models run DCP on the CPU engine)")
        self._dcp = None
        if self.device.type == "cuda" and sp_group is not None and (enable_prefix_caching or enable_chunked_prefill):
            raise NotImplementedError("GPU SP prefill: no prefix caching or chunked prefill")
        self._sp_group = sp_group
        self._ep_group = ep_group
        if speculative_method not in ("mtp", "dspark", "dflash", "eagle3"):
            raise ValueError(f"speculative_method {speculative_method!r}: mtp | dspark | dflash | eagle3")
        if speculative_method == "eagle3" and pipeline_parallel_size > 1:
            raise NotImplementedError("EAGLE-3 drafting runs on one pipeline stage")
        if speculative_method == "eagle3" and self.device.type == "cuda" and (
                tensor_parallel_size > 1 or tp_group is not None or ep_group is not None or sp_group is not None
                or dcp_group is not None or cfg.hc_mult > 1):
            raise NotImplementedError("GPU EAGLE-3 drafting: one GPU per replica (no TP / EP / SP / DCP), "
                                      "single-stream models")
        if speculative_method == "dflash":
            # DFlash: the same parallel context drafter without the Markov and confidence
            # heads; every block is verified whole
            dspark = dict(dspark or {}, model="context", markov=False, tau=0.0, budget_frac=1.0)
            speculative_method = "dspark"
        if speculative_method == "dspark" and self.device.type == "cuda":
            raise NotImplementedError("DSpark / DFlash block drafting runs on the CPU engine; the GPU runner drafts with MTP")
        if cfg.hc_mult > 1 and self.device.type == "cuda" and pipeline_parallel_size > 1:
            raise NotImplementedError("hyper-connections on the GPU: no pipeline stages (the stage boundary "
                                      "carries one residual stream)")
        simple_dspark = speculative_method == "dspark" and ((dspark or {}).get("model", "context") != "context"
                                                            or (dspark or {}).get("drafter") is not None)
        if cfg.hc_mult > 1 and (sp_group is not None or simple_dspark):
            raise NotImplementedError("hyper-connections: not with SP prefill or a context-free DSpark drafter "
                                      "(both read a single-stream hidden state)")
        self._chunk_budget = None
        if enable_chunked_prefill:
            if sp_group is not None or dcp_group is not None or ep_group is not None:
                raise ValueError("chunked prefill: not with SP prefill, DCP decode or DP + EP")
            self._chunk_budget = int(max_num_batched_tokens or 2048)
            if self._chunk_budget < 1:
                raise ValueError("max_num_batched_tokens must be >= 1")
        if (self._chunk_budget is None and self.device.type == "cuda" and cfg.index_heads and ep_group is None
                and sp_group is None and dcp_group is None):
            # DSA models on the GPU: prompts run in chunks of index_topk tokens.  The first chunk
            # sees at most index_topk keys per query (dense == sparse); every later chunk runs the
            # absorbed attention over the paged cache with the indexer's top-k selection per row,
            # so a long prompt is prefilled with sparse attention and never builds a T x T score
            self._chunk_budget = int(max_num_batched_tokens or cfg.index_topk)
        if enable_prefix_caching and (sp_group is not None or dcp_group is not None):
            raise ValueError("prefix caching keeps whole per-sequence caches: not with SP prefill / DCP decode")
        if self.device.type == "cuda" and cfg.expert_scale != "ue8m0":
            cfg = cfg.replace(expert_scale="ue8m0")
        if self.device.type == "cuda" and cfg.dense_dtype != "fp8":
            cfg = cfg.replace(dense_dtype="fp8")
        self.cfg = cfg
        self.ecfg = EngineConfig(model=cfg, moet=MoetConfig.from_env(),
                                 parallel=ParallelConfig(tp=tensor_parallel_size, pp=pipeline_parallel_size),
                                 max_num_seqs=max_num_seqs, max_model_len=max_model_len,
                                 kv_cache_dtype=kv_cache_dtype, num_speculative_tokens=num_speculative_tokens,
                                 cuda_graphs=cuda_graphs, seed=seed, device=str(self.device))
        self.tokenizer = tokenizer_for(cfg.vocab, ckpt)
        if self.device.type == "cuda" and weights is None and not expert_cache_slots \
                and self.ecfg.moet.base_cache_gb <= 0 and not self.ecfg.moet.force_resident:
            self._resident_hardstop(cfg, tensor_parallel_size, expert_parallel, num_layers)
        self.expert_source = None
        if weights is None and self.ecfg.moet.planes_cache:
            # boot the expert planes from the persistent quantisation cache (first boot fills it)
            from ..residency import PlanesCache, checkpoint_id
            from ..residency.sources import PlanesSource
            self.expert_source = PlanesSource(PlanesCache(
                self.ecfg.moet.planes_cache,
                self.ecfg.moet.ckpt_id or (checkpoint_id(model_path=ckpt) if ckpt else checkpoint_id(cfg=cfg, seed=seed)),
                tp_world=tensor_parallel_size, tp_rank=tp_rank))
        if weights is None and ckpt is not None:
            weights = load_weights(ckpt, cfg, self.device, tp_rank=tp_rank, tp_size=tensor_parallel_size,
                                   with_mtp=num_speculative_tokens > 0, pp_rank=pp_rank,
                                   pp_size=pipeline_parallel_size, expert_parallel=expert_parallel,
                                   expert_source=self.expert_source)
        # TP attention: "shard" (heads split, o_proj reduced) or "replicate" (whole attention on
        # every rank, no o_proj reduction: half the decode reductions for ~42 MB / layer of FP8
        # weights read per rank; DS4 TP2 measured 184.6 against 174.9 tok/s).  Default replicate
        # for random-init models without EP; MOET_TP_ATTN overrides
        tp_attention = tp_attention or os.environ.get(
            "MOET_TP_ATTN", "replicate" if (weights is None and ckpt is None and not expert_parallel) else "shard")
        if tp_attention not in ("shard", "replicate"):
            raise ValueError("tp_attention: shard | replicate")
        if tp_attention == "replicate" and tensor_parallel_size > 1 and (ckpt is not None or weights is not None
                                                                         or expert_parallel):
            raise NotImplementedError("replicated TP attention: random-init weights with sharded experts")
        self.mw = weights if weights is not None else random_weights(
            cfg, self.device, seed=seed, tp_rank=tp_rank, tp_size=tensor_parallel_size,
            with_mtp=num_speculative_tokens > 0, pp_rank=pp_rank, pp_size=pipeline_parallel_size,
            with_delta=(("split" if self.ecfg.moet.delta_split else True) if delta_slots and self.device.type == "cuda"
                        else False), expert_parallel=expert_parallel,
            expert_source=self.expert_source, attn_tp=tp_attention == "shard")
        if self.expert_source is not None:
            self.expert_source.flush()
        self.bf12_stats = None
        if self.ecfg.moet.bf12:
            # lossless 12-bit re-pack of the dense BF16 linears, before any capture (the GPU
            # runner's dense linears are FP8, so there it finds nothing to convert)
            from ..formats.bf12 import convert_model
            m = self.ecfg.moet
            self.bf12_stats = convert_model(self.mw, m.bf12_min_numel,
                                            tuple(x for x in m.bf12_exclude.split(",") if x), m.bf12_verify)
        if speculative_method == "eagle3" and num_speculative_tokens > 0:
            from ..models.eagle3_model import attach_eagle3, random_eagle3_weights
            attach_eagle3(self.mw, random_eagle3_weights(self.mw, seed=seed))
            self.mw.mtp = None                     # the EAGLE-3 module drafts instead of the MTP module
        if speculative_method == "eagle3":
            self._has_mtp = num_speculative_tokens > 0
        elif pipeline_parallel_size > 1:
            # MTP presence is a property of the model, known on every stage
            self._has_mtp = num_speculative_tokens > 0 and cfg.num_mtp_layers > 0
        else:
            self._has_mtp = self.mw.mtp is not None
        self.k = num_speculative_tokens if self._has_mtp else 0
        self.max_blocks = -(-(max_model_len + self.k + 2) // 64)
        self.stats = {}
        self._ids = itertools.count()
        if self.device.type == "cuda":
            from .gpu_runner import DecodeState, NativeRunner
            nb = num_gpu_blocks or (max_num_seqs * self.max_blocks + 1)
            self.blocks = BlockManager(nb, prefix_caching=enable_prefix_caching)
            if ep_group is not None:
                import torch.distributed as dist
                from ..parallel.ep import ep_partition
                if expert_cache_slots or delta_slots or enable_prefix_caching or enable_chunked_prefill:
                    raise NotImplementedError("GPU DP + EP: no expert cache, delta tier, prefix caching or "
                                              "chunked prefill")
                ep_partition(self.mw, dist.get_rank(ep_group), dist.get_world_size(ep_group))
            self.runner = NativeRunner(self.mw, self.ecfg, nb, self.device)
            if sp_group is not None:
                self.runner.set_sp_group(sp_group)
            if dcp_group is not None:
                import torch.distributed as dist
                self.runner.set_dcp_group(dcp_group, dcp_interleave)
                self._dcp = (dist.get_world_size(dcp_group), dist.get_rank(dcp_group), int(dcp_interleave))
            if ep_group is not None:
                # the most routed rows of one decode-sized layer on one rank: verify rows x top-k
                self.runner.set_ep_group(ep_group, self._bucket(max_num_seqs) * (self.k + 1) * cfg.top_k)
                self._ep_dummy = None
            if tp_group is not None:
                self.runner.set_tp_group(tp_group)
            if pp_group is not None:
                self.runner.set_pp_group(pp_group)
                self.ecfg.cuda_graphs = False      # pipeline stages run eager steps (p2p per step)
            self.cache = self.replay = None
            self.spec_guard = self.affinity = self.pilot = None
            self._spec_draft = True
            slots = expert_cache_slots
            if not slots and self.ecfg.moet.base_cache_gb > 0:
                from ..residency import moe_layers
                sb = moe_layers(self.mw)[0].experts.layout.slot_bytes
                slots = int(self.ecfg.moet.base_cache_gb * (1 << 30) // sb)
            if slots:
                self._attach_cache(slots, expert_store, expert_store_dir, tp_group)
            self.delta = self.gate = None
            m = self.ecfg.moet
            if not delta_slots and m.delta and str(m.delta_gb) not in ("0", ""):
                # VLLM_MOE_W2_DELTA=1 with a size in GiB or auto (free HBM after load - reserve)
                from ..residency import moe_layers
                from ..residency.delta import delta_layout, delta_slots_for
                lay = moe_layers(self.mw)[0].experts.layout
                free = torch.cuda.mem_get_info(self.device)[0]
                delta_slots = delta_slots_for(m.delta_gb, delta_layout(lay.H, lay.I)[0], free,
                                              m.delta_reserve_gb, m.delta_max_gb)
            if delta_slots:
                self._attach_delta(delta_slots, gate)
            trellis_pack = trellis_pack or os.environ.get("VLLM_MOE_W2_EXL3_PACK") or None
            self.trellis = None
            if trellis_pack:
                if slots or delta_slots:
                    raise NotImplementedError("trellis base tier: not with an expert cache or an FP4 delta tier")
                self.trellis = self._attach_trellis(trellis_pack, tp_group, pp_group, sp_group, dcp_group, ep_group)
            self._attach_tracing()
            self._DecodeState = DecodeState
            self._states = {}
            self._pin_active = None
        else:
            from .torch_runner import TorchRunner
            self.blocks = None
            if ep_group is not None:
                import torch.distributed as dist
                from ..parallel.ep import ep_partition
                ep_partition(self.mw, dist.get_rank(ep_group), dist.get_world_size(ep_group))
            self.runner = TorchRunner(self.mw, self.k, max_model_len, self.device, tp_group=tp_group,
                                      sp_group=sp_group, dcp_group=dcp_group, dcp_interleave=dcp_interleave,
                                      ep_group=ep_group,
                                      dspark=(dspark or {}) if speculative_method == "dspark" else None,
                                      prefix_block=prefix_block_size if enable_prefix_caching else 0)
            trellis_pack = trellis_pack or os.environ.get("VLLM_MOE_W2_EXL3_PACK") or None
            self.trellis = None
            if trellis_pack:
                self.trellis = self._attach_trellis(trellis_pack, tp_group, pp_group, sp_group, dcp_group, ep_group)

    def _attach_trellis(self, pack_dir, *groups):
        """Serve the routed experts of every MoE layer that has a pack in ``pack_dir`` from
        the trellis base tier (single rank, unsharded experts): on the CPU engine through
        the oracle's MoE hook, on the GPU inside the runner's MoE step."""
        from ..residency.trellis_tier import TrellisBaseTier, pack_path
        if any(g is not None for g in groups):
            raise NotImplementedError("trellis base tier: one rank with every expert (no TP / PP / SP / DCP / EP)")
        layers = [li for li, lw in enumerate(self.mw.layers) if lw.is_moe and os.path.exists(pack_path(pack_dir, li))]
        if not layers:
            raise FileNotFoundError(f"no trellis packs (exl3-lNN.safetensors) for the MoE layers in {pack_dir}")
        tier = TrellisBaseTier(pack_dir, layers, device=self.device, act_limit=self.mw.cfg.swiglu_limit)
        if self.device.type == "cuda":
            self.runner.attach_trellis(tier)       # inside the GPU runner's MoE step (capturable)
        else:
            self.runner.moe_impl = tier.moe_fn(self.mw)
        return tier

    def _kpi_gauges(self, runner):
        """The KPI line's latest-value fields (cheap host reads; the LOOKA recall reads two
        small device counters, so only on the steps the line is printed)."""
        c = self.cache
        g = dict(pool_slots=c.n_slots, pool_pct=100.0 * c.n_slots / max(1, c.L * c.E))
        if self.spec_guard is not None:
            g["replay_ema"] = 100.0 * float(self.spec_guard.ema)
        if getattr(runner, "_looka", None) is not None and (self.kpi.steps + 1) % self.kpi.every == 0:
            g["looka"] = runner.looka_recall()
        self.kpi.gauge(**g)

    def _attach_tracing(self):
        """Prefill span timers, routing capture, delta trace / dump and the gate JSONL
        (reference env names: VLLM_PREFILL_TIMERS_FLUSH, VLLM_MOE_W2_DELTA_TRACE / _DUMP /
        _CAPTURE, VLLM_MOE_W2_GATE_FIRE_TIMING / _DUMP)."""
        from ..utils import observability as obs
        m = self.ecfg.moet
        self.timers = obs.SpanTimers(flush_every=m.prefill_timers_flush) if m.prefill_timers_flush > 0 else None
        self.runner.timers = self.timers
        self.routing = obs.RoutingCapture() if m.delta_capture else None
        self.delta_trace = (obs.DeltaTrace(level=m.delta_trace, every=m.kpi_every)
                            if m.delta_trace and self.delta is not None else None)
        self.gate_log = obs.JsonlWriter(m.gate_dump) if m.gate_dump and self.gate is not None else None
        self.hcap = (obs.HiddenCapture(m.gate_hcap_dir, m.gate_hcap_flush)
                     if self.gate_log is not None and m.gate_hcap_dir else None)
        self._decode_steps = 0

    def dump_traces(self):
        """Write the configured dumps now (also done by shutdown)."""
        from ..residency.fsutil import atomic_write_json
        from ..utils import observability as obs
        m = self.ecfg.moet
        if m.delta_dump:
            d = {"base": obs.precision_map(self.cache) if getattr(self, "cache", None) is not None else None,
                 "delta": obs.precision_map(self.delta, "fp4-split" if getattr(self.delta, "split", False)
                                            else "fp4-direct8") if getattr(self, "delta", None) is not None else None}
            if getattr(self, "delta_trace", None) is not None:
                d["trace"] = self.delta_trace.snapshot(self.delta)
            atomic_write_json(m.delta_dump, d)
        if getattr(self, "routing", None) is not None:
            self.routing.save(m.delta_capture)
        if getattr(self, "timers", None) is not None:
            obs.log.info("[moet] prefill timers: %s", self.timers.summary())

    def _resident_hardstop(self, cfg, tp, ep, num_layers):
        """Refuse early when fully resident experts cannot fit beside a KV floor and
        suggest a base-cache size instead (VLLM_MOE_W2_FORCE_RESIDENT=1 overrides)."""
        from ..models.weights import ExpertLayout
        from ..residency import resident_fit
        L = (num_layers or cfg.num_layers) + (1 if self._mtp_requested else 0)
        moe_layers = max(0, L - cfg.num_dense_layers)
        I = cfg.moe_intermediate if ep else cfg.moe_intermediate // tp
        E = cfg.num_experts // tp if ep else cfg.num_experts
        need = moe_layers * E * ExpertLayout(H=cfg.hidden, I=I).slot_bytes
        free, _ = torch.cuda.mem_get_info(self.device)
        kv_floor = self.ecfg.max_model_len * self.ecfg.max_num_seqs * 1168 * (L + 1)
        fits, gb = resident_fit(need, free, kv_floor)
        if not fits:
            raise MemoryError(f"routed experts need {need / 2**30:.1f} GiB resident but only {gb:.1f} GiB fit beside "
                              f"the KV floor; set VLLM_MOE_W2_BASE_CACHE_GB (e.g. {max(1.0, 0.9 * gb):.0f}) to serve "
                              "them through the expert cache, or VLLM_MOE_W2_FORCE_RESIDENT=1")

    def reload_weights(self, *a, **k):
        """Weight updates are refused on the 2-bit expert path: the expert planes,
        their caches and the captured graphs derive from the loaded weights."""
        raise NotImplementedError("reload_weights is not supported with 2-bit experts; build a new LLM")

    def shutdown(self):
        """Write the configured dumps, stop the residency managers (tiers first), then
        release stores and peer buffers."""
        if hasattr(self, "_decode_steps"):
            self.dump_traces()
        kpi = getattr(self, "kpi", None)
        if kpi is not None and kpi.steps % kpi.every:      # the last partial window's KPI line
            kpi.flush()
        self._dump_heat()
        if getattr(self, "gate_log", None) is not None:
            self.gate_log.close()
            self.gate_log = None
        if getattr(self, "hcap", None) is not None:
            self.hcap.close()
            self.hcap = None
        for tier in (getattr(self, "delta", None), getattr(self, "cache", None)):
            if tier is not None:
                tier.close()
                tier.store.release()
        ar = getattr(getattr(self, "runner", None), "ar", None)
        if ar is not None:
            ar.close()

    def _attach_delta(self, slots, gate):
        """FP4 delta tier of `slots` hot experts (+ the confidence gate that fills it)."""
        from ..residency import ConfidenceGate, moe_layers
        from ..residency.delta import DeltaTier
        m = self.ecfg.moet
        layers = moe_layers(self.mw)
        rows = [lw.experts.delta_rows for lw in layers]
        if any(r is None for r in rows):
            raise ValueError("delta tier needs weights built with delta rows")
        lay = layers[0].experts.layout
        self.delta = DeltaTier(rows, lay.H, lay.I, slots, device=self.device, policy=m.delta_policy,
                               decay=m.delta_decay, split=m.delta_split, promo_hyst=m.promo_hyst)
        if getattr(self, "cache", None) is not None:
            self.delta.couple(self.cache)
        for lw in layers:
            lw.experts.delta_rows = None
        self.runner.attach_delta_tier(self.delta)
        if gate if gate is not None else m.gate:
            self.gate = ConfidenceGate(tau=m.gate_tau, signal=m.gate_signal, agg=m.gate_agg, fp_max=m.gate_fp_max,
                                       max_promote=m.gate_max_promote, tau_file=m.gate_tau_file,
                                       max_promote_file=m.gate_max_promote_file)
            self.ecfg.cuda_graphs = self.ecfg.cuda_graphs  # gate replays reuse the captured graph

    def _routed_pairs(self, B):
        ids = self.runner.route_ids(B)
        pairs = []
        for li, t in enumerate(ids):
            if t is not None:
                pairs += [(li, int(e)) for e in torch.unique(t).tolist()]
        return pairs

    def _step_weights(self, B) -> dict:
        """(layer, expert) -> the largest routing weight it got in the last decode step."""
        out = {}
        ws_fn = getattr(self.runner, "route_weights", None)
        if ws_fn is None:
            return out
        for li, (ids, w) in enumerate(zip(self.runner.route_ids(B), ws_fn(B))):
            if ids is None or w is None:
                continue
            for e, x in zip(ids.reshape(-1).tolist(), w.reshape(-1).tolist()):
                k = (li, int(e))
                if x > out.get(k, -1.0):
                    out[k] = float(x)
        return out

    def _routed_token_counts(self, B):
        """{(layer, expert): rows routed to it} of the last decode step."""
        out = {}
        for li, t in enumerate(self.runner.route_ids(B)):
            if t is not None:
                e, n = torch.unique(t, return_counts=True)
                out.update({(li, int(a)): int(b) for a, b in zip(e.tolist(), n.tolist())})
        return out

    def _attach_cache(self, slots, kind, store_dir, tp_group):
        """Routed experts from a host store through a GPU expert cache of `slots` slots,
        with in-graph miss counting and fixed-point replay of missed decode steps; the spec
        guard (VLLM_MOE_W2_SPEC_GUARD, replay-EMA percent) and draft-affinity prefetch
        (VLLM_MOE_W2_PREFETCH=1) ride on the same loop."""
        from ..residency import ReplayEngine, build_expert_cache, checkpoint_id, rank_suffix
        m = self.ecfg.moet
        kw = {}
        if kind in ("pack", "tiered"):
            kw = dict(dir=store_dir or m.store_dir, ckpt_id=m.ckpt_id or checkpoint_id(cfg=self.cfg, seed=self.ecfg.seed),
                      suffix=rank_suffix(self.mw.tp_rank, self.mw.tp_size), direct=m.tier_direct,
                      threads=m.store_threads, scan=m.tier_scan)
            if kw["dir"] is None:
                raise ValueError("pack / tiered expert stores need a store directory (VLLM_MOE_W2_STORE_DIR)")
        from ..utils.observability import KpiLogger
        self.kpi = KpiLogger(every=m.kpi_every)
        from ..residency.control import DraftAffinity, SpecGuard
        self.spec_guard = (SpecGuard(alpha=m.spec_guard_ema, hi=m.spec_guard / 100.0, lo=m.spec_guard / 200.0)
                           if m.spec_guard > 0 and self.k > 0 and self._pp_group is None else None)
        from ..residency import moe_layers, working_set_floor
        floor = working_set_floor(len(moe_layers(self.mw)), self.cfg.top_k, self.k, self.ecfg.max_num_seqs,
                                  self.cfg.num_experts)
        if slots < floor and not m.force_pool:
            raise ValueError(f"expert cache of {slots} slots is below the working-set floor {floor} "
                             "(one decode step's routed experts); raise it or set VLLM_MOE_W2_FORCE_POOL=1")
        self.cache = build_expert_cache(self.mw, slots, kind, self.device, **kw)
        self.runner.attach_expert_cache(self.cache)
        self._warm_start(m)
        self.replay = ReplayEngine(self.cache, tp_group=tp_group, pp_group=self._pp_group, mode=m.replay_mode,
                                   fp_max=m.fp_max,
                                   miss_tol=m.base_miss_tol, miss_tol_file=m.base_miss_tol_file,
                                   fp_thresh=m.fp_thresh, fp_thresh_file=m.fp_thresh_file)
        self.affinity = DraftAffinity(self.cache) if m.prefetch and self.k > 0 else None
        self.pilot = None
        if m.looka or m.pilot:
            # router lookahead in the decode graph; PILOT prefetches its predictions
            from ..residency import Pilot
            self.runner.enable_looka(m.pilot_k, m.pilot, self._bucket(self.ecfg.max_num_seqs) * (self.k + 1))
            if m.pilot:
                self.pilot = Pilot(self.cache, self.runner.pilot_log, m.pilot_cap, m.pilot_min_replay)

    def _heat_path(self):
        """Where the expert cache's heat lives: beside the pack (pack / tiered stores) or in
        the store directory; None without either."""
        st = self.cache.store
        if getattr(st, "pack_path", None):
            return st.pack_path[:-5] + ".pool.heat.json"
        d = self.ecfg.moet.store_dir
        if d:
            from ..residency import rank_suffix
            return os.path.join(d, f"pool.{rank_suffix(self.mw.tp_rank, self.mw.tp_size)}.heat.json")
        return None

    def _warm_start(self, m):
        """Warm state at boot (reference: pool heat P:8636-8738, tiered preheat P:13468-13517):
        the tiered arena refills from its heat file, the expert cache preloads the experts
        its last run ranked hottest.  Without a heat file the pool starts cold."""
        st = self.cache.store
        if m.tier_preheat and hasattr(st, "preheat"):
            self.stats_warm = {"arena_rows": st.preheat()}
        path = self._heat_path() if m.pool_heat else None
        if path and os.path.exists(path):
            n = self.cache.preload(path)
            self.stats_warm = dict(getattr(self, "stats_warm", {}), pool_experts=n)

    def _dump_heat(self):
        m = self.ecfg.moet
        if getattr(self, "cache", None) is None:
            return
        st = self.cache.store
        if m.tier_preheat and hasattr(st, "dump_heat"):
            st.dump_heat()
        path = self._heat_path() if m.pool_heat else None
        if path:
            self.cache.dump_heat(path)

    # ------------------------------------------------------------------ API
    def _normalize(self, prompts) -> List[List[int]]:
        if isinstance(prompts, (str, dict)) or (prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        out = []
        for p in prompts:
            if isinstance(p, str):
                out.append([self.tokenizer.bos_token_id] + self.tokenizer.encode(p))
            elif isinstance(p, dict):
                out.append(list(p["prompt_token_ids"]))
            else:
                out.append([int(t) for t in p])
        for p in out:
            if not p:
                raise ValueError("empty prompt")
            if any(t < 0 or t >= self.cfg.vocab for t in p):
                raise ValueError("prompt token id out of range")
        return out

    def _generate_n(self, toks, params, callbacks):
        """n completions per prompt: each prompt is expanded into n requests (copy i samples
        with seed + i when the request is seeded) and regrouped into one RequestOutput."""
        import dataclasses
        flat_t, flat_p, owner = [], [], []
        for i, (t, sp) in enumerate(zip(toks, params)):
            for j in range(sp.n):
                seed = None if sp.seed is None else sp.seed + j
                flat_t.append(t)
                flat_p.append(dataclasses.replace(sp, n=1, seed=seed))
                owner.append(i)
        cbs = None
        if callbacks is not None:
            cbs = [callbacks[i] for i in owner]
        outs = self.generate(flat_t, flat_p, callbacks=cbs)
        grouped = []
        for i, t in enumerate(toks):
            mine = [o for o, w in zip(outs, owner) if w == i]
            comps = [dataclasses.replace(o.outputs[0], index=j) for j, o in enumerate(mine)]
            grouped.append(RequestOutput(mine[0].request_id, t, comps, metrics=mine[0].metrics,
                                         prompt_logprobs=mine[0].prompt_logprobs))
        return grouped

    def chat(self, messages, sampling_params: Optional[SamplingParams] = None, reasoning_effort: str = "none",
             tools=None) -> List[RequestOutput]:
        """One conversation (list of {"role", "content"} messages) or a list of them, rendered
        with the DeepSeek-V4 chat encoding (a checkpoint tokenizer's own chat template
        when it has one)."""
        from ..entrypoints import chat_encoding
        convs = [messages] if messages and isinstance(messages[0], dict) else list(messages)
        prompts = []
        for m in convs:
            if hasattr(self.tokenizer, "tok") and getattr(self.tokenizer.tok, "chat_template", None):
                prompts.append(self.tokenizer.apply_chat_template(m))
            else:
                text = chat_encoding.render(m, tools=tools, reasoning_effort=reasoning_effort)
                prompts.append([self.tokenizer.bos_token_id] + self.tokenizer.encode(text))
        return self.generate(prompts, sampling_params)

    def _check_request(self, t, sp):
        if sp.bad_words and sp.bad_word_ids is None:     # vLLM: the word and its leading-space form
            ids = []
            for w in sp.bad_words:
                for form in (w, " " + w.lstrip()):
                    seq = list(self.tokenizer.encode(form))
                    if seq and seq not in ids:
                        ids.append(seq)
            sp.bad_word_ids = ids
        if sp.bad_word_ids and self.device.type == "cuda" and any(len(w) > 1 for w in sp.bad_word_ids):
            raise NotImplementedError("bad_words of several tokens: CPU engine (the GPU bans one-token words)")
        if sp.prompt_logprobs is not None and self.device.type == "cuda":
            raise NotImplementedError("prompt_logprobs: the GPU prefill keeps only each prompt's last logits")
        if sp.processes_logits or sp.min_p > 0:
            if getattr(self.runner, "sp_group", None) is not None or getattr(self.runner, "dspark", None):
                raise NotImplementedError("penalties / logit_bias / min_p: not with SP prefill or DSpark drafting")
        if len(t) + sp.max_tokens + self.k + 1 > self.ecfg.max_model_len:
            raise ValueError(f"prompt ({len(t)}) + max_tokens ({sp.max_tokens}) exceeds max_model_len")

    def get_tokenizer(self):
        """The engine's tokenizer (vLLM's ``LLM.get_tokenizer``)."""
        return self.tokenizer

    def beam_search(self, prompts, params):
        """Beam search (vLLM's ``LLM.beam_search``): ``params`` is a
        ``BeamSearchParams``; returns one ``BeamSearchOutput`` per prompt with up to
        ``beam_width`` sequences, best first.  Built on ``generate`` (one batched call per
        step over every live beam), so it runs on either engine."""
        from .beam_search import beam_search
        return beam_search(self, self._normalize(prompts), params)

    def generate(self, prompts, sampling_params: Union[SamplingParams, Sequence[SamplingParams], None] = None,
                 use_tqdm: bool = False, callbacks: Optional[Sequence] = None, request_ids: Optional[Sequence] = None,
                 between_steps=None) -> List[RequestOutput]:
        """Generation for a batch of prompts (str, token-id lists or
        {"prompt_token_ids": [...]}).  `callbacks[i](new_ids, finish_reason)` is
        called as tokens of prompt i are emitted (streaming).

        `between_steps(n_free) -> (new, abort_ids)` (serving): called before every
        step; `new` = [(request_id, prompt_ids, params, callback)] requests that join
        the running batch (at most n_free: the batch size of the running CUDA-graph
        bucket), `abort_ids` = request ids to finish now with reason "abort".  Joined
        requests report through their callbacks only."""
        toks = self._normalize(prompts)
        if sampling_params is None:
            sampling_params = SamplingParams()
        if isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * len(toks)
        if any(sp.n > 1 for sp in sampling_params):
            return self._generate_n(toks, sampling_params, callbacks)
        reqs = []
        for i, (t, sp) in enumerate(zip(toks, sampling_params)):
            self._check_request(t, sp)
            rid = request_ids[i] if request_ids is not None else f"req-{next(self._ids)}"
            reqs.append(_Req(rid, t, sp, t_arrive=time.perf_counter(),
                             callback=callbacks[len(reqs)] if callbacks is not None else None))
        self._between = between_steps
        try:
            if self.device.type == "cuda" and self._ep_group is not None:
                self._run_native_ep(reqs)
            elif self.device.type == "cuda":
                self._run_native(reqs)
            else:
                self._run_torch(reqs)
        finally:
            self._between = None
        return [RequestOutput(r.rid, r.prompt, [CompletionOutput(
                    0, r.text if r.text is not None else self.tokenizer.decode(r.out), r.out, r.finish, r.stop_reason,
                    r.logprobs, (sum(d[t] for d, t in zip(r.logprobs, r.out)) if r.logprobs is not None else None))],
                              metrics=self._req_metrics(r),
                              prompt_logprobs=r.prompt_logprobs)
                for r in reqs]

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _req_metrics(r: _Req) -> dict:
        """Latencies and the request's acceptance length: tokens emitted per decode step after
        the first token (1 + accepted drafts on average)."""
        steps = max(r.emits - 1, 0)
        return dict(ttft_s=r.t_first - r.t_arrive, e2e_s=r.t_done - r.t_arrive, decode_steps=steps,
                    tokens_per_step=(len(r.out) - 1) / steps if steps else None)

    def _emit(self, r: _Req, tokens, logits=None) -> bool:
        """Append emitted tokens (stop conditions apply per token); `logits` [n, V] are the
        rows that predicted them (for requested logprobs)."""
        n0 = len(r.out)
        r.emits += 1
        p = r.params
        entries = None
        if p.logprobs is not None and logits is not None:
            from .sampling_params import logprob_entries
            entries = logprob_entries(logits[: len(tokens)], [int(t) for t in tokens], p.logprobs)
            if r.logprobs is None:
                r.logprobs = []
        for j, t in enumerate(tokens):
            if r.finish:
                break
            t = int(t)
            r.out.append(t)
            if entries is not None:
                r.logprobs.append(entries[j])
            if len(r.out) >= p.min_tokens:
                if t in p.stop_token_ids:
                    r.finish, r.stop_reason = "stop", t
                elif not p.ignore_eos and t == self.tokenizer.eos_token_id:
                    r.finish = "stop"
                elif p.stop:
                    text = self.tokenizer.decode(r.out)
                    cut, hit = cut_at_stop(text, p.stop, p.include_stop_str_in_output)
                    if hit is not None:
                        r.finish, r.stop_reason, r.text = "stop", hit, cut
            if not r.finish and len(r.out) >= p.max_tokens:
                r.finish = "length"
        if r.finish and not r.t_done:
            r.t_done = time.perf_counter()
        if r.callback is not None and (len(r.out) > n0 or r.finish):
            if p.logprobs is not None:
                r.callback(r.out[n0:], r.finish, (r.logprobs or [])[n0:])
            else:
                r.callback(r.out[n0:], r.finish)
        return r.finish is not None

    def _poll(self, waiting, rows, n_free, release):
        """Serving hook: admit joined requests into `waiting`, finish aborted ones."""
        hook = getattr(self, "_between", None)
        if hook is None:
            return
        new, aborts = hook(n_free)
        for rid, prompt, sp, cb in new:
            try:
                self._check_request(prompt, sp)
            except (ValueError, NotImplementedError) as e:
                if cb is not None:
                    cb([], "error:" + str(e))
                continue
            waiting.append(_Req(rid, list(prompt), sp, t_arrive=time.perf_counter(), callback=cb))
        if not aborts:
            return
        for r in [r for r in waiting if r.rid in aborts]:
            waiting.remove(r)
            r.finish = "abort"
            if r.callback is not None:
                r.callback([], "abort")
        for r in list(rows):
            if r is not None and r.rid in aborts and not r.finish:
                r.finish, r.t_done = "abort", time.perf_counter()
                if r.callback is not None:
                    r.callback([], "abort")
                release(r)

    def _run_torch(self, reqs):
        waiting = deque(reqs)
        # serving: room for requests that join between steps (rows cost nothing on the CPU engine)
        B = self.ecfg.max_num_seqs if self._between is not None else max(1, min(len(reqs), self.ecfg.max_num_seqs))
        rows = [None] * B
        steps = accepted = 0
        prefilling = {}                 # row -> request whose chunked prefill is in progress
        self._decode_rows_last = 0
        self._chunk_log = []

        def release(r):
            rows[r.row] = None
            prefilling.pop(r.row, None)
            self.runner.release(r.row)
        ep = self._ep_group

        def group_max(v: int) -> int:
            """DP + EP: every rank makes the same MoE all-to-all calls, so row counts and
            the loop's end are agreed (MAX) and short ranks run empty rows."""
            if ep is None:
                return v
            import torch.distributed as dist
            t = torch.tensor([v], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ep)
            return int(t)
        while True:
            self._poll(waiting, rows, sum(r is None for r in rows) - len(waiting), release)
            if not group_max(int(bool(waiting or any(rows)))):
                break
            free = [i for i, r in enumerate(rows) if r is None]
            adm = []
            while waiting and free:
                r = waiting.popleft(); r.row = free.pop(0); rows[r.row] = r; adm.append(r)
            n_pref = group_max(len(adm))
            if self._chunk_budget is not None:
                self._chunked_prefills(adm, rows, prefilling)
                adm = []
            if adm:
                firsts = self.runner.prefill([r.prompt for r in adm], [r.row for r in adm], [r.params for r in adm])
                for r, f in zip(adm, firsts):
                    r.t_first = time.perf_counter()
                    pl = self.runner.prompt_logits.get(r.row)
                    if r.params.prompt_logprobs is not None and pl is not None:
                        from .sampling_params import logprob_entries
                        r.prompt_logprobs = [None] + (logprob_entries(pl, r.prompt[1:], r.params.prompt_logprobs)
                                                      if len(r.prompt) > 1 else [])
                    if self._emit(r, [f], self.runner.last_logits.get(r.row)):
                        rows[r.row] = None; self.runner.release(r.row)
            if ep is not None:
                self.runner.dummy_rows(n_pref - len(adm))
            live = [i for i, r in enumerate(rows) if r is not None and r.row not in prefilling]
            n_step = group_max(len(live))
            if not live:
                if ep is not None:
                    self.runner.dummy_rows(n_step)
                continue
            self._decode_rows_last = len(live)
            res = self.runner.step(live)
            if ep is not None:
                self.runner.dummy_rows(n_step - len(live))
            steps += 1
            for i, (toks, a) in res.items():
                accepted += a
                if self._emit(rows[i], toks, self.runner.last_logits.get(i)):
                    self.runner.release(i); rows[i] = None
        self.stats = dict(steps=steps, accepted=accepted, prefill_chunks=len(self._chunk_log))

    def _chunked_prefills(self, adm, rows, prefilling):
        """Chunked prefill: the step's token budget goes first to the running decode rows
        ((k + 1) tokens each), the rest to prefills in arrival order, a chunk at a time, so a
        long prompt never stalls the decoding rows for more than one budget of tokens.
        A prefill that completes emits its first token; its row decodes from the next step."""
        for r in adm:
            self.runner.start_prefill(r.prompt, r.row, r.params)
            prefilling[r.row] = r
        n_dec = sum(1 for r in rows if r is not None and r.row not in prefilling)
        budget = max(self._chunk_budget - n_dec * (self.k + 1), 1)       # prefills always advance
        for row in list(prefilling):
            if budget <= 0:
                break
            r = prefilling[row]
            before = self.runner.partial[row]["done"]
            f = self.runner.prefill_chunk(row, budget)
            done = len(r.prompt) if f is not None else self.runner.partial[row]["done"]
            budget -= done - before
            self._chunk_log.append((r.rid, before, done, n_dec))
            if f is None:
                continue
            del prefilling[row]
            r.t_first = time.perf_counter()
            pl = self.runner.prompt_logits.get(row)
            if r.params.prompt_logprobs is not None and pl is not None:
                from .sampling_params import logprob_entries
                r.prompt_logprobs = [None] + (logprob_entries(pl, r.prompt[1:], r.params.prompt_logprobs)
                                              if len(r.prompt) > 1 else [])
            if self._emit(r, [f], self.runner.last_logits.get(row)):
                rows[row] = None
                self.runner.release(row)

    def _state(self, B):
        st = self._states.get(B)
        if st is None:
            st = self._DecodeState(B, self.k, self.max_blocks, self.device)
            self._states[B] = st
        return st

    def _grow_state(self, st, B_new: int):
        """Serving: move the running rows to the decode state of a larger graph bucket (rows
        keep their index; KV caches are paged, so only tokens / positions / block tables move)."""
        st2 = self._state(B_new)
        n = st.B
        for name in ("tokens", "seq_pos", "block_table") + tuple(getattr(st, "SAMPLING", ())):
            dst, src = getattr(st2, name), getattr(st, name)
            dst.zero_()
            dst[:n].copy_(src)
        if getattr(st, "proc", None) is not None:
            pr2 = st2.ensure_processing(st.proc["counts"].shape[1])
            for name, src in st.proc.items():
                pr2[name][:n].copy_(src)
        return st2

    @staticmethod
    def _bucket(n: int) -> int:
        B = 1
        while B < n:
            B *= 2
        return B

    def _run_native(self, reqs):
        runner = self.runner
        B = self._bucket(min(len(reqs), self.ecfg.max_num_seqs))
        cap = self._bucket(self.ecfg.max_num_seqs)
        st = self._state(B)
        kp1 = self.k + 1
        pin_active = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        pin_out = torch.zeros(B, kp1, dtype=torch.int32, pin_memory=True)
        pin_acc = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        waiting = deque(reqs)
        rows: List[Optional[_Req]] = [None] * B
        steps = accepted = 0
        t_decode = 0.0
        bt_host = torch.zeros(B, self.max_blocks, dtype=torch.int32)
        prefilling = {}            # row -> (request, next prompt position, samples) of a chunked prefill
        self._chunk_log = []
        while True:
            # serving: the batch may grow into a larger bucket, so offer room up to `cap` rows
            room = (cap if self._between is not None else B) - sum(r is not None for r in rows) - len(waiting)
            self._poll(waiting, rows, room, lambda r: self._finish_row(r, rows))
            if not (waiting or any(r is not None for r in rows)):
                break
            n_live = sum(r is not None for r in rows)
            if self._between is not None and waiting and n_live >= B and B < cap:
                B_new = min(cap, self._bucket(n_live + len(waiting)))
                st = self._grow_state(st, B_new)
                rows = rows + [None] * (B_new - B)
                pin_active = torch.zeros(B_new, dtype=torch.int32, pin_memory=True)
                pin_out = torch.zeros(B_new, kp1, dtype=torch.int32, pin_memory=True)
                pin_acc = torch.zeros(B_new, dtype=torch.int32, pin_memory=True)
                bt_new = torch.zeros(B_new, self.max_blocks, dtype=torch.int32)
                bt_new[:B] = bt_host
                bt_host, B = bt_new, B_new
            free = [i for i, r in enumerate(rows) if r is None]
            adm = []
            pc = getattr(self.blocks, "prefix_caching", False)
            starts = []
            while waiting and free and self.blocks.can_allocate(
                    self._kv_rows(len(waiting[0].prompt) + waiting[0].params.max_tokens + kp1 + 1),
                    waiting[0].prompt if pc else None):
                r = waiting.popleft()
                r.row = free.pop(0)
                rows[r.row] = r
                n_tok = self._kv_rows(len(r.prompt) + r.params.max_tokens + kp1 + 1)
                if pc:
                    # shared prefix blocks; the block holding the position before the first new
                    # token is copied and that position computed again (its MTP entry differs)
                    blocks, m, cow = self.blocks.allocate_with_prefix(r.rid, n_tok, r.prompt)
                    if cow is not None:
                        runner.copy_block(*cow)
                        self.blocks.copied(r.rid)
                    starts.append(max(m - 1, 0))
                else:
                    blocks = self.blocks.allocate(r.rid, n_tok)
                    starts.append(0)
                bt_host[r.row].zero_()
                bt_host[r.row, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
                adm.append(r)
            if not adm and all(r is None for r in rows):
                raise MemoryError("KV cache too small for the next request")
            if adm:
                st.block_table.copy_(bt_host, non_blocking=False)
                sample_pf = self._set_sampling(st, adm)
                if self._chunk_budget is not None:
                    for r, s0 in zip(adm, starts):
                        prefilling[r.row] = (r, s0, sample_pf)
                else:
                    self._prefill_rows(adm, starts, sample_pf, st, bt_host, rows)
            if prefilling:
                self._gpu_chunks(prefilling, st, bt_host, rows)
            live = [r is not None and i not in prefilling for i, r in enumerate(rows)]
            if not any(live):
                continue
            for i, on in enumerate(live):
                pin_active[i] = 1 if on else 0
            st.set_active(pin_active.to(self.device, non_blocking=True))
            # a batch with a sampling row runs the bucket's speculative-sampling variant
            sample = any(r is not None and (r.params.temperature > 0 or r.params.processes_logits) for r in rows)
            self._step_sample = sample
            # spec guard: greedy batches switch to the no-draft step while the pool replays
            draft = self._spec_draft or sample or self.delta is not None
            self._step_draft = draft
            graph = None
            if self.ecfg.cuda_graphs:
                graph = (runner.sample_graphs if sample else runner.graphs if draft else runner.nodraft_graphs).get(B)
                if graph is None:
                    graph = runner.capture(st, **({"sample": True} if sample else {}),
                                           **({} if draft else {"draft": False}))
            t0 = time.perf_counter()
            if self.delta is not None:
                self._delta_snap = st.snapshot()
            if self.cache is not None:
                self.cache.wait_idle()           # safe point: no pool / slot-table mutation in flight
                self.cache.step_begin()
                snap = st.snapshot()
                step = graph.replay if graph is not None else (lambda: self._decode_eager(st))
                f0 = self.cache.stats["fetched_rows"]
                n_rep = self.replay.run(step, lambda: st.restore(snap), lambda: runner.route_ids(B))
                self.cache.step_end()
                self.kpi.step(replayed=n_rep > 0, misses=self.cache.stats["fetched_rows"] - f0,
                              fetched_rows=self.cache.stats["fetched_rows"] - f0)
                if self.spec_guard is not None:
                    self._spec_draft = self.spec_guard.observe(n_rep > 0)
                if getattr(self, "pilot", None) is not None:
                    self.pilot.observe(n_rep > 0)
                    self.pilot.consume()
                if self.affinity is not None and draft:
                    # learn token -> experts from this step's verify rows, then prefetch what the
                    # next step's drafts routed to before (asynchronously, off the decode stream)
                    self.affinity.record(snap[0].reshape(-1).tolist(),
                                         [t if t is not None and t.dim() == 2 else None for t in runner.route_ids(B)])
                    n_pf = self.affinity.prefetch(st.tokens[:, 1:].reshape(-1).tolist())
                    self.kpi.c["draft_prefetched"] += n_pf
                self._kpi_gauges(runner)
            elif graph is not None:
                graph.replay()
            else:
                self._decode_eager(st)
            if self.delta is not None:
                self._delta_step(st, B, graph, kp1)
            if self.routing is not None:
                self.routing.record(runner.route_ids(B))
            self._decode_steps += 1
            pin_out.copy_(st.out_tokens, non_blocking=True)
            pin_acc.copy_(st.n_acc, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            t_decode += time.perf_counter() - t0
            runner.check_status("decode step")
            steps += 1
            dl = self._full_logits(runner.main_logits(B)) \
                if any(r is not None and r.params.logprobs is not None for r in rows) else None
            if getattr(st, "proc", None) is not None:          # generated-token counts for the penalties
                cr, ct = [], []
                for i, r in enumerate(rows):
                    if r is not None and i not in prefilling:
                        n_i = int(pin_acc[i]) + 1
                        cr += [i] * n_i
                        ct += pin_out[i, :n_i].tolist()
                st.count_tokens(cr, ct)
            for i, r in enumerate(rows):
                if r is None or i in prefilling:
                    continue
                a = int(pin_acc[i])
                accepted += a
                lg = dl[i * kp1: i * kp1 + a + 1] if dl is not None else None      # verify rows of this request
                if self._emit(r, pin_out[i, :a + 1].tolist(), lg):
                    self._finish_row(r, rows)
        self.stats = dict(steps=steps, accepted=accepted, decode_s=t_decode, bucket=B)
        if getattr(runner, "_looka", None) is not None:
            self.stats["looka_recall"] = runner.looka_recall()
        if getattr(self, "pilot", None) is not None:
            self.stats["pilot"] = dict(self.pilot.stats)

    def _run_native_ep(self, reqs):
        """GPU engine loop under data-parallel attention + expert parallelism.  Every rank of
        the EP group serves its own requests, but every MoE layer is a collective, so the
        ranks step in lockstep: one small all-reduce per iteration agrees on whether anyone
        prefills (a rank with nothing to admit prefills a one-token dummy prompt into a
        private row) and whether anyone decodes (a rank with no live rows replays its step
        with every row inactive).  All ranks use one bucket per call (that of the busiest
        rank), so their decode graphs are captured in the same iteration.  Greedy only."""
        import torch.distributed as dist
        if any(r.params.temperature > 0 or r.params.processes_logits for r in reqs):
            raise NotImplementedError("GPU DP + EP decodes greedily (temperature 0, no logits processors)")
        runner, G = self.runner, self._ep_group
        # one bucket for the whole call on every rank: the smallest that holds the busiest rank
        nb = torch.tensor([min(len(reqs), self.ecfg.max_num_seqs)], dtype=torch.int32, device=self.device)
        dist.all_reduce(nb, op=dist.ReduceOp.MAX, group=G)
        B = self._bucket(max(int(nb), 1))
        st = self._state(B)
        kp1 = self.k + 1
        pin_active = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        pin_out = torch.zeros(B, kp1, dtype=torch.int32, pin_memory=True)
        pin_acc = torch.zeros(B, dtype=torch.int32, pin_memory=True)
        waiting = deque(reqs)
        rows: List[Optional[_Req]] = [None] * B
        bt_host = torch.zeros(B, self.max_blocks, dtype=torch.int32)
        flag = torch.zeros(3, dtype=torch.int32, device=self.device)
        steps = accepted = 0
        t_decode = 0.0
        if self._ep_dummy is None:      # private row of the dummy prefill: its own state and KV block
            blocks = self.blocks.allocate("__ep_dummy__", 8)
            bt = [0] * self.max_blocks
            bt[0] = blocks[0]
            self._ep_dummy = (self._DecodeState(1, self.k, self.max_blocks, self.device), bt)
        while True:
            free = [i for i, r in enumerate(rows) if r is None]
            adm = []
            while waiting and free and self.blocks.can_allocate(
                    len(waiting[0].prompt) + waiting[0].params.max_tokens + kp1 + 1):
                r = waiting.popleft()
                r.row = free.pop(0)
                rows[r.row] = r
                blocks = self.blocks.allocate(r.rid, len(r.prompt) + r.params.max_tokens + kp1 + 1)
                bt_host[r.row].zero_()
                bt_host[r.row, :len(blocks)] = torch.tensor(blocks, dtype=torch.int32)
                adm.append(r)
            flag[0] = 1 if adm else 0
            flag[1] = 1 if any(r is not None for r in rows) else 0
            flag[2] = 1 if waiting else 0
            dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=G)
            f = flag.tolist()
            if not (f[0] or f[1]):
                if f[2]:
                    raise MemoryError("KV cache too small for the next request")
                break
            if f[0]:
                if adm:
                    st.block_table.copy_(bt_host, non_blocking=False)
                    self._set_sampling(st, adm)
                    self._prefill_rows(adm, [0] * len(adm), False, st, bt_host, rows)
                else:
                    dst, dbt = self._ep_dummy
                    runner.prefill([[1]], [dbt], [0], dst)
            if not f[1] and not f[0]:
                continue
            for i, r in enumerate(rows):
                pin_active[i] = 1 if r is not None else 0
            st.set_active(pin_active.to(self.device, non_blocking=True))
            self._step_sample = False
            graph = None
            if self.ecfg.cuda_graphs:
                graph = runner.graphs.get(B)
                if graph is None:
                    graph = runner.capture(st)
            t0 = time.perf_counter()
            if graph is not None:
                graph.replay()
            else:
                self._decode_eager(st)
            pin_out.copy_(st.out_tokens, non_blocking=True)
            pin_acc.copy_(st.n_acc, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            t_decode += time.perf_counter() - t0
            runner.check_status("decode step")
            steps += 1
            for i, r in enumerate(rows):
                if r is None:
                    continue
                a = int(pin_acc[i])
                accepted += a
                if self._emit(r, pin_out[i, :a + 1].tolist()):
                    self._finish_row(r, rows)
        self.stats = dict(steps=steps, accepted=accepted, decode_s=t_decode, bucket=B)

    def _prefill_rows(self, adm, starts, sample_pf, st, bt_host, rows):
        """Prefill admitted requests whose positions before `starts` are cached; emit their
        first tokens."""
        runner = self.runner
        bts = [bt_host[r.row].tolist() for r in adm]
        with self.timers.span("prefill") if self.timers is not None else contextlib.nullcontext():
            kw = dict(({"sample": True} if sample_pf else {}), **({"starts": starts} if any(starts) else {}))
            sp = getattr(self, "_sp_group", None) is not None and not sample_pf and not any(starts)
            if sp and all(runner.sp_chunk(len(r.prompt)) is not None for r in adm):
                # sequence-parallel prefill, one prompt at a time over the group's ranks
                firsts = [runner.prefill_sp(r.prompt, bt, r.row, st) for r, bt in zip(adm, bts)]
            else:
                firsts = runner.prefill([r.prompt for r in adm], bts, [r.row for r in adm], st, **kw).tolist()
        if getattr(self.blocks, "prefix_caching", False):
            for r in adm:
                self.blocks.register(r.rid, r.prompt)
        now = time.perf_counter()
        want_lp = any(r.params.logprobs is not None for r in adm)
        pl = self._full_logits(runner.ws_prefill.get("main.logits", (len(adm), self._vocab_local()), torch.float32)) \
            if want_lp else None
        if getattr(st, "proc", None) is not None:
            st.count_tokens([r.row for r in adm], firsts)
        for j, (r, f) in enumerate(zip(adm, firsts)):
            r.t_first = now
            if self._emit(r, [f], pl[j:j + 1] if pl is not None else None):
                self._finish_row(r, rows)

    def _vocab_local(self) -> int:
        head = getattr(getattr(self, "mw", None), "lm_head", None)
        return head.shape[0] if head is not None and self._tp_group is not None else self.cfg.vocab

    def _full_logits(self, lg):
        """Logprobs under TP: the ranks' vocab shards gathered into whole rows (every rank
        runs the same host loop, so the collective lines up)."""
        if lg is None or self._tp_group is None or self.device.type != "cuda":
            return lg
        from ..spec.device_sampler import gather_vocab
        return gather_vocab(lg.contiguous(), self._tp_group)

    def _gpu_chunks(self, prefilling, st, bt_host, rows):
        """Chunked prefill on the GPU runner: the step's token budget goes to the decoding
        rows first ((k + 1) each), the rest to prefills in arrival order.  A non-final chunk
        runs `prefill_chunk`; the last one is a prefill from its start position."""
        kp1 = self.k + 1
        n_dec = sum(1 for i, r in enumerate(rows) if r is not None and i not in prefilling)
        budget = max(self._chunk_budget - n_dec * kp1, 1)
        finals = []
        for row in list(prefilling):
            r, s0, smp = prefilling[row]
            if rows[row] is not r:                     # aborted while prefilling
                del prefilling[row]
                continue
            if budget <= 0:
                break
            n = len(r.prompt)
            e = min(n, s0 + budget)
            self._chunk_log.append((r.rid, s0, e, n_dec))
            budget -= e - s0
            if e < n:
                self.runner.prefill_chunk(r.prompt, bt_host[row].tolist(), s0, e)
                prefilling[row] = (r, e, smp)
            else:
                finals.append((r, s0, smp))
                del prefilling[row]
        if finals:
            self._prefill_rows([f[0] for f in finals], [f[1] for f in finals], any(f[2] for f in finals), st,
                               bt_host, rows)

    def _decode_eager(self, st):
        if getattr(self, "_step_sample", False):
            self.runner.decode_body(st, True)
        elif not getattr(self, "_step_draft", True):
            self.runner.decode_body(st, draft=False)
        else:
            self.runner.decode_body(st)

    def _set_sampling(self, st, adm) -> bool:
        """Write the admitted rows' sampling parameters into the decode state (an unseeded
        request gets a random seed) -> whether any of them samples."""
        if hasattr(st, "ensure_processing"):
            # the state's processing tensors exist before its sampling-variant graph is captured
            if any(r.params.processes_logits or r.params.temperature > 0 for r in adm):
                st.ensure_processing(self.cfg.vocab)
            if st.proc is not None:
                for r in adm:
                    st.set_processing(r.row, r.prompt, r.params)
        if not any(r.params.temperature > 0 or r.params.processes_logits for r in adm):
            if hasattr(st, "set_sampling"):
                st.set_sampling([r.row for r in adm], [0.0] * len(adm), [0] * len(adm), [1.0] * len(adm),
                                [0.0] * len(adm), [0] * len(adm))
            return False
        ps = [r.params for r in adm]
        drawn = self._shared_seeds(len(ps))
        st.set_sampling([r.row for r in adm], [p.temperature for p in ps], [p.top_k for p in ps],
                        [p.top_p for p in ps], [p.min_p for p in ps],
                        [p.seed if p.seed is not None else d for p, d in zip(ps, drawn)])
        return True

    def _kv_rows(self, n: int) -> int:
        """Cache rows this rank keeps for n positions (DCP: only its own positions)."""
        if getattr(self, "_dcp", None) is None:
            return n
        from .gpu_runner import dcp_local_count
        return dcp_local_count(n, *self._dcp)

    def _shared_seeds(self, n: int) -> list:
        """n random seeds, equal on every rank of the tensor-parallel group."""
        from .sampling_params import shared_seeds
        return shared_seeds(n, getattr(self, "_seed_group", getattr(self, "_tp_group", None)), self.device)

    def _delta_step(self, st, B, graph, kp1):
        """After a decode step: feed routing to the delta tier's frequency policy and,
        with the confidence gate, promote this step's routed experts to FP4 and
        replay the step while the verify rows are not confident."""
        from ..residency import gate_promote_consensus
        pairs = self._routed_pairs(B)
        for li, e in pairs:
            self.delta.note_routed(li, [e])
        if self.delta_trace is not None:
            self.delta_trace.step(self.delta, self._routed_token_counts(B))
        if self.gate is not None:
            m = self.ecfg.moet
            logits = self.runner.main_logits(B)
            step = (graph.replay if graph is not None else (lambda: self._decode_eager(st)))
            snap = self._delta_snap

            def gate_rows():
                # the verify rows the gate scores: every active row, or with GATE_SPEC_MASK only
                # the rows the step emits (a row past the first rejected draft is discarded)
                act = st.active_rows.reshape(-1).bool()
                if m.gate_spec_mask and self.k > 0:
                    act = act & (st.arange_kp1[None, :] <= st.n_acc.reshape(-1, 1)).reshape(-1)
                return torch.nonzero(act).flatten()
            rows = gate_rows()

            def run_step():
                st.restore(snap)
                if self.cache is not None:      # base misses met by the replayed step are repaired too
                    self.cache.wait_idle()
                    self.replay.run(step, lambda: st.restore(snap), lambda: self.runner.route_ids(B))
                else:
                    step()
                return logits[gate_rows()] if logits is not None else None   # no head before the last PP stage
            if self._pp_group is not None:
                fired = self._pp_gate(B, run_step, lambda: self.gate.score(logits[rows], tp_group=self._tp_group))
                self.delta.stats["gate_replays"] += fired
                self.delta.step_end()
                return
            # the step already ran once: score it, fire, replay (at most gate_fp_max times)
            score = self.gate.score(logits[rows], tp_group=self._tp_group)
            score0, fired, iters = score, 0, []
            timing = self.ecfg.moet.gate_fire_timing
            pre = logits[rows].argmax(-1).cpu() if logits is not None else None
            # audit: a confident step fires anyway with probability p, so the logged flips give
            # unbiased labels of what the gate misses; a seeded generator, the same on every rank
            audit = (m.gate_audit > 0 and not self.gate.should_fire(score)
                     and self._audit_rng().random() < m.gate_audit)
            if m.gate_capture:     # measurement mode: the decision is logged, nothing changes
                if self.gate_log is not None:
                    self.gate_log.write({"step": self._decode_steps, "score": score0, "tau": self.gate.tau,
                                         "would_fire": bool(self.gate.should_fire(score)), "capture": True})
                self.delta.step_end()
                return
            while fired < self.gate.fp_max and (self.gate.should_fire(score) or (audit and fired == 0)):
                promote = [p for p in self._routed_pairs(B) if not self.delta.resident(*p)]
                if len(promote) > self.gate.max_promote:
                    # a binding cap promotes the most-needed experts first (the tier's decayed
                    # rank: repeat offenders across fires), ties in routing order
                    fq = self.delta.freq
                    if m.delta_rank == "step_w":     # this step's heaviest routing weight first
                        sw = self._step_weights(B)
                        promote = sorted(promote, key=lambda p: (-sw.get(p, 0.0), -float(fq[p[0], p[1]])))
                    else:
                        promote = sorted(promote, key=lambda p: -float(fq[p[0], p[1]]))
                promote = promote[: self.gate.max_promote]
                t0 = time.perf_counter()
                # fail-safe: a failed host read on any TP rank means no rank replays
                if not gate_promote_consensus(lambda: self.delta.promote(promote) if promote else 0,
                                              self._tp_group, self.device):
                    break
                t1 = time.perf_counter()
                if timing:
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                if not m.gate_reforward:     # promoted for the next steps; this step stands
                    iters.append({"promoted": len(promote), "reforward": False})
                    fired += 1
                    break
                score = self.gate.score(run_step(), tp_group=self._tp_group)
                it = {"promoted": len(promote), "score": score}
                if timing:
                    e1.record()
                    e1.synchronize()
                    it.update(promote_ms=(t1 - t0) * 1e3, replay_ms=e0.elapsed_time(e1))
                iters.append(it)
                fired += 1
                if m.gate_trace:
                    import logging
                    logging.getLogger("vllm_moet_b200").info(
                        "gate %s step %d: score %.4f -> %.4f (tau %.3f), promoted %d",
                        "audit" if audit else "fire", self._decode_steps, score0, score, self.gate.tau, len(promote))
            if m.gate_reforward:
                self.delta.stats["gate_replays"] += fired
            else:
                self.delta.stats["gate_promote_only"] += fired
            self.delta.stats["gate_audits"] += int(audit and fired > 0)
            if self.gate_log is not None:
                rec = {"step": self._decode_steps, "score": score0, "tau": self.gate.tau,
                       "fired": fired, "final_score": score, "iters": iters, "audit": bool(audit and fired > 0)}
                if fired and pre is not None:
                    post = logits[gate_rows()].argmax(-1).cpu()
                    n = min(len(pre), len(post))
                    rec["flips"] = int((pre[:n] != post[:n]).sum())
                self.gate_log.write(rec)
                hid = getattr(self.runner, "main_hidden", None)
                if fired and getattr(self, "hcap", None) is not None and hid is not None:
                    h = hid(B)
                    if h is not None:
                        self.hcap.store(self._decode_steps, h[gate_rows()])
        else:
            self.delta.tick(self.ecfg.moet.delta_promote)
        self.delta.step_end()

    def _audit_rng(self):
        import random
        if getattr(self, "_gate_audit_rng", None) is None:
            self._gate_audit_rng = random.Random(self.ecfg.seed * 7919 + 17)
        return self._gate_audit_rng

    def _pp_gate(self, B, run_step, score_fn) -> int:
        """The gate under pipeline parallelism: only the last stage has the verify logits,
        every stage owns its layers' experts.  Per round, the last stage's fire decision is
        broadcast, every stage promotes its own routed experts, the outcome is agreed
        (TP, then PP; fail closed), and then every stage replays the step together (its
        sends / receives pair up).  -> replays."""
        from ..residency import FetchError, pp_gate_barrier
        last = self.runner.last_stage
        score = score_fn() if last else 0.0
        fired = 0
        while fired < self.gate.fp_max:
            fire = bool(last and self.gate.should_fire(score))

            def promote():
                pairs = [p for p in self._routed_pairs(B) if not self.delta.resident(*p)][: self.gate.max_promote]
                if pairs and self.delta.promote(pairs) == 0:
                    raise FetchError("nothing promoted")
            if not pp_gate_barrier(fire, promote, tp_group=self._tp_group, pp_group=self._pp_group,
                                   device=self.device):
                break
            out = run_step()
            score = self.gate.score(out, tp_group=self._tp_group) if last else 0.0
            fired += 1
        return fired

    def _finish_row(self, r, rows):
        rows[r.row] = None
        self.blocks.release(r.rid)
