"""Native (sm_100a) model executor: prefill, MTP speculative decode steps and
CUDA-graph capture of the decode step.

All per-step state lives on the device (input tokens, positions, block
tables, acceptance), so one captured graph per batch bucket replays a whole
decode step -- main model over B*(1+k) verify rows, greedy acceptance, two
chained MTP draft passes and the advance of every sequence -- with no host
round trip inside.  The host only reads the emitted tokens back.

Kernel order of one decoder layer (T rows):
  rmsnorm_quant -> gemv(qkv_a) -> rmsnorm_quant(q_a) | kv_prep(norm, rope, cache write)
  -> gemv(q_b) -> q_prep(rope, fp8 q_nope) -> gemv_batched(W_uk^T) -> mla_decode -> mla_combine(fp8)
  -> gemv_batched(W_uv) -> quant -> gemv(o, +residual)
  -> rmsnorm_quant(bf16 + fp8 natural + fp8 w2 layout) -> router logits -> router_topk -> build_pairs
  -> moe_w2_gemv(w13) -> swiglu_quant -> moe_w2_gemv(w2) ; shared expert gemvs -> moe_combine(+residual)
Prefill replaces the absorbed attention with the non-absorbed flash kernel.
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass
from typing import Optional

import torch

from ..config import EngineConfig, ModelConfig
from ..models.reference import rope_cos_sin
from ..models.weights import LayerWeights, ModelWeights
from ..ops import native

KV_BLOCK = 64
BF16_ROW = 584      # bf16 elements per cache row (512 latent + 64 rope + 8 pad)
NVFP4_ROW = 352     # bytes per NVFP4 row


def _split_cols(lin, k0: int, k1: int):
    """Columns [k0, k1) of a linear (input features) as a linear of its own (contiguous);
    FP8 weights split on their 128-column scale blocks."""
    from ..models.weights import Fp8Linear, FloatLinear
    if isinstance(lin, Fp8Linear):
        if k0 % 128 or k1 % 128:
            raise ValueError("FP8 column split on 128-column blocks")
        return Fp8Linear(lin.w[:, k0:k1].contiguous(), lin.s[:, k0 // 128:k1 // 128].contiguous())
    if isinstance(lin, FloatLinear):
        return FloatLinear(lin.w[:, k0:k1].contiguous())
    raise NotImplementedError(f"column split of {type(lin).__name__}")


def dcp_local_count(n, W: int, r: int, I: int):
    """How many of positions [0, n) rank r of W holds when position p lives on rank
    (p // I) % W (ints or tensors)."""
    cyc = I * W
    rem = n % cyc - r * I
    if isinstance(rem, torch.Tensor):
        return (n // cyc) * I + rem.clamp(0, I)
    return (n // cyc) * I + min(max(rem, 0), I)


def dcp_slots(bt, seq, pos, W: int, r: int, I: int):
    """Cache slots of positions `pos` of rows `seq` on rank r: the rank keeps its positions
    densely (local index (p // (I W)) I + p % I through its block table); -1 where another
    rank holds the position."""
    own = (pos // I) % W == r
    lp = (pos // (I * W)) * I + pos % I
    blk = bt[seq, torch.where(own, lp // KV_BLOCK, torch.zeros_like(lp))].long()
    return torch.where(own, blk * KV_BLOCK + lp % KV_BLOCK, torch.full_like(lp, -1))


class Workspace:
    """Grow-only named device buffers; frozen once a graph has been captured."""

    def __init__(self, device):
        self.device = device
        self.bufs = {}
        self.frozen = False

    def get(self, name, shape, dtype):
        n = 1
        for s in shape:
            n *= s
        b = self.bufs.get((name, dtype))
        if b is None or b.numel() < n:
            if self.frozen:
                raise RuntimeError(f"workspace {name} must grow to {shape} after graph capture")
            b = torch.empty(max(n, 1), dtype=dtype, device=self.device)
            self.bufs[(name, dtype)] = b
        return b[:n].view(*shape)

    def zeros(self, name, shape, dtype):
        """Like get(), but zero-initialised on first allocation (kernels keep it zero after use)."""
        key = (name, dtype)
        fresh = key not in self.bufs
        t = self.get(name, shape, dtype)
        if fresh:
            self.bufs[key].zero_()
        return t


@dataclass
class StepCtx:
    T: int
    pos: torch.Tensor            # [T] int32
    seq: torch.Tensor            # [T] int32 (row into block_table)
    slot: torch.Tensor           # [T] int64
    block_table: torch.Tensor    # [S, max_blocks] int32
    mode: str                    # "decode" | "prefill" | "cached" (prefill compute, attention over the
                                 # paged cache: a prompt whose leading positions are already cached)
    cu_seqlens: Optional[torch.Tensor] = None
    max_len: int = 0
    mb: int = 8                  # rows per expert pair
    # "cached" mode on the flash path: cache slots of every key row (sequence i's positions
    # [0, end_i)) and their cu_seqlens; None = attention reads the paged cache (absorbed)
    kv_idx: Optional[torch.Tensor] = None
    cu_k: Optional[torch.Tensor] = None
    # decode context parallelism: per row, the index of its last key among this rank's
    # positions (-1: none yet); None without DCP
    lpos: Optional[torch.Tensor] = None


class NativeRunner:
    def __init__(self, mw: ModelWeights, ecfg: EngineConfig, num_blocks: int, device="cuda"):
        self.C = native()
        self.mw = mw
        self.cfg: ModelConfig = mw.cfg
        self.ecfg = ecfg
        self.dev = torch.device(device)
        self._init_draft_module(mw)
        has_mtp = self._draft is not None or (mw.extra.get("pp_size", 1) > 1 and mw.cfg.num_mtp_layers > 0)
        self.k = ecfg.num_speculative_tokens if has_mtp else 0
        # heads per rank: all of them when attention is replicated across the TP group
        attn_tp = all(getattr(lw, "attn_tp", True) for lw in mw.layers)
        self.Hh = self.cfg.num_heads // mw.tp_size if attn_tp else self.cfg.num_heads
        cfg = self.cfg
        self.num_blocks = num_blocks
        self.kv_mode = 2 if ecfg.kv_cache_dtype == "nvfp4" else 1
        n_cache = len(mw.layers) + (1 if self._draft is not None else 0)
        if self.kv_mode == 2:      # NVFP4 latent cache: 352 bytes per token (3.3x the context of bf16 rows)
            self.kv = [torch.zeros(num_blocks, KV_BLOCK, NVFP4_ROW, dtype=torch.uint8, device=self.dev)
                       for _ in range(n_cache)]
        else:
            self.kv = [torch.zeros(num_blocks, KV_BLOCK, BF16_ROW, dtype=torch.bfloat16, device=self.dev)
                       for _ in range(n_cache)]
        self.cos_sin = rope_cos_sin(cfg, ecfg.max_model_len + 64, self.dev)
        # DSA indexer key caches (bf16 [blocks, 64, D] per layer with an indexer)
        self.idx_kv = [torch.zeros(num_blocks, KV_BLOCK, cfg.index_head_dim, dtype=torch.bfloat16, device=self.dev)
                       if lw.idx_wq is not None else None
                       for lw in list(mw.layers) + ([self._draft.layer] if self._draft is not None else [])]
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.miss = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.ws_decode_by_bucket = {}
        self.ws_prefill = Workspace(self.dev)
        self.ws = self.ws_prefill
        self.scale = 1.0 / math.sqrt(cfg.qk_head_dim)
        self.graphs = {}
        self.sample_graphs = {}       # bucket -> graph of the speculative-sampling decode step
        self.nodraft_graphs = {}      # bucket -> graph of the greedy step without drafts (spec guard)
        self.tp_group = None
        self.tp_rank, self.tp_size = mw.tp_rank, mw.tp_size
        self.ar = None            # fused peer-memory all-reduce (SymmAllReduce) for decode-sized steps
        self.ep = None            # expert-parallel all-to-all buffers (EpSymm) under DP attention + EP
        self.ep_group = None
        self.sp_group = None      # sequence-parallel prefill ranks (replicated weights)
        self.dcp = None           # decode context parallelism: (group, world, rank, interleave)
        self._sp = None           # active SP prefill: (group, world, rank, block ids per rank's chunk)
        self.cache = None         # residency.ExpertCache when routed experts are served from a host store
        self.delta = None         # residency.DeltaTier (FP4 hot experts) when enabled
        self._moe_index = {}
        self._looka = None        # router lookahead (enable_looka)
        self.trellis = None       # residency.TrellisBaseTier serving the routed experts of its layers
        self.trellis_delta = None
        self._trellis_li = {}
        self._route_tag = ""      # routing-buffer suffix of the current MTP draft pass
        self._pend = None         # (residual, out) of a pushed reduction the next RMSNorm completes
        self._pend_add = None     # (residual, reduced partial, out): decode residual add left to the next norm
        self._decode = False
        self._fused = False
        self._init_hyper_connections()
        # pipeline parallelism: this stage's layers; first stage embeds, last stage owns head + MTP
        self.pp_group = None
        self.pp_rank, self.pp_size = mw.extra.get("pp_rank", 0), mw.extra.get("pp_size", 1)
        self.first_stage, self.last_stage = self.pp_rank == 0, self.pp_rank == self.pp_size - 1
        self.nsplit = 8
        self._side = torch.cuda.Stream(device=self.dev)   # second graph branch for independent chains
        import os
        self.debug_finite = os.environ.get("MOET_DEBUG_FINITE", "0") == "1"
        self.branches = os.environ.get("MOET_BRANCHES", "1") != "0"
        self.gemv_stream = os.environ.get("MOET_GEMV_STREAM", "1") != "0"
        self.timers = None          # SpanTimers of prefill components (VLLM_PREFILL_TIMERS_FLUSH)
        # token count from which dense linears run on the tcgen05 GEMM (128-token tiles)
        self.tc_min_t = int(os.environ.get("MOET_TC_MIN_T", "16"))
        # "cached" chunks of at least this many rows run the flash prefill kernel over key
        # rows gathered from the cache (W_kv_b applied to them) instead of absorbed attention
        self.cached_flash_min = int(os.environ.get("MOET_CACHED_FLASH_MIN", "128"))
        # decode expert tiles: 8-token pairs up to this many routed rows, 16-token pairs above
        self.mb8_max_r = int(os.environ.get("MOET_MB8_MAX_R", "2048"))
        # decode experts on the tcgen05 kernel with this token tile (0: mma.sync GEMV)
        self.decode_tc_nt = int(os.environ.get("MOET_DECODE_TC_NT", "0"))
        # decode experts over the 2-bit base: "legacy" (mma.sync GEMV, default) or "tcd" (tcgen05
        # block-scaled, K-sliced; measured slower at 1-32 streams, see moe_w2_tcd.cu); 128-k stages
        # per K slice of the tcgen05 kernel
        self.w2_decode = os.environ.get("MOET_W2_DECODE", "legacy")
        self.w2_tcd_spt = int(os.environ.get("MOET_W2_TCD_SPT", "8"))
        # K-split the mma.sync decode expert GEMV when its grid is small (MOET_W2_KSPLIT=0: off)
        self.w2_ksplit = os.environ.get("MOET_W2_KSPLIT", "1") != "0"

    # ------------------------------------------------------------------ helpers
    @staticmethod
    def _pad128(T):
        return (T + 127) // 128 * 128

    def _fp8(self, name, T, K):
        """FP8 activation buffers; rows are allocated in multiples of 128 so the
        tensor-core GEMM can read whole 128-row TMA boxes (callers see [:T])."""
        Tp = self._pad128(T) if T >= self.tc_min_t else T
        q = self.ws.get(name + ".q", (Tp, K), torch.uint8)
        s = self.ws.get(name + ".s", (Tp, K // 64), torch.uint8)
        return q[:T], s[:T]

    @staticmethod
    def _padded_view(t, rows):
        """The 128-row padded parent of a [:T] view made by _fp8, or None."""
        if not t.is_contiguous():
            return None
        need = rows * t.shape[1] * t.element_size()
        if t.untyped_storage().nbytes() - t.storage_offset() * t.element_size() < need:
            return None
        return t.as_strided((rows, t.shape[1]), t.stride())

    def _gemv(self, aq, as_, lin, out, resid=None):
        """Dense FP8 linear: the warp-specialized tcgen05 GEMM for prefill-sized
        token counts, the weight-streaming GEMV for decode-sized ones."""
        T, K = aq.shape[0], lin.w.shape[-1]
        N = lin.w.shape[0]
        if T >= self.tc_min_t and K % 128 == 0 and lin.w.dim() == 2 and N % 8 == 0:
            Tp = self._pad128(T)
            ap, sp = self._padded_view(aq, Tp), self._padded_view(as_, Tp)
            if ap is not None and sp is not None:
                self.C.ws_gemm_fp8(ap, sp, lin.w, lin.s, out, resid, T, self.status)
                return
        if T > 128 and K % 128 == 0 and lin.w.dim() == 2 and aq.stride(0) % 16 == 0:
            self.C.tc_gemm_fp8(aq, as_, lin.w, lin.s, out, resid, 128, self.status)
        elif (T <= 8 and lin.w.dim() == 2 and K % 128 == 0 and K <= 5120 and aq.stride(0) % 16 == 0
              and self.gemv_stream):
            # persistent TMA-ring GEMV: weight rows stream through shared memory continuously
            self.C.gemv_stream_fp8(aq, as_, lin.w, lin.s, out, resid, self.status)
        else:
            self.C.gemv_fp8(aq, as_, lin.w, lin.s, out, resid)

    def _argmax(self, logits, ids):
        R = logits.shape[0]
        part = self.ws.get("argmax.part", (max(R, 1), 32, 3), torch.float32)
        assert R <= 8192, "argmax rows"
        cnt = self.ws.zeros("argmax.cnt", (8192,), torch.int32)
        if self.tp_group is None:
            self.C.argmax_split(logits, ids, None, self.status, part, cnt)
            return
        # vocab-parallel head: local (max, global id) per row, gathered, merged
        mv = self.ws.get("argmax.mv", (R, 2), torch.float32)
        self.C.argmax_split(logits, None, None, self.status, part, cnt, mv, self.tp_rank * logits.shape[1])
        if self.ar is not None and 2 * R <= self.ar.cap:
            # one kernel: push the pairs to every peer over NVLink, wait, merge in rank order
            self.C.argmax_merge_ar(mv, ids, self.ar.desc)
            return
        allmv = self.ws.get("argmax.all", (self.tp_size, R, 2), torch.float32)
        torch.distributed.all_gather_into_tensor(allmv, mv, group=self.tp_group)
        self.C.argmax_merge(allmv, ids)

    def _router_logits(self, hb, lw, logits):
        """Router logits; decode-sized batches (up to 512 rows) give the kernel scratch for
        K-sliced partials and per-tile counters, so tens of rows still fill the GPU."""
        T, E = logits.shape
        if 64 < T <= 512:
            part = self.ws.get("router.part", (16 * T * E,), torch.float32)
            cnt = self.ws.zeros("router.cnt", (64,), torch.int32)
            self.C.router_logits(hb, self._router_w(lw), logits, part, cnt)
        else:
            self.C.router_logits(hb, self._router_w(lw), logits)

    def _router_w(self, lw):
        w = getattr(lw, "_router_w_bf16", None)
        if w is None:
            w = lw.router_w.to(torch.bfloat16).contiguous()
            lw._router_w_bf16 = w
        return w

    def set_tp_group(self, group, fused: Optional[bool] = None):
        """Join a tensor-parallel group.  Decode-sized reductions (at most
        MOET_TP_FUSED_MAX_T rows, default 8) run fused over peer memory: the
        producing kernel's epilogue (streaming GEMV, expert combine) pushes its
        partial into every peer, the next norm -- the streaming GEMV's fused-norm
        prologue or rmsnorm_quant -- waits and reduces; the vocab-parallel argmax
        merges over the same buffers.  Larger reductions use NCCL all-reduce.
        MOET_TP_FUSED=1 turns the fused path on (off by default until measured on NVLink)."""
        import os
        self.tp_group = group
        self.fused_max_t = int(os.environ.get("MOET_TP_FUSED_MAX_T", "8"))
        if fused is None:
            fused = os.environ.get("MOET_TP_FUSED", "0") == "1"
        if fused and group is not None:
            from ..parallel.symm import SymmAllReduce
            self.ar = SymmAllReduce(group, 128 * self.cfg.hidden, self.dev, self.status)

    def set_ep_group(self, group, cap_rows: int):
        """Data-parallel attention + expert-parallel MoE: this rank holds the routed experts
        [rank * E / W, (rank + 1) * E / W) and its own tokens.  Decode-sized MoE layers move
        their rows over peer memory (dispatch kernel, owner's pair list, w2 GEMV epilogue
        storing into the source's return rows, combine after a bounded wait); prefill-sized
        ones use NCCL all-to-all.  ``cap_rows``: the most routed rows (tokens x top-k) of one
        rank in one decode-sized layer."""
        from ..parallel.symm import EpSymm
        from ..residency import moe_layers
        ex = moe_layers(self.mw)[0].experts
        if ex.n_local is None:
            raise ValueError("set_ep_group: the experts are not partitioned (parallel.ep.ep_partition)")
        if self.cache is not None or self.delta is not None:
            raise NotImplementedError("expert parallelism with the expert cache / delta tier")
        self.ep_group = group
        self.ep = EpSymm(group, cap_rows, self.cfg.hidden, ex.n_local, self.cfg.top_k, self.dev, self.status)

    def _moe_ep_decode(self, h2q, h2s, ids, ex, MB):
        """Decode-sized EP layer up to the owners' return stores (the caller's combine waits)."""
        C, cfg, ep = self.C, self.cfg, self.ep
        H, I = cfg.hidden, ex.layout.I
        L = ex.layout
        R = ep.world * ep.cap
        P = R // MB + min(ep.E_loc, R)
        idr = self.ws.get("ep.ids", (R,), torch.int32)
        rank = self.ws.get("ep.rank", (R,), torch.int32)
        stok = self.ws.get("ep.stok", (R,), torch.int32)
        posof = self.ws.get("ep.posof", (R,), torch.int32)
        pairs = self.ws.get("ep.pairs", (P, 4), torch.int32)
        npairs = self.ws.get("ep.npairs", (1,), torch.int32)
        nrows = self.ws.get("ep.nrows", (1,), torch.int32)
        C.ep_dispatch(ep.desc, h2q, h2s, ids)
        C.ep_recv_pairs(ep.desc, MB, idr, rank, stok, posof, pairs, npairs, nrows)
        c13 = self.ws.get("ep.c13", (self._w2_ksplit(2 * I, H, cfg.top_k * ep.world), R, 2 * I), torch.float32)
        C.moe_w2_gemv(ep.rx, ep.rs, stok, pairs, npairs, ex.pool, L.off_codes13, L.off_sc13, ex.slot_table, c13,
                      2 * I, H, MB, self.miss)
        a2q, a2s = self._fp8("ep.a2", R, I)
        C.swiglu_quant(c13, cfg.swiglu_limit or 0.0, nrows, 1, a2q, a2s)
        C.moe_w2_gemv(a2q, a2s, None, pairs, npairs, ex.pool, L.off_codes2, L.off_sc2, ex.slot_table, ep.ret,
                      H, I, MB, self.miss, ep=ep.desc, ret_rows=stok)

    def _moe_ep_prefill(self, h2q, h2s, ids, ex, T, MB):
        """Prefill-sized EP layer with NCCL all-to-all (the parallel/ep.py algorithm) around
        this rank's expert kernels -> [T * k, H] f32 expert outputs in (token, slot) order."""
        import torch.distributed as dist
        C, cfg, ep = self.C, self.cfg, self.ep
        H, k, W = cfg.hidden, cfg.top_k, ep.world
        flat = ids.reshape(-1).long()
        dest = flat // ep.E_loc
        order = torch.argsort(dest, stable=True)
        send = torch.bincount(dest, minlength=W).to(torch.int64)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.ep_group)
        sc, rc = send.tolist(), recv.tolist()

        def a2a(x, scnt, rcnt):
            out = x.new_empty((sum(rcnt),) + tuple(x.shape[1:]))
            dist.all_to_all_single(out, x.contiguous(), rcnt, scnt, group=self.ep_group)
            return out
        tok = torch.arange(T, device=ids.device).repeat_interleave(k)[order]
        q = a2a(h2q[tok], sc, rc)
        sq = a2a(h2s[tok], sc, rc)
        lid = a2a((flat[order] - dest[order] * ep.E_loc).to(torch.int32), sc, rc)
        Rr = q.shape[0]
        yr = torch.zeros(Rr, H, dtype=torch.float32, device=ids.device)
        if Rr:
            L = ex.layout
            tc = Rr >= self.tc_min_t and H % 128 == 0 and L.I % 128 == 0
            y2, pos = (self._moe_tc(q, sq, lid.view(-1, 1), ex, Rr, Rr, ep.E_loc, -1) if tc else
                       self._moe_gemv(q, sq, lid.view(-1, 1), ex, Rr, MB, None, ep.E_loc, -1))
            one = torch.ones(Rr, 1, dtype=torch.float32, device=ids.device)
            C.moe_combine(y2, pos, one, None, None, None, yr)
        back = a2a(yr, rc, sc)
        res = torch.empty(T * k, H, dtype=torch.float32, device=ids.device)
        res[order] = back
        return res

    def set_sp_group(self, group):
        """Sequence-parallel prefill over `group` (every rank holds the whole model): a long
        prompt is split into block-aligned chunks, rank r runs chunk r through every layer,
        and before each layer's attention (and the DSA indexer's scores) the ranks all-gather
        their chunks' blocks of that layer's paged caches, so chunk r attends to every earlier
        position.  Afterwards every rank holds the prompt's full caches and decodes it
        (replicated, deterministic)."""
        self.sp_group = group

    def set_dcp_group(self, group, interleave: int = 1):
        """Decode context parallelism over `group` (replicated weights): position p's latent
        cache row lives only on rank (p // interleave) % W.  Prefill computes every row on
        every rank and writes the owned ones; a decode-sized attention runs the split-KV
        kernel over the rank's own rows, all-gathers the (partial output, max, sum) splits of
        every rank and merges them in one fixed order (so every rank emits the same tokens)."""
        import torch.distributed as dist
        if self.cfg.index_heads:
            raise NotImplementedError("GPU DCP: dense MLA attention only (no DSA indexer)")
        W = dist.get_world_size(group)
        if W > 32:
            raise ValueError("GPU DCP: at most 32 ranks (one merge warp)")
        self.dcp = (group, W, dist.get_rank(group), int(interleave))

    def _slots(self, bt, seq, pos):
        """Cache slots of (row, position) pairs (DCP: this rank's, -1 elsewhere)."""
        seq, pos = seq.long(), pos.long()
        if self.dcp is None:
            return bt[seq, pos // KV_BLOCK].long() * KV_BLOCK + pos % KV_BLOCK
        _, W, r, I = self.dcp
        return dcp_slots(bt, seq, pos, W, r, I)

    def _lpos(self, pos):
        """DCP: per row, the local index of the last key it sees (None without DCP)."""
        if self.dcp is None:
            return None
        _, W, r, I = self.dcp
        return (dcp_local_count(pos.long() + 1, W, r, I) - 1).int()

    def sp_chunk(self, n: int):
        """-> (chunk length, block-aligned) of an n-token prompt over the SP group, or None
        when some rank would get no token (a short prompt prefills replicated)."""
        import torch.distributed as dist
        W = dist.get_world_size(self.sp_group)
        Tc = -(-(-(-n // W)) // KV_BLOCK) * KV_BLOCK
        return Tc if (W - 1) * Tc < n else None

    def prefill_sp(self, prompt: list, block_table: list, row: int, state):
        """Sequence-parallel prefill of one prompt into decode-state row `row` -> first token
        (the same on every rank).  Rank r computes positions [r * Tc, min(n, (r + 1) * Tc)):
        a non-final chunk as `prefill_chunk`, the rank holding the last position as the final
        chunk (head, first token, MTP drafts); that rank then broadcasts the row's state."""
        import torch.distributed as dist
        G = self.sp_group
        W, r = dist.get_world_size(G), dist.get_rank(G)
        n = len(prompt)
        Tc = self.sp_chunk(n)
        assert Tc is not None, "sp prefill: prompt too short for the group"
        nb = Tc // KV_BLOCK
        bt = torch.tensor(block_table, dtype=torch.long)
        blocks = torch.stack([bt[q * nb:(q + 1) * nb] for q in range(W)]).to(self.dev)
        self._sp = (G, W, r, blocks)
        lo, hi = r * Tc, min(n, (r + 1) * Tc)
        owner = (n - 1) // Tc
        try:
            if r == owner:
                first = self.prefill([prompt], [block_table], [row], state, starts=[lo] if lo else None)
            else:
                self.prefill_chunk(prompt, block_table, lo, hi)
        finally:
            self._sp = None
        src = dist.get_global_rank(G, owner)
        rows = torch.tensor([row], device=self.dev)
        tok, pos = state.tokens[rows].contiguous(), state.seq_pos[rows].contiguous()
        dist.broadcast(tok, src=src, group=G)
        dist.broadcast(pos, src=src, group=G)
        state.tokens[rows] = tok
        state.seq_pos[rows] = pos
        return int(tok[0, 0])

    def _sp_gather(self, caches, li):
        """All-gather of layer li's cache blocks of every rank's SP chunk (a no-op outside an
        SP prefill; callers skip decode-mode passes, e.g. the owner's MTP draft chain).  Block
        ids are the same on every rank (one block table)."""
        if self._sp is None or li >= len(caches) or caches[li] is None:
            return
        import torch.distributed as dist
        G, W, r, blocks = self._sp
        cache = caches[li]
        mine = cache.index_select(0, blocks[r]).contiguous()
        out = torch.empty((W,) + tuple(mine.shape), dtype=mine.dtype, device=mine.device)
        dist.all_gather_into_tensor(out, mine, group=G)
        for q in range(W):
            if q != r:
                cache.index_copy_(0, blocks[q], out[q])

    def attach_expert_cache(self, cache):
        """Serve routed experts through `cache` (pools already rewired by
        residency.build_expert_cache).  Kernels count misses into cache.miss_count;
        every MoE layer keeps its own routing buffer so misses can be fetched."""
        from ..residency import moe_layers
        self.cache = cache
        self.miss = cache.miss_count
        self._moe_index = {id(lw): i for i, lw in enumerate(moe_layers(self.mw))}

    def enable_looka(self, K: int, pilot: bool, max_rows: int):
        """Router lookahead in the decode graph (expert cache attached): at every main-stack
        MoE layer L, layer L + 1's router on L's MoE input predicts L + 1's top-K experts
        (the model's own top-k selection with K picks).  Recall counters score them against
        the routing L + 1 then does, and the previous step's routing of the same layer as
        the baseline predictor; with ``pilot`` the predictions also go to ``pilot_log``
        [layers, max_rows, K] for the host prefetcher.  (Reference: LOOKA / PILOT, patch
        P:11740-11940.)"""
        from ..residency import moe_layers
        layers = moe_layers(self.mw)
        n_main = sum(1 for lw in self.mw.layers if lw.is_moe)
        k = self.cfg.top_k
        self._looka = dict(K=int(K), layers=layers, n_main=n_main, rows=int(max_rows))
        self.looka_hits = torch.zeros(2, dtype=torch.int64, device=self.dev)
        self.looka_tot = torch.zeros(2, dtype=torch.int64, device=self.dev)
        self._looka_prev = [torch.full((max_rows, k), -1, dtype=torch.int32, device=self.dev) for _ in range(n_main)]
        self._looka_pred = torch.full((max_rows, int(K)), -1, dtype=torch.int32, device=self.dev)
        self.pilot_log = (torch.full((n_main, max_rows, int(K)), -1, dtype=torch.int32, device=self.dev)
                          if pilot else None)

    def looka_recall(self) -> dict:
        """Recall of the two predictors so far: the previous step's routing of the same
        layer, and the router lookahead."""
        h, t = self.looka_hits.tolist(), self.looka_tot.tolist()
        return {"previous_step": h[0] / max(1, t[0]), "router_lookahead": h[1] / max(1, t[1]),
                "routed": t[0]}

    def _looka_step(self, mli, hb, ids, ctx):
        """In-graph lookahead bookkeeping at main-stack MoE layer `mli` of a decode pass."""
        L = self._looka
        if L is None or mli is None or ctx.mode != "decode" or self._route_tag or mli >= L["n_main"]:
            return
        T, k = ids.shape
        if T > L["rows"]:
            return
        prev = self._looka_prev[mli][:T]
        self.looka_hits[0] += (ids.unsqueeze(2) == prev.unsqueeze(1)).any(dim=2).sum()
        self.looka_tot[0] += T * k
        prev.copy_(ids)
        pred = self._looka_pred[:T]
        if mli > 0:
            self.looka_hits[1] += (ids.unsqueeze(2) == pred.unsqueeze(1)).any(dim=2).sum()
            self.looka_tot[1] += T * k
        if mli + 1 < L["n_main"]:
            cfg, nxt, K = self.cfg, L["layers"][mli + 1], L["K"]
            lg = self.ws.get("looka.logits", (T, cfg.num_experts), torch.float32)
            self._router_logits(hb, nxt, lg)
            pid = self.ws.get("looka.ids", (T, K), torch.int32)
            pw = self.ws.get("looka.w", (T, K), torch.float32)
            self.C.router_topk(lg, nxt.router_bias, K, cfg.router == "sigmoid", cfg.n_group, cfg.topk_group,
                               cfg.norm_topk_prob, cfg.routed_scaling, pid, pw)
            pred.copy_(pid)
            if self.pilot_log is not None:
                self.pilot_log[mli + 1, :T].copy_(pid)

    def attach_trellis(self, tier, delta=None):
        """Serve the routed experts of the tier's layers from trellis-coded weights (one rank,
        no expert cache / delta tier): the router as usual, then the tier's rotation +
        trellis-decode kernels per routing pair, then the usual expert combine.  Fixed shapes
        and no host synchronisation, so the step stays capturable."""
        self.trellis, self.trellis_delta = tier, delta
        self._trellis_li = {id(lw): li for li, lw in enumerate(self.mw.layers) if li in tier.layers}

    def attach_delta_tier(self, tier):
        """Serve experts that hold a delta slot at FP4 precision (decode GEMVs)."""
        from ..residency import moe_layers
        self.delta = tier
        if not self._moe_index:
            self._moe_index = {id(lw): i for i, lw in enumerate(moe_layers(self.mw))}

    def main_hidden(self, B: int):
        """Final normed hidden states [B*(1+k), H] of bucket B's last decode step (None where
        this rank has no head)."""
        b = self._bucket_ws(B).bufs.get(("main.hid", torch.bfloat16))
        if b is None:
            return None
        H = self.cfg.hidden
        return b[: B * (self.k + 1) * H].view(B * (self.k + 1), H)

    def main_logits(self, B: int):
        """Logits [B*(1+k), V] of the last decode step of bucket B (verify rows, row i*(k+1)+j);
        None where this rank has no head (PP stages before the last).  V is this rank's
        vocab shard under TP."""
        b = self._bucket_ws(B).bufs.get(("main.logits", torch.float32))
        if b is None or getattr(self.mw, "lm_head", None) is None:
            return None
        V = self.mw.lm_head.w.shape[0]
        return b[: B * (self.k + 1) * V].view(B * (self.k + 1), V)

    def route_ids(self, B: int):
        """Per-MoE-layer routed expert ids of the last decode step of bucket B (the MTP layer's
        draft passes concatenated)."""
        ws = self._bucket_ws(B)
        out = []
        for i in range(len(self._moe_index)):
            parts = [ws.bufs.get((f"topk_ids.{i}", torch.int32))]
            parts += [ws.bufs.get((f"topk_ids.{i}.p{j}", torch.int32)) for j in range(1, max(self.k, 1))]
            parts = [t.reshape(-1) for t in parts if t is not None]
            out.append(torch.cat(parts) if len(parts) > 1 else (parts[0] if parts else None))
        return out

    def route_weights(self, B: int):
        """The routing weights matching ``route_ids`` entry for entry."""
        ws = self._bucket_ws(B)
        out = []
        for i in range(len(self._moe_index)):
            parts = [ws.bufs.get((f"topk_w.{i}", torch.float32))]
            parts += [ws.bufs.get((f"topk_w.{i}.p{j}", torch.float32)) for j in range(1, max(self.k, 1))]
            parts = [t.reshape(-1) for t in parts if t is not None]
            out.append(torch.cat(parts) if len(parts) > 1 else (parts[0] if parts else None))
        return out

    def _ensure_experts(self, li, ids, mode: str = "decode"):
        """Eager passes (prefill, un-captured decode): fetch this layer's routed experts now.
        With VLLM_MOE_W2_PREFILL_FP4=ensure an eager prefill chunk also makes its routed
        experts resident in the FP4 delta tier first, so every prefill pair is served at FP4
        (the pool needs one layer's chunk working set; a larger set keeps the hottest)."""
        if li is None or torch.cuda.is_current_stream_capturing():
            return
        es = None
        if self.cache is not None:
            es = torch.unique(ids).tolist()
            self.cache.ensure_resident(li, es)
        if (self.delta is not None and mode in ("prefill", "cached")
                and self.ecfg.moet.prefill_fp4 == "ensure"):
            es = es if es is not None else torch.unique(ids).tolist()
            cap = self.delta.n_slots
            if len(es) > cap:               # keep the most-routed experts of the chunk
                cnt = torch.bincount(ids.reshape(-1).long(), minlength=max(es) + 1)
                es = sorted(es, key=lambda e: -int(cnt[e]))[:cap]
            self.delta.ensure_resident(li, es)

    def set_pp_group(self, group):
        """Join a pipeline group: stage activations travel by NCCL send/recv and
        the last stage broadcasts each step's accepted tokens, drafts and
        positions to every stage."""
        self.pp_group = group

    def _pp_peer(self, r):
        return torch.distributed.get_global_rank(self.pp_group, r)

    def _pp_broadcast_state(self, st, rows=None):
        """Last stage -> all stages: the decode state every stage needs for the next step."""
        if self.pp_group is None or self.pp_size == 1:
            return
        src = self._pp_peer(self.pp_size - 1)
        for t in (st.tokens, st.seq_pos, st.out_tokens, st.n_acc):
            torch.distributed.broadcast(t, src=src, group=self.pp_group)

    def _materialize(self, x):
        """Complete a pending fused all-reduce / residual add into x (no norm outputs)."""
        if self._pend_add is not None:
            x0, part, xout = self._pend_add
            self._pend_add = None
            torch.add(x0, part, out=xout)
        if self._pend is not None:
            resid, xout = self._pend
            self._pend = None
            ones = self.ws.get("pp.ones", (self.cfg.hidden,), torch.bfloat16)
            ones.fill_(1.0)
            self.C.rmsnorm_quant(resid, None, xout, ones, self.cfg.rms_eps, None, None, None, None, None, 0,
                                 self.ar.desc)
        return x

    def _tp_allreduce(self, t):
        if self.tp_group is not None:
            torch.distributed.all_reduce(t, group=self.tp_group)

    def _norm_in(self, x, w, y_out=None, q0=None, s0=None, q1=None, s1=None, ostride=0):
        """RMSNorm + quant of a sublayer input; completes a pending fused
        all-reduce first (x = residual + sum of the ranks' partials, written to x)."""
        pend, self._pend = self._pend, None
        padd, self._pend_add = self._pend_add, None
        if padd is not None:      # x = residual + all-reduced partial, then the norm (one kernel)
            x0, part, xout = padd
            self.C.rmsnorm_quant(x0, part, xout, w, self.cfg.rms_eps, y_out, q0, s0, q1, s1, ostride)
        elif pend is not None:
            resid, xout = pend
            assert xout.data_ptr() == x.data_ptr()
            self.C.rmsnorm_quant(resid, None, xout, w, self.cfg.rms_eps, y_out, q0, s0, q1, s1, ostride, self.ar.desc)
        else:
            self.C.rmsnorm_quant(x, None, None, w, self.cfg.rms_eps, y_out, q0, s0, q1, s1, ostride)

    def _row_parallel_out(self, aq, as_, lin, x, out, T):
        """out = x + all-reduce(aq @ lin^T) for a row-parallel linear."""
        if self.tp_group is None:
            self._gemv(aq, as_, lin, out, x)
        elif self._fused:
            K = lin.w.shape[-1]
            if (T <= 8 and self.gemv_stream and lin.w.dim() == 2 and K % 128 == 0 and K <= 5120
                    and aq.stride(0) % 16 == 0):
                self.C.gemv_stream_fp8(aq, as_, lin.w, lin.s, out, None, self.status, ar_push=self.ar.desc)
            else:
                self.C.gemv_fp8(aq, as_, lin.w, lin.s, out, None, self.ar.desc)
            self._pend = (x, out)
        else:
            part = self.ws.get("rp_part", (T, self.cfg.hidden), torch.bfloat16)
            self._gemv(aq, as_, lin, part)
            self._tp_allreduce(part)
            if self._decode:
                self._pend_add = (x, part, out)     # the next norm adds the residual
            else:
                torch.add(x, part, out=out)

    def _fork(self):
        """Start a side branch: work issued under the returned context runs
        concurrently with the main stream (a parallel branch when captured into
        the CUDA graph).  MOET_BRANCHES=0 keeps everything on one stream."""
        if not self.branches:
            import contextlib
            return contextlib.nullcontext()
        self._side.wait_stream(torch.cuda.current_stream())
        return torch.cuda.stream(self._side)

    def _join(self):
        if self.branches:
            torch.cuda.current_stream().wait_stream(self._side)

    # ------------------------------------------------------------------ layer
    def _attention(self, lw: LayerWeights, x, ctx: StepCtx, cache, li, out, resid=None):
        """out = resid + attention(norm(x)); resid defaults to x (a zero buffer under
        hyper-connections, whose streams take the block output)."""
        cfg, C, T, Hh = self.cfg, self.C, ctx.T, self.Hh
        rx = x if resid is None else resid
        H, ql, lat, rope, nope, vd = cfg.hidden, cfg.q_lora_rank, cfg.kv_lora_rank, cfg.qk_rope_dim, cfg.qk_nope_dim, cfg.v_head_dim
        hq, hs = self._fp8("h", T, H)
        qkva = self.ws.get("qkva", (T, ql + lat + rope), torch.bfloat16)
        qaq, qas = self._fp8("qa", T, ql)
        ovq, ovs = self._fp8("ov", T, Hh * vd)
        qb = self.ws.get("qb", (T, Hh * (nope + rope)), torch.bfloat16)
        # decode: the input norms are fused into the streaming GEMVs' prologues (no separate
        # RMSNorm launches); needs no pending TP reduction and no indexer (which reads hq / qa)
        fuse = (ctx.mode == "decode" and T <= 8 and self.gemv_stream and (self._pend is None or self._fused)
                and lw.idx_wq is None and isinstance(lw.qkv_a.w, torch.Tensor) and lw.qkv_a.w.dim() == 2
                and H % 128 == 0 and ql % 128 == 0 and H <= 5120 and ql <= 5120)
        if fuse:
            padd, self._pend_add = self._pend_add, None
            pend, self._pend = self._pend, None
            if pend is not None:     # fused TP all-reduce completed in the prologue: x = resid + sum of partials
                resid, xout = pend
                assert xout.data_ptr() == x.data_ptr() and resid.is_contiguous()
                C.gemv_stream_fp8(None, None, lw.qkv_a.w, lw.qkv_a.s, qkva, None, self.status, resid, lw.attn_norm,
                                  cfg.rms_eps, None, xout, None, self.ar.desc)
            elif padd is not None:     # residual add of a pending TP reduction folded into the prologue
                x0, part, xout = padd
                C.gemv_stream_fp8(None, None, lw.qkv_a.w, lw.qkv_a.s, qkva, None, self.status, x0, lw.attn_norm,
                                  cfg.rms_eps, part, xout)
            else:
                C.gemv_stream_fp8(None, None, lw.qkv_a.w, lw.qkv_a.s, qkva, None, self.status, x, lw.attn_norm,
                                  cfg.rms_eps)
        else:
            self._norm_in(x, lw.attn_norm, None, hq, hs)
            self._gemv(hq, hs, lw.qkv_a, qkva)
        # attention reads the paged latent cache (absorbed) unless this "cached" chunk has
        # key rows to gather for the flash kernel (dense attention, bf16 cache)
        flash_cached = ctx.mode == "cached" and ctx.kv_idx is not None and lw.idx_wq is None and self.kv_mode == 1
        absorbed = ctx.mode == "decode" or (ctx.mode == "cached" and not flash_cached)
        if absorbed:
            with self._fork():     # latent KV path (norm, rope, cache write) beside the query path
                C.kv_prep(qkva[:, ql:], lat, rope, lw.kv_a_norm, cfg.rms_eps, ctx.pos, self.cos_sin, ctx.slot,
                          self.kv_mode, cache, None, None, None, None, self.status)
        if fuse:
            C.gemv_stream_fp8(None, None, lw.q_b.w, lw.q_b.s, qb, None, self.status, qkva[:, :ql], lw.q_a_norm,
                              cfg.rms_eps)
        else:
            C.rmsnorm_quant(qkva[:, :ql], None, None, lw.q_a_norm, cfg.rms_eps, None, qaq, qas, None, None, 0)
            self._gemv(qaq, qas, lw.q_b, qb)
        sel = self._indexer(lw, hq, hs, qaq, qas, ctx, li) if lw.idx_wq is not None else None
        if absorbed:
            qnq = self.ws.get("qn.q", (T, Hh, nope), torch.uint8)
            qns = self.ws.get("qn.s", (T, Hh, nope // 64), torch.uint8)
            qcat = self.ws.get("qcat", (T, Hh, lat + rope), torch.bfloat16)
            C.q_prep(qb, Hh, nope, rope, ctx.pos, self.cos_sin, qnq, qns, qcat, lat, None)
            C.gemv_fp8(qnq.permute(1, 0, 2), qns.permute(1, 0, 2), lw.w_uk_t.w, lw.w_uk_t.s,
                       qcat[:, :, :lat].permute(1, 0, 2), None)
            self._join()
            if ctx.mode != "decode":
                self._sp_gather(self.kv, li)  # SP prefill: the other ranks' chunks of this layer's cache
            S = max(1, min(32, 256 // T))
            if ctx.lpos is not None:
                S = max(1, min(S, 32 // self.dcp[1]))
            opart = self.ws.get("opart", (S, T, Hh, lat), torch.float32)
            mlp = self.ws.get("mlpart", (S, T, Hh, 2), torch.float32)
            C.mla_decode(qcat, cache, ctx.block_table, ctx.seq, ctx.pos if ctx.lpos is None else ctx.lpos, opart,
                         mlp, self.scale, self.status, sel)
            if ctx.lpos is not None:      # DCP: every rank's splits, merged below in rank order
                G, W = self.dcp[0], self.dcp[1]
                oall = self.ws.get("dcp.opart", (W * S, T, Hh, lat), torch.float32)
                mall = self.ws.get("dcp.mlpart", (W * S, T, Hh, 2), torch.float32)
                torch.distributed.all_gather_into_tensor(oall, opart, group=G)
                torch.distributed.all_gather_into_tensor(mall, mlp, group=G)
                opart, mlp = oall, mall
            # split merge + W_uv + e4m3 quantisation in one kernel
            C.mla_combine_uv(opart, mlp, lw.w_uv.w, lw.w_uv.s, ovq, ovs)
        elif flash_cached:
            # a chunk over cached positions: write its rows, then gather every key row of its
            # sequences (cached prefix + the chunk) from the cache, quantise the latents, apply
            # W_kv_b and run the flash kernel with the queries at the end of each key range
            C.kv_prep(qkva[:, ql:], lat, rope, lw.kv_a_norm, cfg.rms_eps, ctx.pos, self.cos_sin, ctx.slot,
                      self.kv_mode, cache, None, None, None, None, self.status)
            self._sp_gather(self.kv, li)      # SP prefill: the other ranks' chunks of this layer's cache
            Nk = ctx.kv_idx.numel()
            rows = self.ws.get("krows", (Nk, BF16_ROW), torch.bfloat16)
            torch.index_select(cache.view(-1, BF16_ROW), 0, ctx.kv_idx, out=rows)
            latq, lats = self._fp8("latk", Nk, lat)
            C.quant_fp8(rows[:, :lat], 0, latq, lats)
            kvb = self.ws.get("kvbk", (Nk, Hh * (nope + vd)), torch.bfloat16)
            self._gemv(latq, lats, lw.kv_b, kvb)
            qf = self.ws.get("qfull", (T, Hh, nope + rope), torch.bfloat16)
            C.q_prep(qb, Hh, nope, rope, ctx.pos, self.cos_sin, None, None, None, 0, qf)
            C.mla_prefill(qf, kvb.view(Nk, Hh, nope + vd), rows[:, lat:lat + rope], ctx.cu_seqlens, ctx.max_len,
                          self.scale, ovq, ovs, None, cu_seqlens_k=ctx.cu_k)
        else:
            latq, lats = self._fp8("lat", T, lat)
            kr = self.ws.get("kr", (T, rope), torch.bfloat16)
            C.kv_prep(qkva[:, ql:], lat, rope, lw.kv_a_norm, cfg.rms_eps, ctx.pos, self.cos_sin, ctx.slot,
                      self.kv_mode, cache, None, kr, latq, lats, self.status)
            self._sp_gather(self.kv, li)      # SP prefill, first chunk: its rows to the other ranks
            kvb = self.ws.get("kvb", (T, Hh * (nope + vd)), torch.bfloat16)
            self._gemv(latq, lats, lw.kv_b, kvb)
            qf = self.ws.get("qfull", (T, Hh, nope + rope), torch.bfloat16)
            C.q_prep(qb, Hh, nope, rope, ctx.pos, self.cos_sin, None, None, None, 0, qf)
            C.mla_prefill(qf, kvb.view(T, Hh, nope + vd), kr, ctx.cu_seqlens, ctx.max_len, self.scale,
                          ovq, ovs, None)
        if getattr(lw, "attn_tp", True):
            self._row_parallel_out(ovq, ovs, lw.o, rx, out, T)
        else:       # replicated attention: the whole o projection, residual added, no reduction
            self._gemv(ovq, ovs, lw.o, out, rx)

    def _indexer(self, lw, hq, hs, qaq, qas, ctx, li):
        """DSA indexer: insert this step's keys, score every cached position
        (head-weighted ReLU dot products), keep the top-k.  Decode returns the
        selection for the sparse MLA decode; prefill only fills the key cache
        (prefill attention is dense and causal)."""
        cfg, C, T = self.cfg, self.C, ctx.T
        Hi, Di = cfg.index_heads, cfg.index_head_dim
        ki = self.ws.get("idx.k", (T, Di), torch.bfloat16)
        self._gemv(hq, hs, lw.idx_wk, ki)
        C.idx_k_write(ki, ctx.slot, self.idx_kv[li], self.status)
        if ctx.mode != "decode":
            self._sp_gather(self.idx_kv, li)  # SP prefill: the other ranks' indexer keys
        if ctx.mode == "prefill":
            return None
        qi = self.ws.get("idx.q", (T, Hi * Di), torch.bfloat16)
        self._gemv(qaq, qas, lw.idx_wq, qi)
        wi = self.ws.get("idx.w", (T, Hi), torch.float32)
        self._gemv(hq, hs, lw.idx_ww, wi)
        S = ctx.block_table.shape[1] * KV_BLOCK
        scores = self.ws.get("idx.scores", (T, S), torch.float32)
        C.indexer_logits(qi.view(T, Hi, Di), wi, self.idx_kv[li], ctx.block_table, ctx.seq, ctx.pos, scores,
                         self.status)
        sel = self.ws.get("idx.sel", (T, cfg.index_topk), torch.int32)
        C.indexer_topk(scores, cfg.index_topk, sel)
        return sel

    def _ffn(self, lw: LayerWeights, x, ctx: StepCtx, out, resid=None):
        """out = resid + ffn(norm(x)); resid defaults to x."""
        cfg, C, T = self.cfg, self.C, ctx.T
        rx = x if resid is None else resid
        H = cfg.hidden
        hb = self.ws.get("hb", (T, H), torch.bfloat16)
        hq, hs = self._fp8("h", T, H)
        if not lw.is_moe:
            self._norm_in(x, lw.ffn_norm, None, hq, hs)
            I2 = lw.gate_up.w.shape[0]
            gu = self.ws.get("gu", (T, I2), torch.float32)
            self._gemv(hq, hs, lw.gate_up, gu)
            aq, as_ = self._fp8("act", T, I2 // 2)
            C.swiglu_quant(gu, 0.0, None, 0, aq, as_)
            self._row_parallel_out(aq, as_, lw.down, rx, out, T)
            return
        h2q, h2s = self._fp8("h2", T, H)
        self._norm_in(x, lw.ffn_norm, hb, hq, hs, h2q, h2s)
        sh = None
        if lw.shared_gate_up is not None:
            with self._fork():     # shared expert beside the router and the routed experts
                Is2 = lw.shared_gate_up.w.shape[0]
                sgu = self.ws.get("sgu", (T, Is2), torch.float32)
                self._gemv(hq, hs, lw.shared_gate_up, sgu)
                sq, ss = self._fp8("sact", T, Is2 // 2)
                C.swiglu_quant(sgu, cfg.swiglu_limit or 0.0, None, 0, sq, ss)
                sh = self.ws.get("sh", (T, H), torch.bfloat16)
                self._gemv(sq, ss, lw.shared_down, sh)
        E, k = cfg.num_experts, cfg.top_k
        logits = self.ws.get("rlogits", (T, E), torch.float32)
        mli = self._moe_index.get(id(lw))
        # per MoE layer (and per MTP draft pass: the MTP layer runs k times a step) its own
        # routing buffer, so the replay engine sees every expert the step routed to
        ids = self.ws.get("topk_ids" if mli is None else f"topk_ids.{mli}{self._route_tag}", (T, k), torch.int32)
        # routing weights per layer / draft pass too (the gate's step_w ranking reads them)
        wts = self.ws.get("topk_w" if mli is None else f"topk_w.{mli}{self._route_tag}", (T, k), torch.float32)
        R = T * k
        ex = lw.experts
        L = ex.layout
        I = L.I
        # expert parallelism: this rank's experts are [e_lo, e_lo + E_loc); other routings are skipped
        ep = ex.n_local is not None
        E_loc = ex.n_local if ep else E
        e_lo = ex.e_lo if ep else -1
        use_tc = ctx.mode in ("prefill", "cached") and H % 128 == 0 and I % 128 == 0 and (2 * I) % 128 == 0
        if use_tc and self.delta is not None and self.ecfg.moet.prefill_fp4 not in ("0", ""):
            # prefill-FP4: experts holding a delta slot are served at FP4 in prefill as in decode;
            # the tcgen05 prefill GEMM reads only the 2-bit base, so the delta-aware GEMV runs
            use_tc = False
        topp = self.ecfg.moet.topp
        if self.ep is not None:
            # DP attention + EP: route over all experts, then the all-to-all around the owners' kernels
            self._router_logits(hb, lw, logits)
            C.router_topk(logits, lw.router_bias, k, cfg.router == "sigmoid", cfg.n_group, cfg.topk_group,
                          cfg.norm_topk_prob, cfg.routed_scaling, ids, wts)
            fused = ctx.mode == "decode" and R <= self.ep.cap and ctx.mb in (8, 16, 32)
            if fused:
                self._moe_ep_decode(h2q, h2s, ids, ex, ctx.mb)
            else:
                yk = self._moe_ep_prefill(h2q, h2s, ids, ex, T, ctx.mb)
            if sh is not None:
                self._join()
            none = self.ws.get("ep.nopos", (0,), torch.int32)
            if fused:
                C.moe_combine(self.ep.ret[:R], none, wts, rx, sh, out, None, None, self.ep.desc)
            else:
                C.moe_combine(yk, none, wts, rx, sh, out, None)
            return
        tl = self._trellis_li.get(id(lw)) if self.trellis is not None else None
        if T <= 64 and not use_tc and H % 1024 == 0 and topp <= 0 and tl is None:
            # decode: logits + top-k + pair list in one launch
            MB = ctx.mb
            P = R // MB + min(E_loc, R)
            rank = self.ws.get("rank", (R,), torch.int32)
            stok = self.ws.get("stok", (R,), torch.int32)
            posof = self.ws.get("posof", (R,), torch.int32)
            pairs = self.ws.get("pairs", (P, 4), torch.int32)
            npairs = self.ws.get("npairs", (1,), torch.int32)
            cnt = self.ws.zeros("route.cnt", (1,), torch.int32)
            C.moe_route_fused(hb, self._router_w(lw), logits, lw.router_bias, k, cfg.router == "sigmoid",
                              cfg.n_group, cfg.topk_group, cfg.norm_topk_prob, cfg.routed_scaling, ids, wts, MB,
                              rank, stok, posof, pairs, npairs, cnt, self.status, max(e_lo, 0), E_loc if ep else 0)
            self._looka_step(mli, hb, ids, ctx)
            self._ensure_experts(mli, ids, ctx.mode)
            y2 = self._moe_gemv_pairs(h2q, h2s, stok, pairs, npairs, ex, R, MB, mli)
        else:
            # bf16 operands, fp32 accumulation; prefill-sized T runs on tensor-core tiles
            self._router_logits(hb, lw, logits)
            C.router_topk(logits, lw.router_bias, k, cfg.router == "sigmoid", cfg.n_group, cfg.topk_group,
                          cfg.norm_topk_prob, cfg.routed_scaling, ids, wts)
            if topp > 0:        # expert top-p pruning: the tail moves to the top-1 expert with weight 0
                from ..models.moe_policy import apply_topp
                pi, pw = apply_topp(ids, wts, topp, self.ecfg.moet.topp_min)
                ids.copy_(pi)
                wts.copy_(pw)
            self._looka_step(mli, hb, ids, ctx)
            self._ensure_experts(mli, ids, ctx.mode)
            if tl is not None:      # trellis base tier: per-pair outputs, combined below
                y2 = self.trellis.forward_pairs(tl, hb, ids, delta=self.trellis_delta)
                posof = self.ws.get("trellis.nopos", (0,), torch.int32)
            elif use_tc:
                y2, posof = self._moe_tc(h2q, h2s, ids, ex, R, T, E_loc, e_lo)
            elif (self.decode_tc_nt and ctx.mode == "decode" and H % 128 == 0 and I % 128 == 0
                  and self.delta is None):
                y2, posof = self._moe_tc(h2q, h2s, ids, ex, R, T, E_loc, e_lo, MB=self.decode_tc_nt)
            else:
                y2, posof = self._moe_gemv(h2q, h2s, ids, ex, R, ctx.mb, mli, E_loc, e_lo)
        if sh is not None:
            self._join()
        if self.tp_group is None:
            C.moe_combine(y2, posof, wts, rx, sh, out, None)
        elif self._fused:
            C.moe_combine(y2, posof, wts, None, sh, None, None, self.ar.desc)
            self._pend = (rx, out)
        else:
            part = self.ws.get("moe_part", (T, H), torch.bfloat16)
            C.moe_combine(y2, posof, wts, None, sh, part, None)
            self._tp_allreduce(part)
            if self._decode:
                self._pend_add = (rx, part, out)
            else:
                torch.add(rx, part, out=out)

    def _moe_tc(self, h2q, h2s, ids, ex, R, T, E=None, e_lo=-1, MB=128):
        """Prefill experts on tensor cores: 128-row expert-aligned pairs, activations
        gathered into expert order, two warp-specialized tcgen05 GEMMs."""
        C, cfg = self.C, self.cfg
        E, H = E or cfg.num_experts, cfg.hidden
        L = ex.layout
        I = L.I
        P = R // MB + min(E, R)
        Rp = P * MB
        rank = self.ws.get("rank", (R,), torch.int32)
        stok = self.ws.get("stok_p", (Rp,), torch.int32)
        posof = self.ws.get("posof", (R,), torch.int32)
        pairs = self.ws.get("pairs", (P, 4), torch.int32)
        npairs = self.ws.get("npairs", (1,), torch.int32)
        nrows = self.ws.get("nrows", (1,), torch.int32)
        C.build_pairs_padded(ids, E, MB, rank, stok, posof, pairs, npairs, nrows, self.status, e_lo)
        xq = self.ws.get("xs.q", (Rp, H), torch.uint8)
        xs = self.ws.get("xs.s", (Rp, H // 64), torch.uint8)
        C.gather_rows(h2q, h2s, stok, nrows, xq, xs)
        c13 = self.ws.get("c13", (Rp, 2 * I), torch.float32)
        C.ws_moe_w2(xq, xs, pairs, npairs, ex.pool, L.off_codes13, L.off_sc13, ex.slot_table, c13, 2 * I, H, MB,
                    self.miss, self.status, None)
        a2q = self.ws.get("a2p.q", (Rp, I), torch.uint8)
        a2s = self.ws.get("a2p.s", (Rp, I // 64), torch.uint8)
        C.swiglu_quant(c13, cfg.swiglu_limit or 0.0, nrows, 1, a2q, a2s)
        y2 = self.ws.get("y2", (Rp, H), torch.float32)
        C.ws_moe_w2(a2q, a2s, pairs, npairs, ex.pool, L.off_codes2, L.off_sc2, ex.slot_table, y2, H, I, MB,
                    self.miss, self.status, None)
        return y2, posof

    def _moe_gemv(self, h2q, h2s, ids, ex, R, MB, mli=None, E=None, e_lo=-1):
        """Decode experts: mma.sync weight-streaming GEMV over the compact pair list."""
        C, cfg = self.C, self.cfg
        E, H = E or cfg.num_experts, cfg.hidden
        L = ex.layout
        I = L.I
        P = R // MB + min(E, R)
        rank = self.ws.get("rank", (R,), torch.int32)
        stok = self.ws.get("stok", (R,), torch.int32)
        posof = self.ws.get("posof", (R,), torch.int32)
        pairs = self.ws.get("pairs", (P, 4), torch.int32)
        npairs = self.ws.get("npairs", (1,), torch.int32)
        C.build_pairs(ids, E, MB, rank, stok, posof, pairs, npairs, self.status, e_lo)
        return self._moe_gemv_pairs(h2q, h2s, stok, pairs, npairs, ex, R, MB, mli), posof

    def _moe_gemv_pairs(self, h2q, h2s, stok, pairs, npairs, ex, R, MB, mli=None):
        C, cfg = self.C, self.cfg
        H = cfg.hidden
        L = ex.layout
        I = L.I
        d13 = d2 = {}
        if self.delta is not None and mli is not None:    # FP4 delta slots first, 2-bit base otherwise
            o13, os13, o2, os2 = self.delta.offsets
            t8 = self.delta.slot_table[mli]
            q = bool(getattr(self.delta, "split", False))
            d13 = dict(pool8=self.delta.pool, codes_off8=o13, scale_off8=os13, slot_table8=t8, quintal=q)
            d2 = dict(pool8=self.delta.pool, codes_off8=o2, scale_off8=os2, slot_table8=t8, quintal=q)
        if not d13 and self.w2_decode == "tcd" and MB in (8, 16):
            # base-only experts: K-sliced outputs [slices, rows, N]; the consumers add the slices in order
            def gemv(a, sa, gather, off_c, off_s, N, K, name):
                if K % 128:                                      # the tcgen05 kernel streams 128-k stages
                    o = self.ws.get(name + ".l", (R, N), torch.float32)
                    C.moe_w2_gemv(a, sa, gather, pairs, npairs, ex.pool, off_c, off_s, ex.slot_table, o, N, K, MB,
                                  self.miss)
                    return o
                ks = -(-(K // 128) // self.w2_tcd_spt)
                o = self.ws.get(name, (ks, R, N), torch.float32)
                C.moe_w2_tcd(a, sa, gather, pairs, npairs, ex.pool, off_c, off_s, ex.slot_table, o, N, K, MB,
                             self.miss, self.status)
                return o
            c13 = gemv(h2q, h2s, stok, L.off_codes13, L.off_sc13, 2 * I, H, "c13s")
            a2q, a2s = self._fp8("a2", R, I)
            C.swiglu_quant(c13, cfg.swiglu_limit or 0.0, None, 1, a2q, a2s)
            return gemv(a2q, a2s, None, L.off_codes2, L.off_sc2, H, I, "y2s")
        P = pairs.shape[0]
        ks13, ks2 = self._w2_ksplit(2 * I, H, min(P, R)), self._w2_ksplit(H, I, min(P, R))
        c13 = self.ws.get("c13", (ks13, R, 2 * I), torch.float32)
        C.moe_w2_gemv(h2q, h2s, stok, pairs, npairs, ex.pool, L.off_codes13, L.off_sc13, ex.slot_table, c13,
                      2 * I, H, MB, self.miss, **d13)
        a2q, a2s = self._fp8("a2", R, I)
        C.swiglu_quant(c13, cfg.swiglu_limit or 0.0, None, 1, a2q, a2s)
        y2 = self.ws.get("y2", (ks2, R, H), torch.float32)
        C.moe_w2_gemv(a2q, a2s, None, pairs, npairs, ex.pool, L.off_codes2, L.off_sc2, ex.slot_table, y2,
                      H, I, MB, self.miss, **d2)
        return y2

    def _w2_ksplit(self, N: int, K: int, pairs: int) -> int:
        """K slices of a decode expert GEMV when its grid holds less than one wave of resident
        warps (16-row blocks x pairs < 148 SMs x 32): small expert shards (TP) otherwise leave
        each warp a long serial K loop on a nearly empty GPU.  At least 4 64-k chunks per
        slice.  Measured on the DS4 shape: rank 0's TP8 decode step (no collectives) 3.99 ->
        3.77 ms; one GPU (already one wave) keeps a single slice, where splitting cost ~3 us
        per expert GEMV plus the consumers' slice sums."""
        if not self.w2_ksplit:
            return 1
        warps = max(1, (N // 16) * max(pairs, 1))
        want = (148 * 32) // warps
        return max(1, min(want, (K // 64) // 4, 16))

    def _check(self, name, t):
        """Debug aid (MOET_DEBUG_FINITE=1, eager only): raise at the first non-finite stage output."""
        if self.debug_finite and self._pend is None and self._pend_add is None and not torch.cuda.is_current_stream_capturing():
            bad = ~torch.isfinite(t.float())
            if bool(bad.any()):
                rows = bad.view(t.shape[0], -1).any(-1).nonzero().flatten()[:8].tolist()
                raise FloatingPointError(f"non-finite values after {name}: shape {tuple(t.shape)}, rows {rows}")

    # ------------------------------------------------------------------ draft module
    def _init_draft_module(self, mw):
        """The module the decode step drafts with: the MTP module, or an EAGLE-3 module
        (``mw.extra["eagle3"]``) seen through the same fields -- its input projection plays
        eh_proj, its norm the head norm -- plus ``fc`` over the target's aux hidden states
        (the residual after each target layer, concatenated).  FP8 copies of its BF16
        projections serve the FP8 GEMV / GEMM kernels."""
        import types
        from ..models.weights import Fp8Linear
        self.eagle = mw.extra.get("eagle3")
        if self.eagle is None:
            self._draft = mw.mtp
            return
        ew = self.eagle

        def fp8(lin):
            return lin if isinstance(lin, Fp8Linear) else Fp8Linear.from_float(lin.dequant().to(self.dev))
        self._eagle_fc = fp8(ew.fc)
        self._eagle_layers = {li: j for j, li in enumerate(ew.target_layers)}
        self._draft = types.SimpleNamespace(enorm=ew.enorm, hnorm=ew.hnorm, eh_proj=fp8(ew.in_proj), layer=ew.layer,
                                            head_norm=ew.norm, hc_head=None)

    def _eagle_aux(self, T):
        """The target's aux hidden states [T, n H] of the last main pass (EAGLE-3)."""
        return self.ws.get("eagle.aux", (T, len(self._eagle_layers) * self.cfg.hidden), torch.bfloat16)

    def _draft_input(self, hid, T):
        """What the first draft pass reads: the final normed hidden (MTP) or the aux states."""
        return self._eagle_aux(T) if self.eagle is not None else hid

    # ------------------------------------------------------------------ hyper-connections
    def _init_hyper_connections(self):
        """hc_mult > 1 (DeepSeek-V4 mHC): the residual is n f32 streams per token; every
        site's mixing weights as f32 device tensors, and the MTP module's eh_proj split into
        its embedding and hidden halves (the hidden half projects each stream)."""
        self.hcn = self.cfg.hc_mult
        self._hc = {}
        self._hc_pend = None      # (block output, post, comb) the next site's hc_mix applies
        if self.hcn <= 1:
            return
        H = self.cfg.hidden
        if H % 128:
            raise NotImplementedError("hyper-connections on the GPU: hidden % 128")
        sites = []
        for lw in self.mw.layers:
            sites += [lw.hc_attn, lw.hc_ffn]
        if self.mw.extra.get("hc_head") is not None:
            sites.append(self.mw.extra["hc_head"])
        m = self.mw.mtp
        if m is not None:
            sites += [m.layer.hc_attn, m.layer.hc_ffn, m.hc_head]
            self._eh_e, self._eh_h = (_split_cols(m.eh_proj, 0, H), _split_cols(m.eh_proj, H, 2 * H))
        for hc in sites:
            if hc is None:
                raise ValueError("hyper-connections: a site without mixing weights")
            self._hc[id(hc)] = tuple(t.to(self.dev, torch.float32).contiguous() for t in (hc.fn, hc.base, hc.scale))

    def _hc_site(self, xs, hc, T):
        """One site: the pending block update (if any) and the partial mixes in one kernel,
        then the mixes and the block input h (bf16 [T, H])."""
        n, H, cfg = self.hcn, self.cfg.hidden, self.cfg
        fn, base, scale = self._hc[id(hc)]
        R = fn.shape[0]
        part = self.ws.get("hc.part", (H // 128, T, R + 1), torch.float32)
        h = self.ws.get("hc.h", (T, H), torch.bfloat16)
        post = self.ws.get("hc.post", (T, n), torch.float32)
        comb = self.ws.get("hc.comb", (T, n, n), torch.float32)
        upd, self._hc_pend = self._hc_pend, None
        if upd is not None:
            self.C.hc_mix(xs, upd[0], upd[1], upd[2], fn, part)
        else:
            self.C.hc_mix(xs, None, None, None, fn, part)
        block = R != n
        self.C.hc_apply(xs, part, base, scale, cfg.hc_eps, cfg.hc_sinkhorn_iters, cfg.rms_eps, h,
                        post if block else None, comb if block else None)
        return h

    def _hc_flush(self, xs):
        """Apply the last block's pending update to the streams."""
        upd, self._hc_pend = self._hc_pend, None
        if upd is not None:
            self.C.hc_mix(xs, upd[0], upd[1], upd[2])

    def _layer_hc(self, lw, xs, ctx, cache, li):
        """A decoder layer over the streams xs [T, n, H] (updated in place): each block reads
        its site's h and adds nothing itself (zero residual); the streams take its output
        through the next site's hc_mix."""
        T, H = ctx.T, self.cfg.hidden
        self._fused = False       # no deferred residual adds: every block output is complete
        self._decode = False
        zero = self.ws.get("hc.zero", (T, H), torch.bfloat16)
        zero.zero_()
        timed = self.timers is not None and ctx.mode in ("prefill", "cached")
        h = self._hc_site(xs, lw.hc_attn, T)
        a = self.ws.get("x_mid", (T, H), torch.bfloat16)
        with self.timers.span("prefill.attention") if timed else contextlib.nullcontext():
            self._attention(lw, h, ctx, cache, li, a, resid=zero)
        self._check(f"attention[{li}] ({ctx.mode})", a)
        self._hc_pend = (a, self.ws.get("hc.post", (T, self.hcn), torch.float32),
                         self.ws.get("hc.comb", (T, self.hcn, self.hcn), torch.float32))
        h = self._hc_site(xs, lw.hc_ffn, T)
        f = self.ws.get("hc.f", (T, H), torch.bfloat16)
        with (self.timers.span("prefill.moe" if self.cfg.is_moe_layer(li) else "prefill.dense_ffn") if timed
              else contextlib.nullcontext()):
            self._ffn(lw, h, ctx, f, resid=zero)
        self._check(f"ffn[{li}] ({ctx.mode})", f)
        self._hc_pend = (f, self.ws.get("hc.post", (T, self.hcn), torch.float32),
                         self.ws.get("hc.comb", (T, self.hcn, self.hcn), torch.float32))

    def _layer(self, lw, x, ctx, cache, li):
        H = self.cfg.hidden
        self._fused = (self.ar is not None and ctx.mode == "decode" and ctx.T <= self.fused_max_t
                       and self.ar.fits(ctx.T, H))
        self._decode = ctx.mode == "decode"
        x2 = self.ws.get("x_mid", (ctx.T, H), torch.bfloat16)
        timed = self.timers is not None and ctx.mode in ("prefill", "cached")
        with self.timers.span("prefill.attention") if timed else contextlib.nullcontext():
            self._attention(lw, x, ctx, cache, li, x2)
        self._check(f"attention[{li}] ({ctx.mode})", x2)
        x3 = self.ws.get("x_a" if li % 2 == 0 else "x_b", (ctx.T, H), torch.bfloat16)
        with (self.timers.span("prefill.moe" if self.cfg.is_moe_layer(li) else "prefill.dense_ffn") if timed
              else contextlib.nullcontext()):
            self._ffn(lw, x2, ctx, x3)
        self._check(f"ffn[{li}] ({ctx.mode})", x3)
        return x3

    # ------------------------------------------------------------------ model pieces
    def _main(self, tokens, ctx: StepCtx):
        xin = self.ws.get("x_in", (ctx.T, self.cfg.hidden), torch.bfloat16)
        if self.first_stage:
            xin.copy_(torch.nn.functional.embedding(tokens.long(), self.mw.embed))
        else:       # activations of the previous pipeline stage
            torch.distributed.recv(xin, src=self._pp_peer(self.pp_rank - 1), group=self.pp_group)
        x = xin
        if self.hcn > 1:          # n residual streams, each starting as the embedding
            if not (self.first_stage and self.last_stage):
                raise NotImplementedError("hyper-connections: no pipeline stages on the GPU")
            x = self.ws.get("hc.x", (ctx.T, self.hcn, self.cfg.hidden), torch.float32)
            x.copy_(xin[:, None, :].expand(-1, self.hcn, -1))
            for li, lw in enumerate(self.mw.layers):
                self._layer_hc(lw, x, ctx, self.kv[li], li)
            self._hc_flush(x)
            return x
        for li, lw in enumerate(self.mw.layers):
            x = self._layer(lw, x, ctx, self.kv[li], li)
            if self.eagle is not None and li in self._eagle_layers:    # EAGLE-3 aux hidden state
                H, j = self.cfg.hidden, self._eagle_layers[li]
                self._eagle_aux(ctx.T)[:, j * H:(j + 1) * H].copy_(self._materialize(x))
        if not self.last_stage:
            x = self._materialize(x)
            torch.distributed.send(x.contiguous(), dst=self._pp_peer(self.pp_rank + 1), group=self.pp_group)
        return x

    def _final(self, x, rows, tag):
        """final RMSNorm -> (normed hidden bf16 [T,H], logits f32 [T,V])."""
        cfg, C = self.cfg, self.C
        T = x.shape[0]
        streams = None
        if self.hcn > 1:          # x: the streams [T, n, H]; the head's gated sum feeds the norm
            streams = x
            x = self._hc_site(x, self.mw.extra["hc_head"] if tag == "main" else self.mw.mtp.hc_head, T)
        hid = self.ws.get(tag + ".hid", (T, cfg.hidden), torch.bfloat16)
        fq, fs = self._fp8(tag + ".f", T, cfg.hidden)
        self._norm_in(x, self.mw.final_norm if tag == "main" else self._draft.head_norm, hid, fq, fs)
        logits = self.ws.get(tag + ".logits", (T, self.mw.lm_head.w.shape[0]), torch.float32)
        self._gemv(fq, fs, self.mw.lm_head, logits)
        self._check(f"lm_head ({tag})", logits)
        if streams is not None:   # the MTP module reads the pre-head streams [T, n H]
            return streams.reshape(T, -1), logits
        return hid, logits

    def _mtp(self, hidden, next_tokens, ctx: StepCtx, rows=None):
        """MTP module over rows (h_i, token_{i+1}) -> (head-normed hidden, logits)."""
        cfg, C, m = self.cfg, self.C, self._draft
        T, H = ctx.T, cfg.hidden
        table = self.mw.embed if self.mw.embed is not None else self.mw.extra["mtp_embed"]
        emb = torch.nn.functional.embedding(next_tokens.long(), table)
        if self.hcn > 1:
            return self._mtp_hc(hidden, emb, ctx, rows)
        if self.eagle is not None and hidden.shape[-1] != H:     # EAGLE-3: aux states through fc
            K = hidden.shape[-1]
            aq, as_ = self._fp8("e3.aux", T, K)
            C.quant_fp8(hidden, 0, aq, as_)
            hidden = self.ws.get("e3.h", (T, H), torch.bfloat16)
            self._gemv(aq, as_, self._eagle_fc, hidden)
        ehq, ehs = self._fp8("eh", T, 2 * H)
        C.rmsnorm_quant(emb, None, None, m.enorm, cfg.rms_eps, None, ehq, ehs, None, None, 2 * H)
        C.rmsnorm_quant(hidden, None, None, m.hnorm, cfg.rms_eps, None, ehq[:, H:], ehs[:, H // 64:], None, None,
                        2 * H)
        xm = self.ws.get("xm", (T, H), torch.bfloat16)
        self._gemv(ehq, ehs, m.eh_proj, xm)
        self._check("mtp eh_proj", xm)
        x = self._layer(m.layer, xm, ctx, self.kv[-1], len(self.mw.layers))
        if self.eagle is not None:
            x = self._materialize(x)
        if rows is not None:      # only these rows need the head (e.g. the last row of each prompt)
            x = x[rows].contiguous()
        if self.eagle is not None:    # EAGLE-3 chains the draft layer's pre-norm output
            return x, self._final(x, None, "mtp")[1]
        return self._final(x, None, "mtp")

    def _mtp_hc(self, hidden, emb, ctx, rows):
        """The MTP module over streams: hidden [T, n H] (pre-head streams), each stream normed
        and projected by eh_proj's hidden half, plus the normed next-token embedding (zero at
        position 0) through its embedding half; the MTP layer over the streams, the module's
        stream reduction and head norm, the shared head."""
        cfg, C, m, n = self.cfg, self.C, self.mw.mtp, self.hcn
        T, H = ctx.T, cfg.hidden
        emb = emb * (ctx.pos != 0).to(emb.dtype)[:, None]
        eq, es = self._fp8("mhc.e", T, H)
        C.rmsnorm_quant(emb.contiguous(), None, None, m.enorm, cfg.rms_eps, None, eq, es, None, None, 0)
        hb = hidden.reshape(T * n, H).to(torch.bfloat16)
        hq, hs = self._fp8("mhc.h", T * n, H)
        C.rmsnorm_quant(hb, None, None, m.hnorm, cfg.rms_eps, None, hq, hs, None, None, 0)
        ye = self.ws.get("mhc.ye", (T, H), torch.float32)
        self._gemv(eq, es, self._eh_e, ye)
        yh = self.ws.get("mhc.yh", (T * n, H), torch.float32)
        self._gemv(hq, hs, self._eh_h, yh)
        xs = self.ws.get("hc.xm", (T, n, H), torch.float32)
        torch.add(yh.view(T, n, H), ye[:, None, :], out=xs)
        self._check("mtp eh_proj", xs)
        self._layer_hc(m.layer, xs, ctx, self.kv[-1], len(self.mw.layers))
        self._hc_flush(xs)
        if rows is not None:
            xs = xs[rows].contiguous()
        return self._final(xs, None, "mtp")

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    @torch.no_grad()
    def prefill_chunk(self, prompt: list, block_table: list, start: int, end: int):
        """A non-final chunk of a chunked prefill: positions [start, end) of `prompt`
        (end < len(prompt)) through the main layers and the MTP layer, caches written, no
        head.  Every MTP row's next token is a prompt token, so nothing is recomputed
        later; the final chunk is a `prefill` with starts=[end]."""
        assert 0 <= start < end < len(prompt)
        self.ws = self.ws_prefill
        dev, T = self.dev, end - start
        toks = torch.tensor(prompt[start:end], dtype=torch.int32, device=dev)
        pos = torch.arange(start, end, dtype=torch.int32, device=dev)
        seq = torch.zeros(T, dtype=torch.int32, device=dev)
        bt = torch.tensor([block_table], dtype=torch.int32, device=dev)
        slot = bt[0, (pos // KV_BLOCK).long()].long() * KV_BLOCK + (pos % KV_BLOCK).long()
        cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
        ctx = StepCtx(T=T, pos=pos, seq=seq, slot=slot, block_table=bt, mode="cached" if start else "prefill",
                      cu_seqlens=cu, max_len=T, mb=32)
        if start:
            self._key_rows(ctx, [end])
        x = self._main(toks, ctx)
        if self.last_stage and self.k:
            if self.hcn > 1:       # the MTP module reads the streams
                hid_all = x.reshape(T, -1)
            elif self.eagle is not None:
                hid_all = self._eagle_aux(T)
            else:
                hid_all = self.ws.get("pf.hid", (T, self.cfg.hidden), torch.bfloat16)
                self.C.rmsnorm_quant(x, None, None, self.mw.final_norm, self.cfg.rms_eps, hid_all, None, None,
                                     None, None, 0)
            nxt = torch.tensor(prompt[start + 1:end + 1], dtype=torch.int32, device=dev)
            self._mtp(hid_all, nxt, ctx, rows=torch.tensor([T - 1], device=dev))
        self.check_status("prefill chunk")

    def _key_rows(self, ctx: StepCtx, ends: list):
        """Give a "cached" step of at least `cached_flash_min` rows the flash path: the cache
        slots of sequence i's positions [0, ends[i]) and their cu_seqlens (queries are the
        last rows of each range)."""
        if ctx.T < self.cached_flash_min:
            return
        bt = ctx.block_table
        seq = torch.cat([torch.full((n,), i, dtype=torch.long) for i, n in enumerate(ends)]).to(self.dev)
        pos = torch.cat([torch.arange(n, dtype=torch.long) for n in ends]).to(self.dev)
        ctx.kv_idx = bt[seq, pos // KV_BLOCK].long() * KV_BLOCK + pos % KV_BLOCK
        ctx.cu_k = torch.tensor([0] + list(torch.tensor(ends).cumsum(0)), dtype=torch.int32, device=self.dev)

    def copy_block(self, src: int, dst: int):
        """Copy one KV block (every layer's latent cache, the MTP layer's and the indexer's):
        the copy-on-write step of prefix sharing."""
        for t in list(self.kv) + list(getattr(self, "idx_kv", None) or []):
            if t is not None:     # idx_kv holds None for layers without an indexer
                t[dst].copy_(t[src])

    def prefill(self, prompts: list, block_tables: list, seq_rows: list, state, sample: bool = False,
                starts: Optional[list] = None):
        """Prefill whole prompts (one chunk each); fills main + MTP caches and the
        decode state rows `seq_rows` (tokens, positions, drafts).  Returns the
        first generated token of each prompt.  `sample`: the first tokens are drawn with
        the rows' sampling parameters (already set in `state`)."""
        self.ws = self.ws_prefill
        try:
            out = self._prefill(prompts, block_tables, seq_rows, state, sample, starts)
        finally:
            self.ws = self.ws_prefill
        self.check_status("prefill")
        return out

    def check_status(self, where: str):
        code = int(self.status.item())
        if code != 0:
            self.status.zero_()
            names = {1: "index out of range", 2: "bounded wait timed out", 3: "bad size", 4: "non-finite logits"}
            raise RuntimeError(f"device status {code} ({names.get(code, '?')}) during {where}")

    def _prefill(self, prompts, block_tables, seq_rows, state, sample=False, starts=None):
        """`starts[i]` > 0: positions [0, starts[i]) of prompt i are already in its blocks
        (a shared prefix); only the rest runs, in "cached" mode."""
        dev, C = self.dev, self.C
        starts = list(starts) if starts is not None else [0] * len(prompts)
        full = [len(p) for p in prompts]
        lens = [n - s0 for n, s0 in zip(full, starts)]                  # rows computed per prompt
        T = sum(lens)
        toks = torch.tensor([t for p, s0 in zip(prompts, starts) for t in p[s0:]], dtype=torch.int32, device=dev)
        pos = torch.cat([torch.arange(s0, n, dtype=torch.int32) for s0, n in zip(starts, full)]).to(dev)
        seq = torch.cat([torch.full((n,), i, dtype=torch.int32) for i, n in enumerate(lens)]).to(dev)
        bt = torch.tensor(block_tables, dtype=torch.int32, device=dev)
        slot = self._slots(bt, seq, pos)
        cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=dev)
        ctx = StepCtx(T=T, pos=pos, seq=seq, slot=slot, block_table=bt,
                      mode="cached" if any(starts) else "prefill", cu_seqlens=cu, max_len=max(lens), mb=32)
        if any(starts):
            self._key_rows(ctx, full)
        x = self._main(toks, ctx)
        B = len(prompts)
        if not self.last_stage:     # the last stage computes the first tokens and drafts, then broadcasts them
            cur = torch.tensor(full, dtype=torch.int32, device=dev)
            state.set_rows(seq_rows, torch.zeros(B, dtype=torch.int32, device=dev), cur,
                           torch.zeros(B, max(self.k, 1), dtype=torch.int32, device=dev)[:, :self.k] if self.k else None)
            self._pp_broadcast_state(state)
            return state.tokens[torch.tensor(seq_rows, device=dev), 0].clone()
        last = (cu[1:] - 1).long()
        xl = x[last].contiguous()
        hid_last, logits = self._final(xl, None, "main")
        tgt = self.ws.get("pf.tgt", (len(prompts),), torch.int32)
        if sample:
            tgt.copy_(self._sample_first(state, seq_rows, logits, full))
        else:
            self._argmax(logits, tgt)
        if self.k == 0:
            state.set_rows(seq_rows, tgt, torch.tensor(full, dtype=torch.int32, device=dev), None)
            self._pp_broadcast_state(state)
            return tgt
        # full hidden for the MTP pass: final norm over all rows
        if self.hcn > 1:           # the MTP module reads the streams
            hid_all = x.reshape(T, -1)
        elif self.eagle is not None:
            hid_all = self._eagle_aux(T)
        else:
            hid_all = self.ws.get("pf.hid", (T, self.cfg.hidden), torch.bfloat16)
            C.rmsnorm_quant(x, None, None, self.mw.final_norm, self.cfg.rms_eps, hid_all, None, None, None, None, 0)
        nxt = torch.empty_like(toks)
        nxt[:-1] = toks[1:]
        nxt[last] = tgt
        mh, ml = self._mtp(hid_all, nxt, ctx, rows=last)     # head only on the last row of each prompt
        drafts = torch.empty(B, self.k, dtype=torch.int32, device=dev)
        d1 = self.ws.get("pf.d1", (B,), torch.int32)
        self._argmax(ml, d1)
        drafts[:, 0] = d1
        h_prev = mh.clone()
        cur_pos = torch.tensor(full, dtype=torch.int32, device=dev)  # position of the first generated token
        prev_tok = d1
        for j in range(1, self.k):
            p2 = cur_pos + (j - 1)
            s2 = torch.arange(B, dtype=torch.int32, device=dev)
            slot2 = self._slots(bt, s2, p2)
            ctx2 = StepCtx(T=B, pos=p2, seq=s2, slot=slot2, block_table=bt, mode="decode", mb=8, lpos=self._lpos(p2))
            h_prev, lg = self._mtp(h_prev.clone(), prev_tok, ctx2)
            dj = self.ws.get("pf.dj", (B,), torch.int32)
            self._argmax(lg, dj)
            drafts[:, j] = dj
            prev_tok = dj.clone()
        state.set_rows(seq_rows, tgt, cur_pos, drafts)
        self._pp_broadcast_state(state)
        return tgt

    # ------------------------------------------------------------------ decode
    def _bucket_ws(self, B):
        ws = self.ws_decode_by_bucket.get(B)
        if ws is None:
            ws = self.ws_decode_by_bucket[B] = Workspace(self.dev)
        return ws

    def decode_body(self, st, sample: bool = False, draft: bool = True):
        """One MTP decode step over the device state `st` (all tensors static).
        Each batch bucket owns its workspace: a captured graph keeps the
        addresses it was recorded with.  `sample`: verify with speculative sampling
        (the state's per-row temperature / top-k / top-p / min-p / seed) instead of
        greedy matching; rows at temperature 0 stay greedy.  `draft=False`: the step
        without drafts the spec guard switches to (greedy)."""
        prev = self.ws
        self.ws = self._bucket_ws(st.B)
        try:
            if draft or self.k == 0:
                self._decode_body(st, sample)
            else:
                self._decode_body_nodraft(st)
        finally:
            self.ws = prev

    def _decode_body_nodraft(self, st):
        """A greedy decode step without drafts (the spec guard's choice while the expert pool
        is cold): the main model over one row per sequence, no MTP pass, so the step routes
        to the experts of one token per sequence instead of k + 1 plus the drafts'.  The
        sequence advances by one token.  The state's stale drafts are verified -- and mostly
        rejected -- by the next drafting step; the MTP layer's cache is not written for this
        position, which can only lower the acceptance of later drafts, never the output."""
        if self.pp_size > 1:
            raise NotImplementedError("the no-draft decode step runs on one pipeline stage")
        C = self.C
        if self.cache is not None:
            self.miss.zero_()
        B = st.B
        pos = st.seq_pos
        slot = self._slots(st.block_table, st.arange_b, pos)
        slot = torch.where(st.active.bool(), slot, torch.full_like(slot, -1))
        ctx = StepCtx(T=B, pos=pos.int(), seq=st.arange_b, slot=slot, block_table=st.block_table, mode="decode",
                      mb=8, lpos=self._lpos(pos))
        x = self._main(st.tokens[:, 0].contiguous(), ctx)
        _, logits = self._final(x, None, "main")
        am = self.ws.get("dec.am", (B,), torch.int32)
        self._argmax(logits, am)
        st.targets[:, 0].copy_(am)
        st.n_acc.zero_()
        st.out_tokens.fill_(-1)
        st.out_tokens[:, 0].copy_(am)
        C.mtp_finalize(st.targets, st.n_acc, st.drafts, st.tokens, st.seq_pos, st.active)

    def _sample_verify(self, st, logits):
        """Speculative sampling of the verify rows into targets / out_tokens / n_acc (the
        outputs of argmax + mtp_accept), in graph-safe tensor ops."""
        from ..spec.device_sampler import sample_verify
        B, kp1 = st.B, self.k + 1
        logits = self._full_vocab(logits).reshape(B, kp1, -1)
        if st.proc is not None:               # penalties / logit bias, verify row j after drafts[:j]
            logits = self._process(st, logits, st.tokens[:, 1:], None)
        n, tok = sample_verify(logits, st.tokens[:, 1:], st.temperature, st.top_k, st.top_p,
                               st.min_p, st.seed, st.seq_pos)
        n = n * st.active
        st.targets.copy_(tok)
        st.n_acc.copy_(n)
        st.out_tokens.copy_(torch.where(st.arange_kp1[None, :] <= n[:, None], tok, torch.full_like(tok, -1)))

    @staticmethod
    def _process(st, logits, drafts, rows):
        from ..spec.device_sampler import process_batch
        pr = st.proc
        sel = (lambda t: t) if rows is None else (lambda t: t[rows])
        return process_batch(logits, drafts, sel(pr["counts"]), sel(pr["prompt_mask"]), sel(pr["repetition"]),
                             sel(pr["frequency"]), sel(pr["presence"]), sel(pr["bias"]))

    def _sample_first(self, state, seq_rows, logits, lens):
        """First generated tokens drawn with the rows' sampling / processing parameters."""
        from ..spec.device_sampler import sample_verify
        dev = logits.device
        B = len(seq_rows)
        r = torch.tensor(seq_rows, dtype=torch.long, device=dev)
        x = self._full_vocab(logits).reshape(B, 1, -1)
        none = torch.zeros(B, 0, dtype=torch.int32, device=dev)
        if state.proc is not None:
            x = self._process(state, x, none, r)
        _, first = sample_verify(x, none, state.temperature[r], state.top_k[r], state.top_p[r], state.min_p[r],
                                 state.seed[r], torch.tensor(lens, dtype=torch.int32, device=dev) - 1)
        return first[:, 0]

    def _full_vocab(self, logits):
        """Sampling under TP: the vocab shards of every rank, gathered (same rows everywhere)."""
        if self.tp_group is None:
            return logits
        from ..spec.device_sampler import gather_vocab
        # a plain allocation, not a workspace buffer: the sampling graph of a bucket may be
        # captured after its greedy graph froze the bucket's workspace (inside a capture the
        # tensor comes from that graph's own pool)
        return gather_vocab(logits, self.tp_group)

    def _decode_body(self, st, sample: bool = False):
        C, k = self.C, self.k
        if self.cache is not None:
            self.miss.zero_()      # per-step miss count (read by the replay engine after the step)
        B = st.B
        kp1 = k + 1
        T = B * kp1
        pos = (st.seq_pos[:, None] + st.arange_kp1[None, :]).reshape(-1)
        slot = self._slots(st.block_table, st.seq_rows, pos)
        slot = torch.where(st.active_rows, slot, torch.full_like(slot, -1))
        ctx = StepCtx(T=T, pos=pos.int(), seq=st.seq_rows, slot=slot, block_table=st.block_table, mode="decode",
                      mb=8 if T * self.cfg.top_k <= self.mb8_max_r else 16, lpos=self._lpos(pos))
        x = self._main(st.tokens.view(-1), ctx)
        if not self.last_stage:
            self._pp_broadcast_state(st)
            return
        hid, logits = self._final(x, None, "main")
        if sample:
            self._sample_verify(st, logits)
        else:
            self._argmax(logits, st.targets.view(-1))
            C.mtp_accept(st.targets, st.tokens, st.out_tokens, st.n_acc, st.active)
        if k == 0:
            st.seq_pos.add_(st.active)
            st.tokens.copy_(st.targets)
            self._pp_broadcast_state(st)
            return
        # MTP pass 1 over the verify rows: (h_j, target_j) at position p + j
        mh, mlog = self._mtp(self._draft_input(hid, T), st.targets.view(-1), ctx)
        am = self.ws.get("dec.am", (T,), torch.int32)
        self._argmax(mlog, am)
        sel = (st.arange_b * kp1 + st.n_acc).long()
        prev_tok = am[sel]
        st.drafts[:, 0] = prev_tok
        h_prev = mh[sel]
        for j in range(1, k):
            self._route_tag = f".p{j}"
            p2 = st.seq_pos + st.n_acc + j
            slot2 = self._slots(st.block_table, st.arange_b, p2)
            slot2 = torch.where(st.active.bool(), slot2, torch.full_like(slot2, -1))
            ctx2 = StepCtx(T=B, pos=p2.int(), seq=st.arange_b, slot=slot2, block_table=st.block_table,
                           mode="decode", mb=8, lpos=self._lpos(p2))
            h_prev, lg = self._mtp(h_prev, prev_tok, ctx2)
            dj = self.ws.get("dec.dj", (B,), torch.int32)
            self._argmax(lg, dj)
            st.drafts[:, j] = dj
            prev_tok = dj
        self._route_tag = ""
        C.mtp_finalize(st.targets, st.n_acc, st.drafts, st.tokens, st.seq_pos, st.active)
        self._pp_broadcast_state(st)

    def capture(self, st, warm: bool = True, sample: bool = False, draft: bool = True):
        """Capture decode_body for the state's batch bucket (after one eager warm-up);
        the sampling variant is a second graph of the bucket (`sample_graphs`), the
        no-draft step a third (`nodraft_graphs`)."""
        if warm:
            self.decode_body_eager_warm(st, sample, draft)
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s, capture_error_mode="thread_local"):
                self.decode_body(st, sample, draft)
        torch.cuda.current_stream().wait_stream(s)
        (self.sample_graphs if sample else self.graphs if draft else self.nodraft_graphs)[st.B] = g
        self._bucket_ws(st.B).frozen = True
        return g

    def decode_body_eager_warm(self, st, sample: bool = False, draft: bool = True):
        snap = st.snapshot()
        self.decode_body(st, sample, draft)
        st.restore(snap)
        torch.cuda.synchronize()


class DecodeState:
    """Static device tensors of the decode loop for a bucket of B sequences."""

    def __init__(self, B: int, k: int, max_blocks: int, device):
        dev = torch.device(device)
        self.B, self.k = B, k
        kp1 = k + 1
        self.tokens = torch.zeros(B, kp1, dtype=torch.int32, device=dev)
        self.seq_pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.block_table = torch.zeros(B, max_blocks, dtype=torch.int32, device=dev)
        self.active = torch.zeros(B, dtype=torch.int32, device=dev)
        self.targets = torch.zeros(B, kp1, dtype=torch.int32, device=dev)
        self.out_tokens = torch.zeros(B, kp1, dtype=torch.int32, device=dev)
        self.n_acc = torch.zeros(B, dtype=torch.int32, device=dev)
        self.drafts = torch.zeros(B, max(k, 1), dtype=torch.int32, device=dev)
        self.arange_kp1 = torch.arange(kp1, dtype=torch.int32, device=dev)
        self.arange_b = torch.arange(B, dtype=torch.int32, device=dev)
        self.seq_rows = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(kp1)
        self.active_rows = torch.zeros(B * kp1, dtype=torch.bool, device=dev)
        # per-row sampling parameters (temperature 0 = greedy)
        self.temperature = torch.zeros(B, dtype=torch.float32, device=dev)
        self.top_k = torch.zeros(B, dtype=torch.int32, device=dev)
        self.top_p = torch.ones(B, dtype=torch.float32, device=dev)
        self.min_p = torch.zeros(B, dtype=torch.float32, device=dev)
        self.seed = torch.zeros(B, dtype=torch.int64, device=dev)

        self.proc = None      # penalty / logit-bias tensors, allocated by the first request that needs them

    SAMPLING = ("temperature", "top_k", "top_p", "min_p", "seed")

    def ensure_processing(self, vocab: int):
        if self.proc is None:
            dev, B = self.tokens.device, self.B
            self.proc = dict(counts=torch.zeros(B, vocab, dtype=torch.float32, device=dev),
                             prompt_mask=torch.zeros(B, vocab, dtype=torch.bool, device=dev),
                             repetition=torch.ones(B, dtype=torch.float32, device=dev),
                             frequency=torch.zeros(B, dtype=torch.float32, device=dev),
                             presence=torch.zeros(B, dtype=torch.float32, device=dev),
                             bias=torch.zeros(B, vocab, dtype=torch.float32, device=dev))
        return self.proc

    def set_processing(self, row: int, prompt, params):
        """Reset row `row` for a new request: its prompt tokens, penalties and bias."""
        pr, dev = self.proc, self.tokens.device
        V = pr["counts"].shape[1]
        pr["counts"][row].zero_()
        pr["prompt_mask"][row].zero_()
        pr["bias"][row].zero_()
        ids = torch.tensor([t for t in prompt if 0 <= t < V], dtype=torch.long)
        if len(ids):
            pr["prompt_mask"][row, ids.to(dev)] = True
        pr["repetition"][row] = float(params.repetition_penalty)
        pr["frequency"][row] = float(params.frequency_penalty)
        pr["presence"][row] = float(params.presence_penalty)
        if params.logit_bias:
            b = {t: v for t, v in params.logit_bias.items() if 0 <= t < V}
            if b:
                pr["bias"][row, torch.tensor(list(b), dtype=torch.long).to(dev)] = \
                    torch.tensor(list(b.values()), dtype=torch.float32).to(dev)
        if params.allowed_token_ids is not None:     # only these tokens: the rest biased out
            from ..spec.logits_process import allowed_bias
            pr["bias"][row] += allowed_bias(params.allowed_token_ids, V, dev)
        one = [w[0] for w in (params.bad_word_ids or []) if len(w) == 1 and 0 <= w[0] < V]
        if one:                                      # one-token bad words: always banned
            from ..spec.logits_process import DISALLOWED
            pr["bias"][row, torch.tensor(one, dtype=torch.long).to(dev)] += DISALLOWED

    def count_tokens(self, rows, tokens):
        """Generated tokens of the last step (host lists) into the rows' counts."""
        if self.proc is None or not rows:
            return
        dev = self.tokens.device
        r = torch.tensor(rows, dtype=torch.long)
        t = torch.tensor(tokens, dtype=torch.long)
        self.proc["counts"].index_put_((r.to(dev), t.to(dev)), torch.ones(len(rows), device=dev), accumulate=True)

    def set_sampling(self, rows, temperature, top_k, top_p, min_p, seed):
        """Host lists, one entry per row in `rows`."""
        idx = torch.tensor(rows, dtype=torch.long)
        for name, vals in zip(self.SAMPLING, (temperature, top_k, top_p, min_p, seed)):
            t = getattr(self, name)
            t[idx.to(t.device)] = torch.tensor(vals, dtype=t.dtype).to(t.device)

    def set_active(self, mask: torch.Tensor):
        self.active.copy_(mask.to(self.active.dtype))
        self.active_rows.copy_(self.active.bool().repeat_interleave(self.k + 1))

    def set_rows(self, rows, first_tokens, positions, drafts):
        rows_t = torch.tensor(rows, dtype=torch.long, device=self.tokens.device)
        self.tokens[rows_t, 0] = first_tokens.to(torch.int32)
        if drafts is not None:
            self.tokens[rows_t, 1:] = drafts.to(torch.int32)
        self.seq_pos[rows_t] = positions.to(torch.int32)

    def snapshot(self):
        return (self.tokens.clone(), self.seq_pos.clone())

    def restore(self, snap):
        self.tokens.copy_(snap[0])
        self.seq_pos.copy_(snap[1])
