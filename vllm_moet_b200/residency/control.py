"""Per-step control around the expert cache: miss replay, confidence gate,
speculation guard, routing prefetchers and the pool-size floors.

* :class:`ReplayEngine` -- after a decode step, read the device miss counter;
  if any routed expert was missing, agree on the missing set across the TP
  group (MAX of the miss count, union of the per-layer missing bitmaps),
  fetch it on every rank, agree that every rank succeeded (MIN of an ok
  flag -- fail closed), restore the step's input state and replay.  Repeats
  to a fixed point (``strict``: at most ``fp_max`` rounds, then raise;
  ``approximate``: accept a step with <= ``miss_tol`` misses).  Reference:
  base-tier replay, patch P:20976-21120 and ``_promote_consensus``.
* :class:`ConfidenceGate` -- ``max_prob = exp(top1 - logsumexp)`` (or the
  top1-top2 margin) over the verify rows, aggregated by min or a quantile;
  at or below ``tau`` the step's routed experts are force-promoted to the
  higher-precision tier and the step replays (at most ``fp_max`` times).
  Reference: confidence gate, patch P:9871-10029.
* :class:`SpecGuard` -- an EMA of the per-step replay indicator; above 0.6
  it latches draft scheduling off (the cold pool would replay every verify
  batch), below 0.3 it resumes, and it backs off if suppression does not
  warm the pool.  Reference: P:8031-8055, ``kpi_step`` P:9565-9626.
* :class:`LookaheadPrefetcher` -- applies layer L+1's router to layer L's
  MoE input and queues the predicted experts (LOOKA); :class:`DraftAffinity`
  folds a token -> experts table from past routing and prefetches the
  experts of the drafted tokens.  Reference: P:11393-11600.
* floors: :func:`gate_fire_floor`; :func:`.tier.working_set_floor`.
"""
from __future__ import annotations

import collections
import math
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import torch

from .tier import ExpertCache, FetchError


def _tp_reduce(t: torch.Tensor, group, op) -> torch.Tensor:
    if group is None:
        return t
    import torch.distributed as dist
    dist.all_reduce(t, op=op, group=group)
    return t


class ReplayEngine:
    """With ``pp_group`` (pipeline stages, each with its own layers' cache) the miss
    count and the fetch outcome are also agreed over the pipeline, so every stage
    replays the step together (its sends and receives pair up); the missing-expert
    bitmap stays per stage (reference: PP base segment replay, M5 / M9)."""

    def __init__(self, cache: ExpertCache, tp_group=None, mode: str = "strict", fp_max: int = 32,
                 miss_tol: int = 0, comm_device=None, pp_group=None, miss_tol_file: Optional[str] = None,
                 fp_thresh: int = 0, fp_thresh_file: Optional[str] = None):
        if mode not in ("strict", "approximate"):
            raise ValueError(mode)
        from ..utils.tunable import tunable
        self.pp_group = pp_group
        self.cache, self.group, self.mode = cache, tp_group, mode
        self.fp_max = fp_max
        # runtime-tunable from a file (BASE_MISS_TOL_FILE); the accept decision is reduced
        # across the ranks, so ranks that read a new value one step apart still agree
        self._miss_tol = tunable(miss_tol, miss_tol_file, int, check=lambda v: v >= 0)
        # approximate mode: after the mandatory first replay, second-order misses are chased
        # only while at most fp_thresh remain (closing distance); more than that means the
        # working set is moving and the step is kept (FP_THRESH / FP_THRESH_FILE)
        self._fp_thresh = tunable(fp_thresh, fp_thresh_file, int, check=lambda v: v >= 0)
        self.comm_device = comm_device or cache.dev
        self.stats = collections.Counter()

    @property
    def miss_tol(self) -> int:
        from ..utils.tunable import resolve
        return resolve(self._miss_tol)

    @miss_tol.setter
    def miss_tol(self, v: int) -> None:      # a fixed value (replaces a file-backed one)
        self._miss_tol = v

    @property
    def fp_thresh(self) -> int:
        from ..utils.tunable import resolve
        return resolve(self._fp_thresh)

    @fp_thresh.setter
    def fp_thresh(self, v: int) -> None:
        self._fp_thresh = v

    def missing_pairs(self, route_ids: Sequence[Optional[torch.Tensor]]) -> List[Tuple[int, int]]:
        """route_ids[li]: int tensor of routed expert ids of layer li this step (any shape)."""
        bitmap = torch.zeros(self.cache.L, self.cache.E, dtype=torch.int32)
        for li, ids in enumerate(route_ids):
            if ids is None:
                continue
            u = torch.unique(ids.detach().reshape(-1).cpu().long())
            u = u[(u >= 0) & (u < self.cache.E)]
            bitmap[li, u] = 1
        bitmap &= (self.cache.mirror < 0).to(torch.int32)
        if self.group is not None:
            import torch.distributed as dist
            bitmap = _tp_reduce(bitmap.to(self.comm_device), self.group, dist.ReduceOp.MAX).cpu()
        nz = bitmap.nonzero().tolist()
        return [(int(li), int(e)) for li, e in nz]

    def read_misses(self) -> int:
        m = self.cache.miss_count.clone()
        import torch.distributed as dist
        for g in (self.group, self.pp_group):
            if g is not None:
                m = _tp_reduce(m.to(self.comm_device), g, dist.ReduceOp.MAX)
        return int(m.item())

    def fetch_consensus(self, pairs) -> None:
        ok = 1
        try:
            self.cache.promote(pairs)
        except FetchError:
            ok = 0
        if self.group is not None or self.pp_group is not None:
            import torch.distributed as dist
            t = torch.tensor([ok], dtype=torch.int32, device=self.comm_device)
            for g in (self.group, self.pp_group):
                if g is not None:
                    t = _tp_reduce(t, g, dist.ReduceOp.MIN)
            ok = int(t.item())
        if not ok:
            self.stats["fetch_failed"] += 1
            raise FetchError("expert fetch failed on at least one rank (fail closed)")

    def run(self, step: Callable[[], None], restore: Callable[[], None],
            route_ids: Callable[[], Sequence[Optional[torch.Tensor]]]) -> int:
        """Run `step` until it is miss-free.  `restore` puts the step's inputs back
        before a replay.  -> number of replays."""
        for it in range(self.fp_max + 1):
            self.cache.miss_count.zero_()
            step()
            misses = self.read_misses()
            self.stats["steps"] += 1
            accept = misses == 0 or (self.mode == "approximate" and misses <= self.miss_tol)
            if not accept and self.mode == "approximate" and it > 0 and misses > self.fp_thresh:
                self.stats["fp_giveup"] += 1          # second-order residue beyond closing distance
                accept = True
            if accept:
                self.stats["replays"] += it
                self.stats["replayed_steps"] += int(it > 0)
                self.stats["second_order_replays"] += max(it - 1, 0)
                return it
            pairs = self.missing_pairs(route_ids())
            if not pairs:     # counted misses of experts that are resident by now (a concurrent prefetch)
                pairs = []
            self.stats["miss_events"] += 1
            self.fetch_consensus(pairs)
            restore()
        if self.mode == "strict":
            raise RuntimeError(f"expert replay did not converge in {self.fp_max} rounds")
        # approximate: within closing distance and still not converged -- ping-pong between
        # evictions; the step keeps the zeroed contributions of the residue (logged, counted)
        self.stats["fp_unfixed"] += 1
        self.stats["replays"] += self.fp_max
        self.stats["replayed_steps"] += 1
        import logging
        logging.getLogger("vllm_moet_b200").warning(
            "expert replay hit fp_max=%d with misses within fp_thresh=%d remaining (ping-pong); step kept",
            self.fp_max, self.fp_thresh)
        return self.fp_max


class ConfidenceGate:
    def __init__(self, tau: float = 0.6, signal: str = "maxprob", agg: str = "min", fp_max: int = 3,
                 max_promote: int = 64, tau_file: Optional[str] = None, max_promote_file: Optional[str] = None):
        from ..utils.tunable import tunable
        # tau and max_promote are runtime-tunable from files (GATE_TAU_FILE / _MAX_PROMOTE_FILE)
        self._tau = tunable(tau, tau_file, float, check=lambda v: 0.0 <= v <= 1.0)
        self._max_promote = tunable(max_promote, max_promote_file, int, check=lambda v: v >= 0)
        self.signal, self.agg = signal, agg
        self.fp_max = fp_max
        self.stats = collections.Counter()

    @property
    def tau(self) -> float:
        from ..utils.tunable import resolve
        return resolve(self._tau)

    @tau.setter
    def tau(self, v: float) -> None:         # a fixed value (replaces a file-backed one)
        self._tau = v

    @property
    def max_promote(self) -> int:
        from ..utils.tunable import resolve
        return resolve(self._max_promote)

    @max_promote.setter
    def max_promote(self, v: int) -> None:
        self._max_promote = v

    @staticmethod
    def row_stats(logits: torch.Tensor) -> torch.Tensor:
        """logits [R, V] (a full vocab or one rank's vocab shard) -> [R, 3] (top1, top2, lse)."""
        x = logits.float()
        top2 = x.topk(min(2, x.shape[-1]), dim=-1).values
        if top2.shape[-1] < 2:
            top2 = torch.cat([top2, torch.full_like(top2, float("-inf"))], dim=-1)
        return torch.stack([top2[:, 0], top2[:, 1], torch.logsumexp(x, dim=-1)], dim=-1)

    @staticmethod
    def merge_stats(parts: torch.Tensor) -> torch.Tensor:
        """[W, R, 3] per-shard stats -> [R, 3] of the whole vocab (exact: global top-2 from
        every shard's top-2, log-sum-exp of the shards' log-sum-exps)."""
        cand = parts[..., :2].permute(1, 0, 2).reshape(parts.shape[1], -1)   # [R, 2W]
        top2 = cand.topk(2, dim=-1).values
        return torch.stack([top2[:, 0], top2[:, 1], torch.logsumexp(parts[..., 2], dim=0)], dim=-1)

    def score_stats(self, st: torch.Tensor) -> float:
        t1, t2, lse = st[:, 0], st[:, 1], st[:, 2]
        s = torch.exp(t1 - lse) if self.signal == "maxprob" else torch.exp(t1 - lse) - torch.exp(t2 - lse)
        if self.agg == "min":
            return float(s.min())
        return float(torch.quantile(s, float(self.agg[1:])))

    def score(self, logits: torch.Tensor, rows: Optional[torch.Tensor] = None, tp_group=None) -> float:
        """logits [R, V] (the verify rows).  maxprob = exp(top1 - lse); margin = p1 - p2.
        Under TP (vocab-sharded logits) the per-shard stats are all-gathered and merged,
        so every rank computes the same score and takes the same fire decision."""
        x = logits if rows is None else logits[rows]
        st = self.row_stats(x)
        if tp_group is not None:
            import torch.distributed as dist
            parts = [torch.empty_like(st) for _ in range(dist.get_world_size(tp_group))]
            dist.all_gather(parts, st.contiguous(), group=tp_group)
            st = self.merge_stats(torch.stack(parts))
        return self.score_stats(st)

    def should_fire(self, score: float) -> bool:
        fire = score <= self.tau
        self.stats["fired" if fire else "passed"] += 1
        return fire

    def run(self, step: Callable[[], torch.Tensor], restore: Callable[[], None],
            routed: Callable[[], List[Tuple[int, int]]], promote: Callable[[List[Tuple[int, int]]], int]) -> int:
        """step() -> verify logits.  Fires at most fp_max times; promotion failure
        leaves the step as computed (fail closed: no partial publication)."""
        n = 0
        for n in range(self.fp_max + 1):
            s = self.score(step())
            if n == self.fp_max or not self.should_fire(s):
                return n
            pairs = routed()[: self.max_promote]
            try:
                if promote(pairs) == 0:
                    return n      # nothing left to promote: replay would change nothing
            except FetchError:
                self.stats["promote_failed"] += 1
                return n
            restore()
            self.stats["replays"] += 1
        return n


class SpecGuard:
    def __init__(self, alpha: float = 0.1, hi: float = 0.6, lo: float = 0.3, patience: int = 200):
        self.alpha, self.hi, self.lo, self.patience = alpha, hi, lo, patience
        self.ema = 0.0
        self.suppressed = False
        self._since = 0
        self.backoff = 1
        self._skip = 0

    def observe(self, replayed: bool) -> bool:
        """Feed one step's replay indicator.  -> whether drafting is allowed next step."""
        self.ema = (1 - self.alpha) * self.ema + self.alpha * float(replayed)
        if not self.suppressed and self.ema > self.hi:
            self.suppressed, self._since = True, 0
        elif self.suppressed:
            self._since += 1
            if self.ema < self.lo:
                self.suppressed, self.backoff = False, 1
            elif self._since >= self.patience * self.backoff:
                # suppression is not warming the pool: resume drafting and back off before latching again
                self.suppressed, self.backoff, self._since = False, min(self.backoff * 2, 64), 0
                self.ema = self.lo
        return not self.suppressed


class LookaheadPrefetcher:
    """Predict layer L+1's experts from layer L's MoE input (routers are cheap)."""

    def __init__(self, cache: ExpertCache, routers: Sequence[torch.Tensor], top_k: int, extra: int = 2):
        self.cache, self.routers, self.top_k, self.extra = cache, routers, top_k, extra
        self.stats = collections.Counter()

    def predict(self, li: int, h: torch.Tensor) -> List[Tuple[int, int]]:
        if li + 1 >= len(self.routers) or self.routers[li + 1] is None:
            return []
        logits = h.float() @ self.routers[li + 1].float().t()
        ids = torch.topk(logits, min(self.top_k + self.extra, logits.shape[-1]), dim=-1).indices
        return [(li + 1, int(e)) for e in torch.unique(ids).tolist()]

    def step(self, li: int, h: torch.Tensor):
        pairs = [p for p in self.predict(li, h) if not self.cache.resident(*p)]
        if pairs:
            self.stats["requested"] += len(pairs)
            self.cache.request_prefetch(pairs)


class Pilot:
    """Host half of the router-lookahead prefetch (PILOT).  The decode graph writes, per
    main-stack MoE layer L + 1, the experts layer L + 1's router picks from layer L's MoE
    input (``log`` [layers, rows, K], -1 = empty).  After a step this reads the log once
    (and clears it, so a stale prediction is never fetched twice), and while the pool is
    cold -- the replay EMA at or above ``min_replay`` percent -- asks the cache to prefetch
    up to ``cap`` predicted non-resident experts off the decode stream.  On a warm pool the
    step's own misses cover the working set and predictions would only churn slots.
    (Reference: the PILOT consumer, patch P:11940-12006.)"""

    def __init__(self, cache: ExpertCache, log: torch.Tensor, cap: int = 32, min_replay: float = 30.0,
                 alpha: float = 0.05):
        self.cache, self.log, self.cap = cache, log, int(cap)
        self.min_replay, self.alpha = float(min_replay), float(alpha)
        self.ema = 1.0                     # a fresh pool is cold
        self.stats = collections.Counter()

    def observe(self, replayed: bool) -> None:
        self.ema += self.alpha * (float(replayed) - self.ema)

    def consume(self) -> int:
        """-> experts requested this step."""
        host = self.log.to("cpu", copy=True)
        self.log.fill_(-1)
        if 100.0 * self.ema < self.min_replay:
            self.stats["warm_skips"] += 1
            return 0
        E = self.cache.E
        flat = host.reshape(host.shape[0], -1)
        pairs: List[Tuple[int, int]] = []
        seen = set()
        for li in range(flat.shape[0]):
            for e in torch.unique(flat[li]).tolist():
                if 0 <= e < E and (li, e) not in seen and not self.cache.resident(li, e):
                    seen.add((li, e))
                    pairs.append((li, int(e)))
        pairs = pairs[: self.cap]
        if pairs:
            self.stats["requested"] += len(pairs)
            self.cache.request_prefetch(pairs)
        return len(pairs)


class DraftAffinity:
    """token -> per-layer expert sets learned from routing; prefetch for drafted tokens."""

    def __init__(self, cache: ExpertCache, max_tokens: int = 65536):
        self.cache = cache
        self.table: Dict[int, List[set]] = {}
        self.max_tokens = max_tokens

    def record(self, tokens: Sequence[int], route_ids: Sequence[Optional[torch.Tensor]]):
        for r, tok in enumerate(tokens):
            ent = self.table.setdefault(int(tok), [set() for _ in range(self.cache.L)])
            for li, ids in enumerate(route_ids):
                if ids is not None and r < ids.shape[0]:
                    ent[li].update(int(e) for e in ids[r].reshape(-1).tolist())
        while len(self.table) > self.max_tokens:
            self.table.pop(next(iter(self.table)))

    def prefetch(self, draft_tokens: Iterable[int]) -> int:
        pairs = set()
        for tok in draft_tokens:
            for li, es in enumerate(self.table.get(int(tok), [])):
                pairs.update((li, e) for e in es if not self.cache.resident(li, e))
        if pairs:
            self.cache.request_prefetch(sorted(pairs))
        return len(pairs)


def gate_fire_floor(moe_layers: int, top_k: int, rows: int, fp_max: int) -> int:
    """Slots an FP4 gate pool needs: one fire promotes every routed expert of the
    step, and each replay round can route to new ones (growth 1 + 0.35 (fp_max - 1))."""
    return int(math.ceil(moe_layers * top_k * rows * (1 + 0.35 * (fp_max - 1))))


def pp_gate_barrier(fire_on_last: bool, promote, tp_group=None, pp_group=None, device="cpu") -> bool:
    """Pipeline-parallel gate consensus (reference: ``_gate_pp_barrier``, patch
    P:22083-22164).  The last PP stage decides whether the confidence gate fires;
    the decision is broadcast to every stage; every rank then promotes its own
    layers' experts and the outcome is agreed fail-closed (MIN over the TP group,
    then over the PP group).  Returns True only when every rank promoted, i.e.
    when the whole pipeline must re-run the step."""
    import torch.distributed as dist
    flag = torch.tensor([1 if fire_on_last else 0], dtype=torch.int32, device=device)
    if pp_group is not None:
        last = dist.get_global_rank(pp_group, dist.get_world_size(pp_group) - 1)
        dist.broadcast(flag, src=last, group=pp_group)
    if not int(flag.item()):
        return False
    ok = 1
    try:
        promote()
    except FetchError:
        ok = 0
    t = torch.tensor([ok], dtype=torch.int32, device=device)
    for g in (tp_group, pp_group):
        if g is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=g)
    return bool(int(t.item()))


def gate_promote_consensus(promote, tp_group=None, device="cpu") -> bool:
    """Confidence-gate promotion under tensor parallelism (reference: the gate is
    fail-safe before its collective, P:21396-21404, P:18947-18957).  Every rank runs
    `promote()` (-> rows promoted; FetchError on a failed host read); the ranks agree
    (MIN of an ok flag, MAX of "promoted something") before anyone replays.  Returns
    True only when every rank succeeded and at least one promoted, i.e. when all ranks
    replay the step together; otherwise nobody replays and the step stands."""
    ok, n = 1, 0
    try:
        n = int(promote() or 0)
    except FetchError:
        ok = 0
    if tp_group is None:
        return bool(ok and n > 0)
    import torch.distributed as dist
    t = torch.tensor([ok, -min(n, 1)], dtype=torch.int32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=tp_group)   # [min ok, -max promoted]
    return bool(int(t[0]) == 1 and int(t[1]) < 0)
