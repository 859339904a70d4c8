"""Observability: residency KPIs, traces and CUDA-event span timers.

* :class:`KpiLogger` -- step counters of the residency tiers (replay rate,
  misses, fetched rows / bytes, gate fires, store hit rates and read-latency
  percentiles) logged as one ``[moet] KPI:`` line every ``every`` steps and
  dumped atomically as JSON (reference: base-tier KPI line and delta traces,
  patch P:9565-9626, P:10400-10520).
* :class:`RoutingCapture` -- bounded capture of per-step routed expert ids
  (per MoE layer) written as ``.npy`` for offline policy replay.
* :func:`precision_map` -- which (layer, expert) is resident in which tier.
* :class:`SpanTimers` -- CUDA-event spans per name, resolved lazily and
  flushed every N spans; no-ops while a CUDA graph is being captured
  (reference: prefill timers, P:13772-13830).
"""
from __future__ import annotations

import collections
import json
import logging
import os
import time
from typing import Dict, List, Optional

import torch

log = logging.getLogger("vllm_moet_b200")


def percentiles(xs: List[float], ps=(50, 99)) -> Dict[str, float]:
    if not xs:
        return {f"p{p}": 0.0 for p in ps}
    s = sorted(xs)
    return {f"p{p}": s[min(len(s) - 1, int(round(p / 100 * (len(s) - 1))))] for p in ps}


class KpiLogger:
    def __init__(self, every: int = 500, path: Optional[str] = None, sink=None):
        self.every, self.path = max(1, every), path
        self.sink = sink or log.info
        self.steps = 0
        self.c = collections.Counter()
        self.read_lat_us: collections.deque = collections.deque(maxlen=4096)
        self.gauges: Dict[str, object] = {}     # latest values (not summed): pool share, EMAs, recalls

    def step(self, replayed: bool = False, misses: int = 0, gate_fired: bool = False, **extra):
        self.steps += 1
        self.c["replayed_steps"] += int(replayed)
        self.c["misses"] += misses
        self.c["gate_fires"] += int(gate_fired)
        for k, v in extra.items():
            self.c[k] += v
        if self.steps % self.every == 0:
            self.flush()

    def gauge(self, **kv):
        """Latest-value fields of the line: ``pool_slots`` / ``pool_pct`` (cache slots, share of
        all experts), ``replay_ema`` (the spec guard's EMA, percent), ``looka`` ({previous_step,
        router_lookahead} recall)."""
        self.gauges.update(kv)

    def record_read(self, us: float):
        self.read_lat_us.append(us)

    def snapshot(self) -> dict:
        d = dict(self.c)
        d["steps"] = self.steps
        d["replay_pct"] = 100.0 * self.c["replayed_steps"] / max(1, self.steps)
        d["read_us"] = percentiles(list(self.read_lat_us))
        d.update(self.gauges)
        return d

    def line(self) -> str:
        d = self.snapshot()
        return (f"[moet] KPI: steps {d['steps']} replay {d['replay_pct']:.1f}% misses {d['misses']} "
                f"fetched {d.get('fetched_rows', 0)} rows ({d.get('fetched_bytes', 0) / 2**20:.1f} MiB) "
                f"gate fires {d['gate_fires']} read p50/p99 {d['read_us']['p50']:.0f}/{d['read_us']['p99']:.0f} us"
                + self._tail(d))

    @staticmethod
    def _tail(d: dict) -> str:
        """The optional fields, in the reference's KPI order: pool share, draft-prefetched
        experts, replay EMA, LOOKA recall."""
        out = []
        if "pool_slots" in d:
            out.append(f"pool {d['pool_slots']} slots = {d.get('pool_pct', 0.0):.1f}% of experts")
        if d.get("draft_prefetched"):
            out.append(f"draft-prefetched {d['draft_prefetched']}")
        if "replay_ema" in d:
            out.append(f"replay EMA {d['replay_ema']:.1f}%")
        if "looka" in d:
            lk = d["looka"]
            out.append(f"LOOKA recall prev/router {lk.get('previous_step', 0.0):.2f}/{lk.get('router_lookahead', 0.0):.2f}")
        return "".join("; " + x for x in out)

    def flush(self):
        self.sink(self.line())
        if self.path:
            from ..residency.fsutil import atomic_write_json
            atomic_write_json(self.path, self.snapshot())


class RoutingCapture:
    def __init__(self, max_steps: int = 10000):
        self.max_steps = max_steps
        self.steps: List[List[torch.Tensor]] = []

    def record(self, route_ids):
        if len(self.steps) < self.max_steps:
            self.steps.append([None if r is None else r.detach().cpu().clone() for r in route_ids])

    def save(self, path: str):
        import numpy as np
        if not self.steps:
            return
        L = len(self.steps[0])
        rows = max((r.numel() for s in self.steps for r in s if r is not None), default=0)
        arr = np.full((len(self.steps), L, rows), -1, dtype=np.int32)
        for i, s in enumerate(self.steps):
            for li, r in enumerate(s):
                if r is not None:
                    v = r.reshape(-1).numpy()
                    arr[i, li, :v.size] = v
        tmp = path + ".tmp.npy"
        np.save(tmp, arr)
        os.replace(tmp, path)


def precision_map(cache, tier: str = "base-2bit") -> dict:
    """{"L": .., "E": .., "tier": .., "resident": [[layer, expert, slot], ...]} of an ExpertCache."""
    res = [[int(li), int(e), int(cache.mirror[li, e])] for li, e in (cache.mirror >= 0).nonzero().tolist()]
    return {"L": cache.L, "E": cache.E, "tier": tier, "resident": res}


class DeltaTrace:
    """Delta-tier coverage and hit rates (reference: VLLM_MOE_W2_DELTA_TRACE, P:9718-9820).
    Per decode step: the routed (layer, expert) pairs and how many of them the FP4
    tier served (distinct pairs, and weighted by the tokens routed to them)."""

    def __init__(self, level: int = 1, every: int = 500, sink=None):
        self.level, self.every = level, max(1, every)
        self.sink = sink or log.info
        self.steps = 0
        self.c = collections.Counter()

    def step(self, delta, routed_tokens: Dict[tuple, int]):
        self.steps += 1
        for (li, e), n in routed_tokens.items():
            hit = delta.resident(li, e)
            self.c["pairs"] += 1
            self.c["pair_hits"] += int(hit)
            self.c["tokens"] += n
            self.c["token_hits"] += n if hit else 0
        if self.steps % self.every == 0:
            self.sink(self.line(delta))

    def snapshot(self, delta) -> dict:
        resident = int((delta.mirror >= 0).sum())
        d = {"steps": self.steps, "coverage": resident / max(1, delta.L * delta.E), "resident": resident,
             "hit_rate_distinct": self.c["pair_hits"] / max(1, self.c["pairs"]),
             "hit_rate_tokens": self.c["token_hits"] / max(1, self.c["tokens"]),
             "promoted_rows": int(delta.stats["fetched_rows"]), "evictions": int(delta.stats["evictions"])}
        if self.level >= 2:
            d["fp4_per_layer"] = (delta.mirror >= 0).sum(dim=1).tolist()
        return d

    def line(self, delta) -> str:
        d = self.snapshot(delta)
        s = (f"[moet] delta: steps {d['steps']} coverage {100 * d['coverage']:.1f}% ({d['resident']} experts) "
             f"hit distinct {100 * d['hit_rate_distinct']:.1f}% tokens {100 * d['hit_rate_tokens']:.1f}% "
             f"promoted {d['promoted_rows']} evicted {d['evictions']}")
        if self.level >= 2:
            s += f" per-layer {d['fp4_per_layer']}"
        return s


class JsonlWriter:
    """Append-only JSON lines (one object per line, flushed per row)."""

    def __init__(self, path: str):
        self.path = path
        self.f = open(path, "a", buffering=1)

    def write(self, row: dict):
        self.f.write(json.dumps(row, sort_keys=True) + "\n")

    def close(self):
        self.f.close()


class HiddenCapture:
    """Hidden states of the gate's dumped (fired / audited) steps, for offline gate-signal
    studies: ``store(step, h)`` keeps one [rows, H] tensor per step, every ``flush``
    records a shard ``hcap-NNNNN.pt`` = {"steps": int64 [n], "h": list of tensors} goes to
    ``dir``; consumers join on the gate dump's ``step`` field.  (Reference: the gate's
    hidden-state capture, VLLM_MOE_W2_GATE_HCAP_DIR / _FLUSH, patch P:11384-11420.)"""

    def __init__(self, dir_: str, flush: int = 256):
        self.dir, self.flush_every = dir_, max(1, int(flush))
        self.steps: List[int] = []
        self.h: List[torch.Tensor] = []
        self.shard = 0

    def store(self, step: int, h: torch.Tensor):
        self.steps.append(int(step))
        self.h.append(h.detach().to("cpu", torch.float32))
        if len(self.steps) >= self.flush_every:
            self.flush()

    def flush(self):
        if not self.steps:
            return
        os.makedirs(self.dir, exist_ok=True)
        path = os.path.join(self.dir, f"hcap-{self.shard:05d}.pt")
        torch.save({"steps": torch.tensor(self.steps, dtype=torch.int64), "h": self.h}, path + ".tmp")
        os.replace(path + ".tmp", path)
        self.shard += 1
        self.steps, self.h = [], []

    def close(self):
        self.flush()


class SpanTimers:
    def __init__(self, flush_every: int = 64, sink=None):
        self.flush_every = flush_every
        self.sink = sink or log.info
        self.pending: List = []
        self.totals: Dict[str, List[float]] = collections.defaultdict(list)

    def span(self, name: str):
        timers = self

        class _Span:
            def __enter__(self):
                self.on = torch.cuda.is_available() and not torch.cuda.is_current_stream_capturing()
                if self.on:
                    self.a = torch.cuda.Event(enable_timing=True)
                    self.a.record()
                else:
                    self.t0 = time.perf_counter()
                return self

            def __exit__(self, *exc):
                if self.on:
                    b = torch.cuda.Event(enable_timing=True)
                    b.record()
                    timers.pending.append((name, self.a, b))
                    if len(timers.pending) >= timers.flush_every:
                        timers.flush()
                elif not (torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()):
                    timers.totals[name].append((time.perf_counter() - self.t0) * 1e3)
                return False
        return _Span()

    def flush(self):
        if self.pending:
            self.pending[-1][2].synchronize()
            for name, a, b in self.pending:
                self.totals[name].append(a.elapsed_time(b))
            self.pending.clear()

    def summary(self) -> Dict[str, dict]:
        self.flush()
        return {k: {"n": len(v), "total_ms": sum(v), "mean_ms": sum(v) / len(v)} for k, v in self.totals.items() if v}

    def dump(self, path: str):
        from ..residency.fsutil import atomic_write_json
        atomic_write_json(path, self.summary())
