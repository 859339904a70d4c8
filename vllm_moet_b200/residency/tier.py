"""GPU expert cache over a host store (the "base cache" residency tier).

The routed experts of every MoE layer live in a host store
(:mod:`.stores`); the GPU holds a pool of ``n_slots`` expert slots
``[n_slots, slot_bytes]`` and a device **slot table** ``int32 [L, E]``
(-1 = not resident) that the expert kernels read inside the captured decode
graph.  A routed expert whose slot is -1 contributes zero rows and bumps a
device ``miss_count``; the runner then fetches the missing experts and
replays the step until it is miss-free (:class:`ReplayEngine`).  This is
the reference's base tier / DeltaTier machinery (moe_w2_delta.py, patch
P:8068-10287), re-designed around one pool and one table for all layers.

Pieces:
* slot allocation with recency (``lru``) or decayed-frequency (``freq``)
  eviction; slots touched by the current step are pinned and never evicted;
* ``ensure_resident(li, experts)`` -- synchronous fetch used by prefill;
* ``promote(pairs)`` -- batched fetch (replay and prefetch), H2D on a side
  stream, one event, slot-table update published only after every row of
  the batch was read successfully (a failed host read publishes nothing);
* a manager thread serving asynchronous prefetch requests, with
  :meth:`wait_idle` as the safe point the runner calls before every graph
  replay, so no slot-table / pool mutation overlaps graph readers;
* pool heat: the frequency ranking is dumped to JSON and preloaded at boot.
"""
from __future__ import annotations

import collections
import json
import os
import queue
import threading
import time
from typing import Iterable, List, Optional, Sequence, Tuple

import torch

from .fsutil import atomic_write_json, read_json
from .stores import HostStore


class FetchError(RuntimeError):
    pass


class ExpertCache:
    def __init__(self, store: HostStore, n_layers: int, E: int, slot_bytes: int, n_slots: int, device="cuda",
                 policy: str = "lru", decay: float = 0.9, manager: bool = True):
        if policy not in ("lru", "freq"):
            raise ValueError("policy must be lru or freq")
        self.store, self.L, self.E, self.slot_bytes = store, n_layers, E, slot_bytes
        self.n_slots = int(n_slots)
        self.dev = torch.device(device)
        self.policy, self.decay = policy, decay
        self.pool = torch.zeros(self.n_slots, slot_bytes, dtype=torch.uint8, device=self.dev)
        self.slot_table = torch.full((n_layers, E), -1, dtype=torch.int32, device=self.dev)
        self.miss_count = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.mirror = torch.full((n_layers, E), -1, dtype=torch.int32)
        self.owner: List[Optional[Tuple[int, int]]] = [None] * self.n_slots
        self.last_use = [0.0] * self.n_slots
        self.freq = torch.zeros(n_layers, E, dtype=torch.float32)
        self.pinned: set = set()
        self.protect = None            # (li, e) -> True: never evict (split-FP4 delta slots read this base)
        self.free = list(range(self.n_slots - 1, -1, -1))
        self.step = 0
        self.lock = threading.RLock()
        self.stats = collections.Counter()
        self._copy_stream = torch.cuda.Stream(device=self.dev) if self.dev.type == "cuda" else None
        self._q: "queue.Queue" = queue.Queue()
        self._idle = threading.Event()
        self._idle.set()
        self._thread = None
        if manager:
            self._thread = threading.Thread(target=self._manager, name="expert-cache-manager", daemon=True)
            self._thread.start()

    # ------------------------------------------------------------------ views
    def layer_table(self, li: int) -> torch.Tensor:
        return self.slot_table[li]

    def resident(self, li: int, e: int) -> bool:
        return int(self.mirror[li, e]) >= 0

    # ------------------------------------------------------------------ scopes
    def step_begin(self):
        with self.lock:
            self.step += 1
            self.freq.mul_(self.decay)

    def step_end(self):
        with self.lock:
            self.pinned.clear()

    def note_routed(self, li: int, experts: Iterable[int], weight: float = 1.0):
        """Record use of (li, e) for the eviction policies and pin them for this step."""
        now = time.monotonic()
        with self.lock:
            for e in experts:
                self.freq[li, e] += weight
                s = int(self.mirror[li, e])
                if s >= 0:
                    self.last_use[s] = now
                    self.pinned.add(s)

    # ------------------------------------------------------------------ slots
    def _victim(self, protect: set) -> int:
        best, best_key = -1, None
        for s in range(self.n_slots):
            if s in self.pinned or s in protect or self.owner[s] is None:
                continue
            li, e = self.owner[s]
            if self.protect is not None and self.protect(li, e):
                continue
            key = self.last_use[s] if self.policy == "lru" else (float(self.freq[li, e]), self.last_use[s])
            if best_key is None or key < best_key:
                best, best_key = s, key
        if best < 0:
            raise FetchError("expert cache: every slot is pinned by the current step (pool below the working-set floor)")
        return best

    def _take_slots(self, n: int, protect: set, evicted: list) -> List[int]:
        """n slots (free first, then victims).  All or nothing: if a victim cannot be
        found, every slot taken so far goes back to its owner or the free list."""
        out, from_free = [], []
        try:
            for _ in range(n):
                if self.free:
                    s = self.free.pop()
                    from_free.append(s)
                    out.append(s)
                else:
                    s = self._victim(protect | set(out))
                    li, e = self.owner[s]
                    self.mirror[li, e] = -1
                    self.owner[s] = None
                    evicted.append((li, e, s))
                    out.append(s)
        except FetchError:
            for li, e, s in evicted:
                self.mirror[li, e] = s
                self.owner[s] = (li, e)
            self.free.extend(reversed(from_free))
            evicted.clear()
            raise
        self.stats["evictions"] += len(evicted)
        evicted[:] = [(li, e) for li, e, _ in evicted]
        return out

    # ------------------------------------------------------------------ fetch
    def _stage_for(self, n: int) -> torch.Tensor:
        st = getattr(self, "_stage", None)
        if st is None or st.shape[0] < n:
            st = torch.empty(max(n, 64), self.slot_bytes, dtype=torch.uint8)
            if self.dev.type == "cuda":
                st = st.pin_memory()
            self._stage = st
        return st

    def promote(self, pairs: Sequence[Tuple[int, int]], stream: Optional[torch.cuda.Stream] = None,
                sync: bool = True) -> int:
        """Make (layer, expert) pairs resident.  -> number of rows fetched.
        Rows are read from the host store, copied H2D on the copy stream and
        published in the slot table only when the whole batch read cleanly."""
        with self.lock:
            want = [(li, e) for li, e in dict.fromkeys(pairs) if int(self.mirror[li, e]) < 0]
            if not want:
                return 0
            if len(want) > self.n_slots - len(self.pinned):
                raise FetchError(f"expert cache: {len(want)} experts needed but only "
                                 f"{self.n_slots - len(self.pinned)} slots can be freed")
            protect = {int(self.mirror[li, e]) for li, e in pairs if int(self.mirror[li, e]) >= 0}
            by_layer = collections.defaultdict(list)
            for li, e in want:
                by_layer[li].append(e)
            # Rows are copied into the cache's own pinned stage right away: a store may
            # reuse its read buffer for the next layer's batch.
            stage = self._stage_for(len(want))
            rows, k = {}, 0
            for li, es in by_layer.items():
                batch = self.store.rows_for(li, es)
                if batch.failed:
                    self.stats["fetch_failures"] += len(batch.failed)
                    raise FetchError(f"host store read failed for layer {li} experts {batch.failed}")
                for e, r in zip(es, batch.rows):
                    stage[k].copy_(r)
                    rows[(li, e)] = stage[k]
                    k += 1
            evicted: list = []
            slots = self._take_slots(len(want), protect, evicted)
            cs = self._copy_stream
            ctx = torch.cuda.stream(cs) if cs is not None else _null()
            if cs is not None:
                cs.wait_stream(stream or torch.cuda.current_stream(self.dev))
            with ctx:
                for (li, e), s in zip(want, slots):
                    self.pool[s].copy_(rows[(li, e)], non_blocking=True)
                # evicted entries go to -1 and new ones to their slot in one indexed copy
                idx = torch.tensor([li * self.E + e for li, e in evicted + want], dtype=torch.long)
                val = torch.tensor([-1] * len(evicted) + slots, dtype=torch.int32)
                self.slot_table.view(-1).index_copy_(0, idx.to(self.dev, non_blocking=True),
                                                     val.to(self.dev, non_blocking=True))
            if cs is not None:
                ev = torch.cuda.Event()
                ev.record(cs)
                (stream or torch.cuda.current_stream(self.dev)).wait_event(ev)
                if sync:
                    ev.synchronize()    # host rows may be reused by the store after return
            now = time.monotonic()
            for (li, e), s in zip(want, slots):
                self.mirror[li, e] = s
                self.owner[s] = (li, e)
                self.last_use[s] = now
                self.pinned.add(s)
            self.stats["fetched_rows"] += len(want)
            self.stats["fetched_bytes"] += len(want) * self.slot_bytes
            return len(want)

    def ensure_resident(self, li: int, experts: Iterable[int]) -> int:
        """Synchronous per-layer fetch (prefill): every listed expert of layer li is resident on return."""
        es = sorted({int(e) for e in experts})
        with self.lock:
            # eager execution is stream-ordered: an earlier layer's slots may be reused
            # (the copy stream waits for the work already queued on the compute stream)
            self.pinned.clear()
        self.note_routed(li, es)
        n = self.promote([(li, e) for e in es])
        self.stats["ensure_calls"] += 1
        return n

    # ------------------------------------------------------------------ manager thread
    def request_prefetch(self, pairs: Sequence[Tuple[int, int]]):
        """Asynchronous promotion (prefetchers).  Served by the manager thread."""
        if self._thread is None:
            self.promote(pairs)
            return
        self._idle.clear()
        self._q.put(list(pairs))

    def _manager(self):
        while True:
            item = self._q.get()
            if item is None:
                return
            try:
                free_now = [(li, e) for li, e in item if int(self.mirror[li, e]) < 0]
                if free_now:
                    self.promote(free_now[: max(0, self.n_slots - len(self.pinned) - 1)])
                    self.stats["prefetched_rows"] += len(free_now)
            except FetchError:
                self.stats["prefetch_failures"] += 1
            finally:
                if self._q.empty():
                    self._idle.set()

    def wait_idle(self, timeout: float = 30.0) -> bool:
        """Safe point: returns when no promotion is queued or running."""
        return self._idle.wait(timeout)

    # ------------------------------------------------------------------ invariants
    def check_invariants(self, host_row=None, base=None) -> None:
        """Residency invariants (reference storm / stress checks I1-I5), raising
        AssertionError on the first violation.  Call at a safe point (no promotion
        in flight).
        I1 every resident slot holds the bytes of its host row (``host_row(li, e)``);
        I2 mirror, owner and free list are one bijection: mirror[li, e] = s exactly
           when owner[s] = (li, e), a free slot has no owner, no slot is both;
        I4 the device slot table (what the kernels dispatch on) equals the mirror;
        I5 with ``base`` (split-FP4 coupling): every resident expert here is resident there."""
        with self.lock:
            seen = set()
            for s, own in enumerate(self.owner):
                if own is None:
                    continue
                li, e = own
                assert int(self.mirror[li, e]) == s, f"I2: owner[{s}] = {own} but mirror = {int(self.mirror[li, e])}"
                assert own not in seen, f"I2: {own} owns two slots"
                seen.add(own)
            for li, e in (self.mirror >= 0).nonzero().tolist():
                s = int(self.mirror[li, e])
                assert self.owner[s] == (li, e), f"I2: mirror[{li},{e}] = {s} but owner = {self.owner[s]}"
            free = set(self.free)
            assert len(free) == len(self.free), "I2: a slot is free twice"
            assert all(self.owner[s] is None for s in free), "I2: a free slot has an owner"
            assert len(free) + len(seen) == self.n_slots, "I2: a slot is neither free nor owned"
            table = self.slot_table.cpu()
            assert torch.equal(table, self.mirror.to(table.dtype)), "I4: device slot table != mirror"
            if host_row is not None:
                for li, e in seen:
                    s = int(self.mirror[li, e])
                    assert torch.equal(self.pool[s].cpu(), host_row(li, e).cpu()), f"I1: slot {s} != host row {li},{e}"
            if base is not None:
                for li, e in seen:
                    assert base.resident(li, e), f"I5: ({li}, {e}) has an FP4 slot but no resident base"

    # ------------------------------------------------------------------ heat
    def dump_heat(self, path: str):
        with self.lock:
            order = torch.argsort(self.freq.view(-1), descending=True)
            ranked = [[int(i) // self.E, int(i) % self.E] for i in order[: self.n_slots * 2]
                      if float(self.freq.view(-1)[i]) > 0]
        atomic_write_json(path, {"version": 1, "L": self.L, "E": self.E, "ranked": ranked})

    def preload(self, path: Optional[str] = None, fraction: float = 0.9) -> int:
        """Fill up to `fraction` of the pool: from a heat file if given, else layer-major order."""
        cap = int(self.n_slots * fraction)
        pairs = []
        meta = read_json(path) if path else None
        if meta and meta.get("L") == self.L and meta.get("E") == self.E:
            pairs = [tuple(p) for p in meta.get("ranked", [])][:cap]
        if not pairs:
            pairs = [(li, e) for li in range(self.L) for e in range(self.E)
                     if self.store.has_layer(li)][:cap]
        n = 0
        for i in range(0, len(pairs), 256):
            n += self.promote(pairs[i:i + 256])
            self.step_end()
        return n

    def close(self):
        if self._thread is not None:
            self._q.put(None)
            self._thread.join(timeout=5)
            self._thread = None


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def working_set_floor(moe_layers: int, top_k: int, spec_tokens: int, max_seqs: int,
                      num_experts: int = 1 << 30) -> int:
    """Slots a base pool needs so one decode step's routed pairs always fit
    (moe layers x min(E, top_k x (1 + spec) x min(seqs, 4)), with a 1.15 margin)."""
    per_layer = min(num_experts, top_k * (1 + spec_tokens) * min(max_seqs, 4))
    return int(1.15 * moe_layers * per_layer + 0.999)


def resident_fit(expert_bytes_total: int, free_bytes: int, kv_floor_bytes: int, reserve_bytes: int = 2 << 30):
    """Hard stop for fully resident experts: -> (fits, suggested cache GiB)."""
    avail = free_bytes - kv_floor_bytes - reserve_bytes
    return expert_bytes_total <= avail, max(0.0, avail / (1 << 30))
