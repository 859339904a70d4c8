"""Host expert stores: where expert rows live when they are not on the GPU.

One interface, three backends (the reference's moe_w2_store.py, patch
P:12830-13771, behaviour re-implemented here):

* :class:`PinnedHostStore` -- per-layer pinned ``[E, slot_bytes]`` tensors;
  rows are zero-copy views handed to ``cudaMemcpyAsync``.
* :class:`MmapPackStore` -- rows in a per-rank **pack file** on disk at
  offset ``(layer * E + expert) * stride`` with ``stride`` = slot bytes rounded
  up to 4 KiB (the same file serves buffered and ``O_DIRECT`` reads); a JSON
  sidecar lists the layers written.  Writes are ``pwrite`` + ``fdatasync``
  under ``flock`` and the sidecar is replaced atomically (fsync + rename +
  directory fsync).  Reads go through the native :class:`PackFile` thread
  pool into a pinned stage.
* :class:`TieredPackStore` -- a pinned MRU **arena** of rows over the same
  pack: hits are zero-copy views, misses are read straight into an arena slot
  (the arena is the bounce buffer).  ``scan=True`` reads (one-shot prefill
  sweeps) bypass the arena so they cannot evict the hot set.  A failed read is
  never published: its slot goes back to the free list and the expert is
  reported in ``failed``.  The arena's recency ranking is dumped to and
  preloaded from a ``.heat.json`` file.

Pack file names: ``<tag>.v2.<key20>.<rank suffix>.{pack,json,lock}`` where
``key20`` is the first 20 hex digits of sha256 over the identity (checkpoint
id, quantizer ABI, zero mode) and the geometry, so two checkpoints or ABIs
never share a pack.  Sidecar fields: version, tag, E, n_layers, slot_bytes,
stride, ckpt_id, zero_mode, quantizer_abi, layers.
"""
from __future__ import annotations

import collections
import hashlib
import json
import os
import threading
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .fsutil import atomic_write_json, exclusive_lock, read_json
from .identity import identity_fields, rank_suffix

ALIGN = 4096
PACK_VERSION = 2
CHECK_FIELDS = ("version", "tag", "E", "n_layers", "slot_bytes", "stride", "ckpt_id", "zero_mode", "quantizer_abi")


def stride_for(slot_bytes: int) -> int:
    return -(-slot_bytes // ALIGN) * ALIGN


def pack_paths(dir_: str, tag: str, n_layers: int, E: int, slot_bytes: int, ckpt_id: Optional[str],
               suffix: str = "rank0of1"):
    """-> (pack path, sidecar path, lock path, identity dict)."""
    identity = identity_fields(ckpt_id)
    key = dict(identity, tag=tag, n_layers=n_layers, E=E, slot_bytes=slot_bytes, stride=stride_for(slot_bytes))
    if key["ckpt_id"] is None:
        key["ckpt_id"] = f"unverified-process-{os.getpid()}"
    h = hashlib.sha256(json.dumps(key, sort_keys=True, separators=(",", ":")).encode()).hexdigest()[:20]
    base = os.path.join(dir_, f"{tag}.v2.{h}.{suffix}")
    return base + ".pack", base + ".json", base + ".lock", identity


def _pinned(nbytes: int) -> torch.Tensor:
    if torch.cuda.is_available():
        return torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    return torch.empty(nbytes, dtype=torch.uint8)


class StoreReadError(IOError):
    pass


@dataclass
class RowBatch:
    """Rows of one ``rows_for`` call, in request order (None where the read failed)."""
    rows: List[Optional[torch.Tensor]]
    failed: List[int] = field(default_factory=list)


class _PyPackFile:
    """Pure-Python stand-in for the native PackFile (used only without the extension)."""

    def __init__(self, path, writable, direct, stride, threads=8):
        self.fd = os.open(path, (os.O_RDWR | os.O_CREAT) if writable else os.O_RDONLY, 0o644)
        self.stride = stride
        self.direct = False
        self._fault_every, self._reads = 0, 0

    def write_rows(self, first_row, rows):
        data = rows.contiguous().numpy()
        for i in range(rows.shape[0]):
            os.pwrite(self.fd, data[i].tobytes(), (first_row + i) * self.stride)

    def sync(self):
        os.fdatasync(self.fd)

    def read_rows(self, rows, dst_ptr, dst_stride, nbytes):
        import ctypes
        out = []
        for i, r in enumerate(rows):
            self._reads += 1
            if self._fault_every and self._reads % self._fault_every == 0:
                out.append(5)
                continue
            b = os.pread(self.fd, nbytes, r * self.stride)
            b = b + bytes(nbytes - len(b))
            ctypes.memmove(dst_ptr + i * dst_stride, b, nbytes)
            out.append(0)
        return out

    def inject_read_faults(self, every):
        self._fault_every, self._reads = every, 0

    def size_bytes(self):
        return os.fstat(self.fd).st_size

    def close(self):
        if self.fd >= 0:
            os.close(self.fd)
            self.fd = -1


def _open_pack(path, writable, direct, stride, threads):
    try:
        from ..ops import native
        return native().PackFile(path, writable, direct, stride, threads)
    except (RuntimeError, AttributeError):
        return _PyPackFile(path, writable, direct, stride, threads)


class HostStore:
    kind = "base"

    def __init__(self, n_layers: int, E: int, slot_bytes: int):
        self.n_layers, self.E, self.slot_bytes = n_layers, E, slot_bytes
        self.stats_ = collections.Counter()

    def add_layer(self, li: int, rows: torch.Tensor) -> None:
        raise NotImplementedError

    def has_layer(self, li: int) -> bool:
        raise NotImplementedError

    def rows_for(self, li: int, experts: List[int], scan: bool = False) -> RowBatch:
        raise NotImplementedError

    def release(self) -> None:
        pass

    def stats(self) -> dict:
        return dict(self.stats_)

    def _check_rows(self, rows):
        if rows.dtype != torch.uint8 or tuple(rows.shape) != (self.E, self.slot_bytes):
            raise ValueError(f"layer rows must be uint8 [{self.E}, {self.slot_bytes}], got {rows.dtype} {tuple(rows.shape)}")


class PinnedHostStore(HostStore):
    kind = "pinned"

    def __init__(self, n_layers, E, slot_bytes, pin: bool = True):
        super().__init__(n_layers, E, slot_bytes)
        self.pin = pin and torch.cuda.is_available()
        self.layers: Dict[int, torch.Tensor] = {}

    def add_layer(self, li, rows):
        self._check_rows(rows)
        t = rows.cpu().contiguous()
        self.layers[li] = t.pin_memory() if self.pin else t.clone()

    def has_layer(self, li):
        return li in self.layers

    def rows_for(self, li, experts, scan=False):
        t = self.layers[li]
        self.stats_["rows"] += len(experts)
        return RowBatch([t[e] for e in experts])

    def release(self):
        self.layers.clear()


class MmapPackStore(HostStore):
    kind = "pack"

    def __init__(self, dir_: str, tag: str, n_layers: int, E: int, slot_bytes: int, ckpt_id: Optional[str] = None,
                 suffix: Optional[str] = None, direct: bool = False, threads: int = 8):
        super().__init__(n_layers, E, slot_bytes)
        os.makedirs(dir_, exist_ok=True)
        self.dir, self.tag = dir_, tag
        self.stride = stride_for(slot_bytes)
        self.pack_path, self.sidecar_path, self.lock_path, identity = pack_paths(
            dir_, tag, n_layers, E, slot_bytes, ckpt_id, suffix or rank_suffix())
        self.expected = dict(version=PACK_VERSION, tag=tag, E=E, n_layers=n_layers, slot_bytes=slot_bytes,
                             stride=self.stride, **identity)
        with exclusive_lock(self.lock_path):
            self.layers = set(self._sidecar_layers())
        self.f = _open_pack(self.pack_path, True, direct, self.stride, threads)
        self._stage = None
        self._lock = threading.Lock()

    # ---- sidecar
    def _sidecar_layers(self) -> List[int]:
        meta = read_json(self.sidecar_path)
        if meta is None or any(meta.get(k) != self.expected[k] for k in CHECK_FIELDS):
            return []           # missing, corrupt or foreign: the layers are rebuilt
        try:
            layers = sorted({int(li) for li in meta.get("layers", [])})
        except (TypeError, ValueError):
            return []
        return [li for li in layers if 0 <= li < self.n_layers]

    def add_layer(self, li, rows):
        self._check_rows(rows)
        if not 0 <= li < self.n_layers:
            raise IndexError(li)
        with exclusive_lock(self.lock_path):
            self.f.write_rows(li * self.E, rows.cpu().contiguous())
            self.f.sync()
            layers = set(self._sidecar_layers()) | {li}
            atomic_write_json(self.sidecar_path, dict(self.expected, layers=sorted(layers)))
            self.layers = layers
        self.stats_["layers_written"] += 1

    def has_layer(self, li):
        return li in self.layers

    def _stage_rows(self, n):
        need = n * self.stride
        if self._stage is None or self._stage.numel() < need:
            self._stage = _pinned(max(need, 64 * self.stride) + ALIGN)
        base = self._stage.data_ptr()
        off = (-base) % ALIGN
        return self._stage, off

    def _read_into(self, li, experts, dst: torch.Tensor, dst_off: int, dst_stride: int):
        rows = [li * self.E + e for e in experts]
        t0 = time.perf_counter()
        st = self.f.read_rows(rows, dst.data_ptr() + dst_off, dst_stride, self.slot_bytes)
        self.stats_["read_s_us"] += int((time.perf_counter() - t0) * 1e6)
        self.stats_["rows_read"] += len(rows)
        self.stats_["bytes_read"] += len(rows) * self.slot_bytes
        return st

    def rows_for(self, li, experts, scan=False):
        if li not in self.layers:
            raise KeyError(f"layer {li} is not in the pack")
        with self._lock:
            stage, off = self._stage_rows(len(experts))
            st = self._read_into(li, experts, stage, off, self.stride)
            out, failed = [], []
            for i, (e, code) in enumerate(zip(experts, st)):
                if code:
                    out.append(None)
                    failed.append(e)
                    self.stats_["read_errors"] += 1
                else:
                    s = off + i * self.stride
                    out.append(stage[s:s + self.slot_bytes])
            return RowBatch(out, failed)

    def inject_read_faults(self, every: int):
        self.f.inject_read_faults(every)

    def release(self):
        self.f.close()


class TieredPackStore(MmapPackStore):
    kind = "tiered"

    def __init__(self, *a, arena_rows: int = 64, scan: bool = True, **kw):
        super().__init__(*a, **kw)
        self.arena_rows = max(1, int(arena_rows))
        self.scan_enabled = bool(scan)      # False: sweeps go through the arena like any read
        self._arena_raw = _pinned(self.arena_rows * self.stride + ALIGN)
        self._arena_off = (-self._arena_raw.data_ptr()) % ALIGN
        self.lru: "collections.OrderedDict[tuple, int]" = collections.OrderedDict()
        self.free = list(range(self.arena_rows - 1, -1, -1))

    def _slot_view(self, slot):
        s = self._arena_off + slot * self.stride
        return self._arena_raw[s:s + self.slot_bytes]

    def rows_for(self, li, experts, scan=False):
        if li not in self.layers:
            raise KeyError(f"layer {li} is not in the pack")
        with self._lock:
            out: List[Optional[torch.Tensor]] = [None] * len(experts)
            miss_idx = []
            for i, e in enumerate(experts):
                slot = self.lru.get((li, e))
                if slot is not None:
                    self.lru.move_to_end((li, e))
                    out[i] = self._slot_view(slot)
                    self.stats_["arena_hits"] += 1
                else:
                    miss_idx.append(i)
            failed = []
            if not miss_idx:
                return RowBatch(out, failed)
            self.stats_["arena_misses"] += len(miss_idx)
            miss_e = [experts[i] for i in miss_idx]
            protect = {(li, e) for e in experts}
            evictable = len(self.free) + sum(1 for k in self.lru if k not in protect)
            if (scan and self.scan_enabled) or len(miss_idx) > evictable:
                # scan resistance (and arena overflow): read through the stage, leave the arena as is
                stage, off = self._stage_rows(len(miss_idx))
                st = self._read_into(li, miss_e, stage, off, self.stride)
                for j, (i, code) in enumerate(zip(miss_idx, st)):
                    if code:
                        failed.append(experts[i])
                    else:
                        s = off + j * self.stride
                        out[i] = stage[s:s + self.slot_bytes]
                self.stats_["read_errors"] += len(failed)
                return RowBatch(out, failed)
            slots = []
            for _ in miss_idx:
                if self.free:
                    slots.append(self.free.pop())
                    continue
                victim = next(k for k in self.lru if k not in protect)
                slots.append(self.lru.pop(victim))
                self.stats_["arena_evictions"] += 1
            # read each miss into its slot (slots are not contiguous: one call per slot run)
            for j, (i, slot) in enumerate(zip(miss_idx, slots)):
                st = self._read_into(li, [experts[i]], self._arena_raw, self._arena_off + slot * self.stride,
                                     self.stride)
                if st[0]:
                    self.free.append(slot)          # never publish a failed read
                    failed.append(experts[i])
                    self.stats_["read_errors"] += 1
                else:
                    self.lru[(li, experts[i])] = slot
                    out[i] = self._slot_view(slot)
            return RowBatch(out, failed)

    # ---- heat
    @property
    def heat_path(self):
        return self.pack_path[:-5] + ".heat.json"

    def dump_heat(self):
        atomic_write_json(self.heat_path, {"rows": [list(k) for k in reversed(self.lru.keys())]})

    def preheat(self, max_rows: Optional[int] = None) -> int:
        meta = read_json(self.heat_path)
        if not meta:
            return 0
        keys = [tuple(k) for k in meta.get("rows", []) if isinstance(k, list) and len(k) == 2]
        n = 0
        for li, e in reversed(keys[: max_rows or int(0.9 * self.arena_rows)]):
            if li in self.layers and 0 <= e < self.E and (li, e) not in self.lru:
                if not self.rows_for(li, [e]).failed:
                    n += 1
        return n


def make_store(kind: str, n_layers: int, E: int, slot_bytes: int, **kw) -> HostStore:
    kind = kind.lower()
    if kind == "pinned":
        return PinnedHostStore(n_layers, E, slot_bytes, pin=kw.get("pin", True))
    if kind == "pack":
        return MmapPackStore(kw["dir"], kw.get("tag", "base"), n_layers, E, slot_bytes, kw.get("ckpt_id"),
                             kw.get("suffix"), kw.get("direct", False), kw.get("threads", 8))
    if kind == "tiered":
        return TieredPackStore(kw["dir"], kw.get("tag", "base"), n_layers, E, slot_bytes, kw.get("ckpt_id"),
                               kw.get("suffix"), kw.get("direct", False), kw.get("threads", 8),
                               arena_rows=kw.get("arena_rows", 64), scan=kw.get("scan", True))
    raise ValueError(f"unknown store kind {kind!r} (pinned | pack | tiered)")


def pack_has_layer(dir_: str, tag: str, n_layers: int, E: int, slot_bytes: int, li: int,
                   ckpt_id: Optional[str] = None, suffix: Optional[str] = None) -> bool:
    """Probe a pack sidecar without opening the pack (boot-from-pack planning)."""
    pack, side, _, identity = pack_paths(dir_, tag, n_layers, E, slot_bytes, ckpt_id, suffix or rank_suffix())
    meta = read_json(side)
    if meta is None or not os.path.exists(pack):
        return False
    exp = dict(version=PACK_VERSION, tag=tag, E=E, n_layers=n_layers, slot_bytes=slot_bytes,
               stride=stride_for(slot_bytes), **identity)
    if any(meta.get(k) != exp[k] for k in CHECK_FIELDS):
        return False
    return li in {int(x) for x in meta.get("layers", []) if isinstance(x, int)}
