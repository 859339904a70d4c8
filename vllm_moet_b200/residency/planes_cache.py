"""Persistent quantization cache for GPU-resident expert planes.

Quantizing a large checkpoint's experts to the 2-bit planes takes minutes;
the planes cache keeps the result on disk so the next boot loads bytes
instead (the reference's moe_w2_planes_cache.py, patch P:12476-12821):

    <root>/v2/<sha20(meta)>/tp{W}-rank{R}/layer{L}.<part>.bin
    <root>/v2/<sha20(meta)>/meta.json

``meta`` holds the cache version, quantizer ABI, checkpoint id, TP world
size, zero-code mode and the FP4 split flag; any change lands in a
different directory.  A hit needs every requested part present with the
exact byte size.  Stores are queued to a background writer thread that
writes each part to a temp file, fsyncs and renames it (so a crash never
leaves a truncated part that looks valid).
"""
from __future__ import annotations

import hashlib
import json
import os
import queue
import threading
from typing import Dict, Optional

import torch

from .fsutil import atomic_write_bytes, atomic_write_json, read_json
from .identity import identity_fields

CACHE_VERSION = 2


class PlanesCache:
    def __init__(self, root: str, ckpt_id: Optional[str], tp_world: int = 1, tp_rank: int = 0,
                 fp4_split: bool = False, background: bool = True):
        self.meta = dict(version=CACHE_VERSION, world=tp_world, fp4_split=bool(fp4_split), **identity_fields(ckpt_id))
        self.enabled = ckpt_id is not None     # an unverified identity is never cached across boots
        key = hashlib.sha256(json.dumps(self.meta, sort_keys=True, separators=(",", ":")).encode()).hexdigest()[:20]
        self.base = os.path.join(root, "v2", key)
        self.rank_dir = os.path.join(self.base, f"tp{tp_world}-rank{tp_rank}")
        self.stats = {"hits": 0, "misses": 0, "stored": 0, "write_errors": 0}
        self._q: "queue.Queue" = queue.Queue()
        self._thread = None
        if self.enabled:
            os.makedirs(self.rank_dir, exist_ok=True)
            if read_json(os.path.join(self.base, "meta.json")) != self.meta:
                atomic_write_json(os.path.join(self.base, "meta.json"), self.meta)
            if background:
                self._thread = threading.Thread(target=self._writer, name="planes-cache-writer", daemon=True)
                self._thread.start()

    def _path(self, li: int, part: str) -> str:
        return os.path.join(self.rank_dir, f"layer{li}.{part}.bin")

    def try_load(self, li: int, parts: Dict[str, int]) -> Optional[Dict[str, torch.Tensor]]:
        """parts: name -> expected byte size.  -> name -> uint8 CPU tensor, or None on any miss."""
        if not self.enabled:
            return None
        out = {}
        for name, nbytes in parts.items():
            p = self._path(li, name)
            try:
                if os.path.getsize(p) != nbytes:
                    self.stats["misses"] += 1
                    return None
                with open(p, "rb") as f:
                    out[name] = torch.frombuffer(bytearray(f.read()), dtype=torch.uint8)
            except OSError:
                self.stats["misses"] += 1
                return None
        self.stats["hits"] += 1
        return out

    def store(self, li: int, parts: Dict[str, torch.Tensor]) -> None:
        if not self.enabled:
            return
        blobs = {k: v.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes() for k, v in parts.items()}
        if self._thread is None:
            self._write(li, blobs)
        else:
            self._q.put((li, blobs))

    def _write(self, li, blobs):
        try:
            for name, data in blobs.items():
                atomic_write_bytes(self._path(li, name), data)
            self.stats["stored"] += 1
        except OSError:
            self.stats["write_errors"] += 1

    def _writer(self):
        while True:
            item = self._q.get()
            if item is None:
                self._q.task_done()
                return
            self._write(*item)
            self._q.task_done()

    def flush(self):
        if self._thread is not None:
            self._q.join()

    def close(self):
        if self._thread is not None:
            self._q.put(None)
            self._thread.join()
            self._thread = None
