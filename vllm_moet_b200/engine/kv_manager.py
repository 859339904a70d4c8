"""Paged KV block manager (64-token blocks), with prefix sharing.

A request reserves every block it can reach (prompt + max_tokens + the
speculative lookahead) at admission, so a sequence's block table never
changes while its decode graph replays -- there is no per-step allocation
and no host round trip for paging.  Blocks return to the free list when the
request finishes.

Prefix caching (``enable_prefix_caching``): a block whose 64 positions are all
prompt tokens is registered under a chain key (a SHA-256 digest of the earlier blocks and its
own tokens), so a later prompt with the same leading blocks maps them into its
table instead of recomputing them.  Shared blocks are reference-counted; a
registered block whose last user finished stays cached, reclaimable
least-recently-used when the free list runs dry.  The last matched block is not
shared but copied (``cow``): the position before the first new token is computed
again -- the MTP module's entry there depends on the next prompt token, which
differs between requests -- so it must be written into a block of the request's
own.
"""
from __future__ import annotations

import hashlib
import struct
from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int = 64, reserved: int = 1, prefix_caching: bool = False):
        # block 0.. reserved-1 are never handed out (padding rows point there)
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.free: List[int] = list(range(num_blocks - 1, reserved - 1, -1))
        self.owned: Dict[str, List[int]] = {}
        self.prefix_caching = prefix_caching
        self.ref: Dict[int, int] = {}                       # block -> users (shared or registered blocks)
        self.key_of: Dict[int, tuple] = {}                  # registered block -> its chain key
        self.by_key: Dict[tuple, int] = {}
        self.cached: "OrderedDict[int, None]" = OrderedDict()   # registered, unused (LRU order)
        self.stats = {"hit_blocks": 0, "lookups": 0, "evicted": 0}
        self._cow_pending: Dict[str, int] = {}              # request -> copy source still referenced

    def blocks_needed(self, n_tokens: int) -> int:
        return -(-n_tokens // self.block_size)

    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.cached)

    def _need(self, n_tokens: int, hit: List[int]) -> Tuple[int, int]:
        """-> (blocks to take from the pool, blocks available) for a request matching `hit`."""
        n = self.blocks_needed(n_tokens)
        if not hit:
            return n, self.num_free
        # shared blocks need no allocation; matched blocks leave the cached pool while in use
        return n - (len(hit) - 1), self.num_free - sum(1 for b in hit if b in self.cached)

    def can_allocate(self, n_tokens: int, prompt: Optional[Sequence[int]] = None) -> bool:
        need, avail = self._need(n_tokens, self._match(prompt)[0])
        return need <= avail

    # ------------------------------------------------------------------ prefix keys
    @staticmethod
    def _digest(prev: bytes, tokens: tuple) -> bytes:
        """SHA-256 of the chain so far and one block's tokens (collision resistant: a client
        cannot craft a prompt whose key lands on another prompt's cached blocks)."""
        h = hashlib.sha256(prev)
        h.update(struct.pack(f"<{len(tokens)}q", *tokens))
        return h.digest()

    def _keys(self, prompt: Sequence[int]) -> List[tuple]:
        """Chain keys of the prompt's full blocks: (digest of every earlier block, the block's
        own tokens).  The tokens are part of the key, so a hit compares them exactly; the
        digest ties the block to its whole prefix."""
        b, keys, prev = self.block_size, [], b""
        for i in range(len(prompt) // b):
            toks = tuple(int(t) for t in prompt[i * b:(i + 1) * b])
            keys.append((prev, toks))
            prev = self._digest(prev, toks)
        return keys

    def _match(self, prompt: Optional[Sequence[int]]) -> Tuple[List[int], List[tuple]]:
        """-> (registered blocks matching the prompt's leading full blocks, all its keys).
        At least one prompt token is always left to compute."""
        if prompt is None or not self.prefix_caching:
            return [], []
        keys = self._keys(prompt)
        hit = []
        for i, k in enumerate(keys):
            if (i + 1) * self.block_size >= len(prompt):
                break
            blk = self.by_key.get(k)
            if blk is None:
                break
            hit.append(blk)
        return hit, keys

    def _pop_free(self) -> int:
        if self.free:
            return self.free.pop()
        blk, _ = self.cached.popitem(last=False)            # least recently used cached block
        key = self.key_of.pop(blk)
        del self.by_key[key]
        self.ref.pop(blk, None)
        self.stats["evicted"] += 1
        return blk

    # ------------------------------------------------------------------ allocation
    def allocate(self, req_id: str, n_tokens: int) -> List[int]:
        n = self.blocks_needed(n_tokens)
        if n > self.num_free:
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {self.num_free} free")
        blocks = [self._pop_free() for _ in range(n)]
        self.owned[req_id] = blocks
        return blocks

    def allocate_with_prefix(self, req_id: str, n_tokens: int, prompt: Sequence[int]):
        """-> (block table, cached tokens m, (source block, destination block) to copy or
        None).  Positions [0, m - 1) are read from shared blocks; the request computes
        from position m - 1 on (m = 0: from 0, nothing shared)."""
        hit, _ = self._match(prompt)
        self.stats["lookups"] += 1
        n = self.blocks_needed(n_tokens)
        if not hit:
            return self.allocate(req_id, n_tokens), 0, None
        shared = hit[:-1]
        need, avail = self._need(n_tokens, hit)
        if need > avail:
            raise MemoryError(f"KV cache exhausted: need {need} blocks, {avail} free")
        for b in shared:                                     # take a reference first (no eviction of them)
            self.cached.pop(b, None)
            self.ref[b] = self.ref.get(b, 0) + 1
        self.cached.pop(hit[-1], None)                       # keep the copy source alive during the copy
        self.ref[hit[-1]] = self.ref.get(hit[-1], 0) + 1
        own = [self._pop_free() for _ in range(n - len(shared))]
        self.owned[req_id] = list(shared) + own
        self.stats["hit_blocks"] += len(hit)
        self._cow_pending[req_id] = hit[-1]
        return list(shared) + own, len(hit) * self.block_size, (hit[-1], own[0])

    def copied(self, req_id: str) -> None:
        """The copy-on-write source of `req_id` has been copied: drop its extra reference."""
        src = self._cow_pending.pop(req_id, None)
        if src is not None:
            self._unref(src)

    def register(self, req_id: str, prompt: Sequence[int]) -> None:
        """After the prefill: make this request's full prompt blocks available for sharing."""
        if not self.prefix_caching:
            return
        blocks = self.owned.get(req_id, [])
        for i, k in enumerate(self._keys(prompt)):
            # a block ending at the prompt's end is not shared: the MTP entry of its last
            # position depends on the first generated token, not on a prompt token
            if i >= len(blocks) or (i + 1) * self.block_size >= len(prompt):
                break
            b = blocks[i]
            if k in self.by_key or b in self.key_of:
                continue
            self.by_key[k], self.key_of[b] = b, k
            self.ref[b] = self.ref.get(b, 0) + 1             # the request's own use

    def _unref(self, b: int) -> None:
        if b not in self.ref:
            self.free.append(b)
            return
        self.ref[b] -= 1
        if self.ref[b] <= 0:
            del self.ref[b]
            if b in self.key_of:
                self.cached[b] = None                        # stays cached, most recently used
            else:
                self.free.append(b)

    def release(self, req_id: str) -> None:
        self.copied(req_id)
        for b in self.owned.pop(req_id, []):
            self._unref(b)

    def check_invariants(self) -> None:
        """Every block is in exactly one place: free, cached (unused), or used."""
        used = [b for bl in self.owned.values() for b in bl]
        free, cached = set(self.free), set(self.cached)
        assert len(free) == len(self.free) and not free & cached, "free / cached overlap"
        assert not (set(used) & free) and not (set(used) & cached), "a used block is free or cached"
        for b, n in self.ref.items():
            assert n > 0 and b not in free
        for b in cached:
            assert b in self.key_of and b not in self.ref
