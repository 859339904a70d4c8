"""Paged KV block manager (64-token blocks).

A request reserves every block it can reach (prompt + max_tokens + the
speculative lookahead) at admission, so a sequence's block table never
changes while its decode graph replays -- there is no per-step allocation
and no host round trip for paging.  Blocks return to the free list when the
request finishes.
"""
from __future__ import annotations

from typing import Dict, List


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int = 64, reserved: int = 1):
        # block 0.. reserved-1 are never handed out (padding rows point there)
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.free: List[int] = list(range(num_blocks - 1, reserved - 1, -1))
        self.owned: Dict[str, List[int]] = {}

    def blocks_needed(self, n_tokens: int) -> int:
        return -(-n_tokens // self.block_size)

    def can_allocate(self, n_tokens: int) -> bool:
        return self.blocks_needed(n_tokens) <= len(self.free)

    def allocate(self, req_id: str, n_tokens: int) -> List[int]:
        n = self.blocks_needed(n_tokens)
        if n > len(self.free):
            raise MemoryError(f"KV cache exhausted: need {n} blocks, {len(self.free)} free")
        blocks = [self.free.pop() for _ in range(n)]
        self.owned[req_id] = blocks
        return blocks

    def release(self, req_id: str) -> None:
        for b in self.owned.pop(req_id, []):
            self.free.append(b)

    @property
    def num_free(self) -> int:
        return len(self.free)
