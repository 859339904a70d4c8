"""Prefix sharing in the paged block manager: chain-hashed full prompt blocks, shared
blocks reference-counted, the last matched block copied, unused registered blocks kept
and evicted least-recently-used, and every block accounted for after any sequence of
requests."""
import random

import pytest

from vllm_moet_b200.engine.kv_manager import BlockManager

B = 4          # block size for the tests


def test_shared_prefix_blocks_and_copy_on_write():
    bm = BlockManager(40, block_size=B, prefix_caching=True)
    p1 = list(range(100, 114))                       # 14 tokens: 3 full blocks, the 3rd ends before the end
    t1, m, cow = bm.allocate_with_prefix("a", 20, p1)
    assert m == 0 and cow is None and len(t1) == 5
    bm.register("a", p1)
    assert len(bm.by_key) == 3
    p2 = p1[:12] + [7, 8, 9]
    t2, m, cow = bm.allocate_with_prefix("b", 20, p2)
    assert m == 12 and t2[:2] == t1[:2] and cow == (t1[2], t2[2]) and t2[2] != t1[2]
    assert bm.ref[t1[0]] == 2
    bm.copied("b")
    bm.check_invariants()
    bm.release("a")
    bm.release("b")
    bm.check_invariants()
    assert set(bm.cached) == set(t1[:3]) and bm.num_free == 39


def test_no_sharing_of_the_block_that_ends_the_prompt():
    bm = BlockManager(20, block_size=B, prefix_caching=True)
    p = list(range(8))                                 # exactly 2 blocks
    bm.allocate_with_prefix("a", 12, p)
    bm.register("a", p)
    assert len(bm.by_key) == 1                        # block 2 ends the prompt: not registered
    _, m, _ = bm.allocate_with_prefix("b", 12, p)     # at least one token is always computed
    assert m == 4


def test_lru_eviction_of_cached_blocks():
    bm = BlockManager(7, block_size=B, prefix_caching=True)    # 6 usable blocks
    pa, pb = list(range(9)), list(range(50, 59))
    bm.allocate_with_prefix("a", 9, pa); bm.register("a", pa); bm.release("a")
    bm.allocate_with_prefix("b", 9, pb); bm.register("b", pb); bm.release("b")
    assert len(bm.cached) == 4 and bm.num_free == 6
    bm.allocate("c", 4 * B)                           # needs 4: the 2 free + the 2 oldest cached (a's)
    assert bm.stats["evicted"] == 2 and bm.can_allocate(1, pb) and not bm._match(pa)[0]
    bm.check_invariants()
    with pytest.raises(MemoryError):
        bm.allocate("d", 3 * B)


def test_random_sequences_keep_the_invariants():
    rng = random.Random(0)
    bm = BlockManager(60, block_size=B, prefix_caching=True)
    live = {}
    prefixes = [[rng.randrange(1000) for _ in range(12)] for _ in range(3)]
    for step in range(400):
        if live and (rng.random() < 0.45 or len(live) > 6):
            rid = rng.choice(sorted(live))
            bm.release(rid)
            del live[rid]
        else:
            p = rng.choice(prefixes)[: rng.randrange(1, 13)] + [rng.randrange(1000) for _ in range(rng.randrange(1, 9))]
            rid = f"r{step}"
            n = len(p) + 5
            if not bm.can_allocate(n, p):
                continue
            table, m, cow = bm.allocate_with_prefix(rid, n, p)
            assert m < len(p) and m % B == 0 and len(table) == bm.blocks_needed(n)
            if cow:
                bm.copied(rid)
            bm.register(rid, p)
            live[rid] = p
        bm.check_invariants()
    assert bm.stats["hit_blocks"] > 0
    for rid in list(live):
        bm.release(rid)
    bm.check_invariants()
    assert bm.num_free == 59


def test_colliding_digest_never_maps_another_prompts_blocks(monkeypatch):
    """Even with a digest that collides for every chain, a lookup only hits blocks whose
    tokens equal the prompt's (and whose whole prefix matched before them)."""
    monkeypatch.setattr(BlockManager, "_digest", staticmethod(lambda prev, toks: b"same"))
    bm = BlockManager(40, block_size=B, prefix_caching=True)
    p1 = [1, 2, 3, 4, 5, 6, 7, 8, 9]
    bm.allocate_with_prefix("a", 12, p1)
    bm.register("a", p1)
    p2 = [9, 9, 9, 9, 5, 6, 7, 8, 9]                  # block 1 equal, block 0 not: no hit at all
    _, m, cow = bm.allocate_with_prefix("b", 12, p2)
    assert m == 0 and cow is None
    p3 = [1, 2, 3, 4, 5, 6, 7, 0, 9]                  # block 0 equal, block 1 not: only block 0
    _, m, _ = bm.allocate_with_prefix("c", 12, p3)
    assert m == 4
    bm.check_invariants()
