"""Exhaustive check of the fused all-reduce's buffer protocol (csrc/kernels/symm.cuh).

The protocol: every rank owns recv slots [2 parities][W sources]; in reduction c a
rank's producer stores its partial into slot [c % 2][rank] of EVERY rank (W peer
stores), then publishes flag[rank] = c + 1 on every rank (W flag stores); its consumer
waits until all W flags of its own area reach c + 1 and reads the W slots of parity c % 2.
A rank's steps run in program order (stream order of the producer and consumer kernels,
kept across the step's kernels by the PDL chain -- ``test_pdl_lint_cpu.py``).  The claim
in symm.cuh is that a peer runs at most one reduction ahead, so the parity it overwrites
next is never the one being read.

Since every slot and flag has exactly one writer, a global state is the vector of the
ranks' program counters; the test walks every reachable state (every interleaving of
the ranks' individual loads and stores) and checks each consumer load sees the partial
of its own reduction.  Two broken variants (one parity; publishing before the stores)
must be caught, which shows the search can see a violation."""
from typing import List, Optional, Tuple

import pytest


def _program(rank: int, W: int, n_calls: int, publish_first: bool) -> List[tuple]:
    ops = []
    for c in range(n_calls):
        stores = [("store", c, dst) for dst in range(W)]
        flags = [("flag", c, dst) for dst in range(W)]
        ops += (flags + stores) if publish_first else (stores + flags)
        ops.append(("wait", c, None))
        ops += [("load", c, src) for src in range(W)]
    return ops


def explore(W: int, n_calls: int, parities: int = 2, publish_first: bool = False) -> Optional[Tuple]:
    """-> None if no reachable state breaks the protocol, else (rank, op, pcs)."""
    progs = [_program(r, W, n_calls, publish_first) for r in range(W)]
    n_ops = len(progs[0])

    def done_before(r: int, pc: int, kind: str, c: int, dst) -> bool:
        """Has rank r, at program counter pc, executed the op (kind, c, dst)?"""
        return progs[r].index((kind, c, dst)) < pc

    def slot_content(pcs, dst: int, parity: int, src: int) -> Optional[int]:
        """Reduction whose partial src last stored into dst's slot [parity][src]."""
        last = None
        for c in range(n_calls):
            if c % parities == parity and done_before(src, pcs[src], "store", c, dst):
                last = c
        return last

    def flag(pcs, dst: int, src: int) -> int:
        v = 0
        for c in range(n_calls):
            if done_before(src, pcs[src], "flag", c, dst):
                v = c + 1
        return v

    seen = set()
    stack = [tuple([0] * W)]
    while stack:
        pcs = stack.pop()
        if pcs in seen:
            continue
        seen.add(pcs)
        for r in range(W):
            pc = pcs[r]
            if pc == n_ops:
                continue
            kind, c, arg = progs[r][pc]
            if kind == "wait" and any(flag(pcs, r, s) < c + 1 for s in range(W)):
                continue                                  # blocked
            if kind == "load" and slot_content(pcs, r, c % parities, arg) != c:
                return (r, (kind, c, arg), pcs)
            nxt = list(pcs)
            nxt[r] += 1
            stack.append(tuple(nxt))
    assert tuple([n_ops] * W) in seen, "the protocol deadlocked"
    return None


@pytest.mark.parametrize("W,n_calls", [(2, 5), (3, 4), (4, 3)])
def test_two_parity_protocol_is_safe(W, n_calls):
    assert explore(W, n_calls) is None


def test_single_parity_is_caught():
    bad = explore(2, 3, parities=1)
    assert bad is not None and bad[1][0] == "load"


def test_publish_before_store_is_caught():
    bad = explore(2, 2, publish_first=True)
    assert bad is not None and bad[1][0] == "load"
