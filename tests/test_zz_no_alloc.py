"""The allocation-free pair-list builder, called through its C symbol.

`moet_build_pairs_noalloc` serves callers that cannot call cudaMalloc (a
C/C++ host without PyTorch's allocator, or a process whose free HBM is
already committed to the KV cache and expert pools).  Its output must match
the regular `build_pairs` op on the same routing, call after call.  Row order
inside one expert (and so which of its pairs a token lands in) comes from
atomics in both entry points, so tokens are compared per expert as a
multiset; the pair list itself and every other output must be equal.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_ROUTINGS = 65536


@pytest.fixture(scope="module")
def lib():
    from vllm_moet_b200.ops import native
    mod = native()
    so = ctypes.CDLL(mod.__file__)
    fn = so.moet_build_pairs_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    return mod, fn


def _outputs(R, P):
    return (torch.full((R,), -7, dtype=torch.int32, device=DEV), torch.full((R,), -7, dtype=torch.int32, device=DEV),
            torch.full((P, 4), -7, dtype=torch.int32, device=DEV), torch.zeros(1, dtype=torch.int32, device=DEV),
            torch.zeros(1, dtype=torch.int32, device=DEV))


def _call(fn, ids, E, MB, outs):
    stok, posof, pairs, npairs, status = outs
    T, k = ids.shape
    rc = fn(ids.data_ptr(), T, k, E, MB, stok.data_ptr(), posof.data_ptr(), pairs.data_ptr(), pairs.shape[0],
            npairs.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc


def _canonical(ids, outs):
    stok, posof, pairs, npairs, status = (t.cpu() for t in outs)
    T, k = ids.shape
    n = int(npairs)
    segs = [tuple(pr[:3]) for pr in pairs[:n].tolist()]
    tokens_of = {}
    for e, start, rows in segs:
        tokens_of.setdefault(e, []).extend(stok[start:start + rows].tolist())
    tokens_of = {e: sorted(v) for e, v in tokens_of.items()}
    # each routing points at a row of its own expert's segment holding its token
    by_expert = {}
    for e, s, m in segs:
        by_expert.setdefault(e, []).append((s, m))
    ids_l, pos_l, tok_l = ids.cpu().view(-1).tolist(), posof.tolist(), stok.tolist()
    for r in range(T * k):
        p = pos_l[r]
        assert tok_l[p] == r // k
        assert any(s <= p < s + m for s, m in by_expert.get(ids_l[r], []))
    return n, segs, tokens_of, int(status)


@pytest.mark.parametrize("T,k,E,MB", [(1, 8, 256, 8), (37, 8, 64, 8), (96, 8, 256, 16), (8192, 8, 256, 32)])
def test_noalloc_matches_build_pairs(lib, T, k, E, MB):
    mod, fn = lib
    g = torch.Generator().manual_seed(T + E)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).int().to(DEV)
    R = T * k
    P = R // MB + min(E, R)
    ref = _outputs(R, P)
    rank = torch.empty(R, dtype=torch.int32, device=DEV)
    mod.build_pairs(ids, E, MB, rank, ref[0], ref[1], ref[2], ref[3], ref[4])
    torch.cuda.synchronize()
    want = _canonical(ids, ref)
    for _ in range(2):  # two calls in a row share the static scratch
        outs = _outputs(R, P)
        assert _call(fn, ids, E, MB, outs) == 0
        assert _canonical(ids, outs) == want


def test_noalloc_rejects_oversize_and_bad_args(lib):
    _, fn = lib
    T, k = MAX_ROUTINGS // 8 + 1, 8
    ids = torch.zeros(T, k, dtype=torch.int32, device=DEV)
    outs = _outputs(1, 1)
    assert _call(fn, ids, 256, 32, outs) == -2
    assert int(outs[3]) == 0 and bool((outs[0] == -7).all())  # nothing was launched
    small = torch.zeros(4, 8, dtype=torch.int32, device=DEV)
    assert _call(fn, small, 256, 8, _outputs(32, 1)) == -1   # pairs buffer too small


def test_noalloc_rejects_misaligned_pairs(lib):
    """The pair records are 16-byte stores: a pairs pointer off a 16-byte boundary is refused
    on the host before anything is launched."""
    _, fn = lib
    ids = torch.zeros(4, 8, dtype=torch.int32, device=DEV)
    stok, posof, pairs, npairs, status = _outputs(32, 64)
    flat = pairs.view(-1)
    rc = fn(ids.data_ptr(), 4, 8, 256, 8, stok.data_ptr(), posof.data_ptr(), flat[1:].data_ptr(), 63,
            npairs.data_ptr(), status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == -1
    assert int(npairs) == 0 and bool((pairs == -7).all())


def test_noalloc_out_of_range_id_sets_caller_zeroed_status(lib):
    """An expert id >= num_experts sets status to 1, as build_pairs does, and the routing is
    counted under expert 0; status is never cleared by the call (the caller zeroes it)."""
    mod, fn = lib
    E, MB = 16, 8
    ids = torch.tensor([[3, 20], [0, 5]], dtype=torch.int32, device=DEV)
    R, P = 4, 4 // MB + min(E, 4)
    ref = _outputs(R, P)
    rank = torch.empty(R, dtype=torch.int32, device=DEV)
    mod.build_pairs(ids, E, MB, rank, ref[0], ref[1], ref[2], ref[3], ref[4])
    outs = _outputs(R, P)
    assert _call(fn, ids, E, MB, outs) == 0
    assert int(outs[4]) == 1 and int(ref[4]) == 1
    assert int(outs[3]) == int(ref[3]) == 3          # experts 0 (two rows), 3 and 5
    # a second, valid call leaves the caller's status word as it found it
    ok = torch.tensor([[1, 2]], dtype=torch.int32, device=DEV)
    outs2 = _outputs(2, 2 // MB + 2)
    outs2[4].fill_(1)
    assert _call(fn, ok, E, MB, outs2) == 0
    assert int(outs2[4]) == 1 and int(outs2[3]) == 2
