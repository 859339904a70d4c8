"""Host arithmetic of the GPU runner's decode context parallelism, on CPU: every position
has exactly one owner, each rank keeps its positions densely in position order through its
own block table, the local counts match, and a prefill writes only the owned rows."""
import pytest
import torch

from vllm_moet_b200.engine.gpu_runner import KV_BLOCK, NativeRunner, dcp_local_count, dcp_slots


@pytest.mark.parametrize("W,I", [(1, 1), (2, 1), (3, 2), (2, 64), (4, 5)])
def test_dcp_ownership_and_local_slots(W, I):
    N = 700
    pos = torch.arange(N)
    bts = [torch.randperm(50)[:20].view(1, 20) for _ in range(W)]     # each rank's own block table
    owners = torch.full((N,), -1)
    for r in range(W):
        sl = dcp_slots(bts[r], torch.zeros(N, dtype=torch.long), pos, W, r, I)
        own = sl >= 0
        assert (owners[own] == -1).all()
        owners[own] = r
        assert own.tolist() == [((p // I) % W) == r for p in range(N)]
        # local index = order among the rank's positions; slot = its block-table entry
        lp = torch.arange(int(own.sum()))
        want = bts[r][0, lp // KV_BLOCK] * KV_BLOCK + lp % KV_BLOCK
        assert sl[own].tolist() == want.tolist()
        for n in (0, 1, I, I * W - 1, I * W, 333, N):
            assert dcp_local_count(n, W, r, I) == int(((pos[:n] // I) % W == r).sum())
            assert int(dcp_local_count(torch.tensor(n), W, r, I)) == dcp_local_count(n, W, r, I)
    assert (owners >= 0).all()


class _Stub:
    """Records the prefill context the runner builds (no kernels)."""

    def __init__(self, dcp):
        import types
        self.dev, self.k, self.last_stage, self.hcn, self.cached_flash_min = torch.device("cpu"), 0, True, 1, 128
        self.dcp = dcp
        self.cfg = types.SimpleNamespace(hidden=8, rms_eps=1e-6)
        self.ws = types.SimpleNamespace(get=lambda name, shape, dtype: torch.zeros(shape, dtype=dtype))
        self.ws_prefill = self.ws
        self.C = types.SimpleNamespace()
        self.calls = []

    def _slots(self, bt, seq, pos):
        return NativeRunner._slots(self, bt, seq, pos)

    def _main(self, toks, ctx):
        self.calls.append(ctx)
        return torch.zeros(ctx.T, 8)

    def _final(self, x, _, tag):
        lg = torch.zeros(x.shape[0], 16)
        lg[:, 3] = 1.0
        return x, lg

    def _argmax(self, logits, out):
        out.copy_(logits.argmax(-1).to(out.dtype))

    def _pp_broadcast_state(self, st):
        pass


def test_dcp_prefill_writes_owned_rows_only():
    from vllm_moet_b200.engine.gpu_runner import DecodeState
    for r in range(2):
        st = DecodeState(1, 0, 4, "cpu")
        stub = _Stub((None, 2, r, 1))
        NativeRunner._prefill(stub, [list(range(100, 230))], [[7, 9, 0, 0]], [0], st)
        ctx = stub.calls[0]
        own = ctx.slot >= 0
        assert own.tolist() == [p % 2 == r for p in range(130)]
        assert ctx.slot[own].tolist() == [(7 if i < 64 else 9) * KV_BLOCK + i % 64 for i in range(65)]
