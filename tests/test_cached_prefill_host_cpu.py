"""Host-side arithmetic of the GPU runner's cached-prefix prefill and prefill chunks,
run on CPU against a stub that records what the kernels would be given: the rows are
the suffix tokens at their true positions, slots land in the right blocks, the MTP pass
reads the next prompt token (the first generated one on each prompt's last row), and
the decode state starts at the full prompt length."""
import types

import torch

from vllm_moet_b200.engine.gpu_runner import KV_BLOCK, DecodeState, NativeRunner


class Stub:
    def __init__(self, k=2, H=8, V=32):
        self.dev, self.k, self.last_stage = torch.device("cpu"), k, True
        self.cfg = types.SimpleNamespace(hidden=H, rms_eps=1e-6)
        self.mw = types.SimpleNamespace(final_norm=torch.ones(H))
        self.V, self.calls = V, []
        self.ws = types.SimpleNamespace(get=lambda name, shape, dtype: torch.zeros(shape, dtype=dtype))
        self.C = types.SimpleNamespace(rmsnorm_quant=lambda *a: None)
        self.ws_prefill = self.ws
        self.cached_flash_min = 1
        self.hcn = 1
        self.dcp = None
        self.eagle = None

    def _slots(self, bt, seq, pos):
        return NativeRunner._slots(self, bt, seq, pos)

    def _lpos(self, pos):
        return None

    def _key_rows(self, ctx, ends):
        return NativeRunner._key_rows(self, ctx, ends)

    def _main(self, toks, ctx):
        self.calls.append(("main", toks.clone(), ctx))
        return torch.zeros(ctx.T, self.cfg.hidden)

    def _final(self, x, _, tag):
        lg = torch.zeros(x.shape[0], self.V)
        lg[:, 7] = 1.0
        return x, lg

    def _argmax(self, logits, out):
        out.copy_(logits.argmax(-1).to(out.dtype))

    def _mtp(self, h, nxt, ctx, rows=None):
        self.calls.append(("mtp", nxt.clone(), ctx))
        n = h.shape[0] if rows is None else len(rows)
        lg = torch.zeros(n, self.V)
        lg[:, 9] = 1.0
        return torch.zeros(n, self.cfg.hidden), lg

    def _pp_broadcast_state(self, st):
        pass

    def check_status(self, where):
        pass


def test_cached_prefill_rows_and_slots():
    r = Stub()
    st = DecodeState(2, 2, 4, "cpu")
    p0, p1 = list(range(100, 180)), list(range(200, 230))     # 80 and 30 tokens
    bt = [[5, 6, 0, 0], [7, 0, 0, 0]]
    first = NativeRunner._prefill(r, [p0, p1], bt, [0, 1], st, starts=[63, 0])
    (_, toks, ctx), (_, nxt, mctx) = r.calls[0], r.calls[1]
    assert ctx.mode == "cached" and ctx.T == (80 - 63) + 30
    assert toks.tolist() == p0[63:] + p1
    assert ctx.pos.tolist() == list(range(63, 80)) + list(range(30))
    blocks = [bt[s][p // KV_BLOCK] for s, p in zip(ctx.seq.tolist(), ctx.pos.tolist())]
    assert (ctx.slot // KV_BLOCK).tolist() == blocks and (ctx.slot % KV_BLOCK).tolist() == [p % KV_BLOCK for p in ctx.pos.tolist()]
    assert nxt.tolist() == p0[64:] + [7] + p1[1:] + [7]          # the first generated token closes each prompt
    assert first.tolist() == [7, 7] and st.seq_pos.tolist() == [80, 30]
    # flash path: every key row of each sequence (cached prefix + suffix), in position order
    assert ctx.cu_k.tolist() == [0, 80, 110]
    want = [bt[0][q // KV_BLOCK] * KV_BLOCK + q % KV_BLOCK for q in range(80)] + [7 * KV_BLOCK + q for q in range(30)]
    assert ctx.kv_idx.tolist() == want
    assert st.tokens[:, 0].tolist() == [7, 7] and st.tokens[:, 1].tolist() == [9, 9]


def test_prefill_chunk_rows():
    r = Stub()
    p = list(range(300, 400))
    NativeRunner.prefill_chunk(r, p, [3, 4, 0, 0], 40, 70)
    (_, toks, ctx), (_, nxt, _) = r.calls
    assert ctx.mode == "cached" and toks.tolist() == p[40:70] and ctx.pos.tolist() == list(range(40, 70))
    assert nxt.tolist() == p[41:71]                                # every MTP row's next token is a prompt token
    assert (ctx.slot // KV_BLOCK).tolist() == [3 if q < 64 else 4 for q in range(40, 70)]
    assert ctx.cu_k.tolist() == [0, 70]
    assert ctx.kv_idx.tolist() == [(3 if q < 64 else 4) * KV_BLOCK + q % KV_BLOCK for q in range(70)]
    r.cached_flash_min = 31              # a 30-row chunk stays on absorbed attention
    r.calls.clear()
    NativeRunner.prefill_chunk(r, p, [3, 4, 0, 0], 40, 70)
    assert r.calls[0][2].kv_idx is None
    r.calls.clear()
    NativeRunner.prefill_chunk(r, p, [3, 4, 0, 0], 0, 16)
    assert r.calls[0][2].mode == "prefill" and r.calls[0][2].cu_seqlens.tolist() == [0, 16]
