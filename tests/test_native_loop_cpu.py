"""The GPU engine's decode loop (`LLM._run_native`) on the CPU, with a fake native runner.

The fake runner stands in for the CUDA kernels with a deterministic model: the token after
`t` at position `p` is f(t, p).  Its decode step verifies the row's drafts against f the
way the captured graph does (accepted drafts + one correction token, `n_acc`), and its
drafts are right on most steps and wrong on some, so acceptance varies.  Whatever the
batching, joins, aborts or bucket growth, every request must come out as the chain of f
from its prompt.  Only the host loop is under test here; the kernels are tested on GPUs.
"""
import itertools
import math
import types

import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import EngineConfig, MoetConfig, tiny_config
from vllm_moet_b200.engine.gpu_runner import DecodeState, NativeRunner
from vllm_moet_b200.engine.kv_manager import BlockManager
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.engine.tokenizer import ByteTokenizer

V = 1024


def f(t: int, p: int) -> int:
    return (int(t) * 7 + int(p) * 3 + 11) % (V - 3) + 3


def chain(prompt, n):
    out, t, p = [], prompt[-1], len(prompt) - 1
    for _ in range(n):
        t = f(t, p)
        out.append(t)
        p += 1
    return out


class FakeRunner:
    def __init__(self, k):
        self.k, self.graphs, self.steps, self.nodraft_steps = k, {}, 0, 0
        self.nodraft_graphs = {}
        self.ws_prefill = self
        self.logits = {}
        self.starts_log, self.copies, self.chunks = [], [], []

    def copy_block(self, src, dst):
        self.copies.append((src, dst))

    def prefill_chunk(self, prompt, bt, start, end):
        self.chunks.append((start, end))

    def _drafts(self, t, p):
        d = []
        for j in range(self.k):
            t = f(t, p + j)
            d.append(t)
        if self.steps % 3 == 1 and d:          # a wrong draft now and then
            d[-1] = (d[-1] + 1) % V
        return d

    def prefill(self, prompts, bts, rows, st, sample=False, starts=None):
        self.starts_log.append(list(starts) if starts is not None else [0] * len(prompts))
        firsts = []
        for pr, r in zip(prompts, rows):
            t0 = f(pr[-1], len(pr) - 1)
            if sample:                                     # the first token drawn as the GPU prefill does
                from vllm_moet_b200.engine.gpu_runner import NativeRunner
                t0 = int(NativeRunner._sample_first(self, st, [r], self._onehot(t0)[None], [len(pr)])[0])
            st.tokens[r] = torch.tensor([t0] + self._drafts(t0, len(pr)), dtype=torch.int32)
            st.seq_pos[r] = len(pr)
            firsts.append(t0)
        self.prefill_logits = torch.stack([self._onehot(t) for t in firsts])
        return torch.tensor(firsts)

    def get(self, name, shape, dtype):                     # ws_prefill.get("main.logits", ...)
        return self.prefill_logits

    @staticmethod
    def _onehot(t):
        x = torch.zeros(V)
        x[int(t)] = 10.0
        return x

    def decode_body(self, st, sample=False, draft=True):
        self.steps += 1
        kp1 = self.k + 1
        lg = torch.zeros(st.B * kp1, V)
        if sample:
            return self._decode_sampled(st)
        if not draft:                     # the no-draft step: one row per sequence, stale drafts kept
            self.nodraft_steps += 1
            for r in range(st.B):
                if not int(st.active[r]):
                    continue
                toks, p = st.tokens[r].tolist(), int(st.seq_pos[r])
                nxt = f(toks[0], p)
                st.out_tokens[r] = torch.tensor([nxt] + [-1] * self.k, dtype=torch.int32)
                st.n_acc[r] = 0
                st.tokens[r] = torch.tensor([nxt] + toks[1:], dtype=torch.int32)
                st.seq_pos[r] = p + 1
            self.logits[st.B] = lg
            return
        for r in range(st.B):
            if not int(st.active[r]):
                continue
            toks, p = st.tokens[r].tolist(), int(st.seq_pos[r])
            tg = [f(toks[j], p + j) for j in range(kp1)]
            a = 0
            while a < self.k and toks[a + 1] == tg[a]:
                a += 1
            st.out_tokens[r] = torch.tensor(tg, dtype=torch.int32)
            st.n_acc[r] = a
            for j in range(kp1):
                lg[r * kp1 + j] = self._onehot(tg[j])
            nxt = tg[a]
            st.tokens[r] = torch.tensor([nxt] + self._drafts(nxt, p + a + 1), dtype=torch.int32)
            st.seq_pos[r] = p + a + 1
        self.logits[st.B] = lg

    def _decode_sampled(self, st):
        """The sampling variant: the verify logits of the model, then the GPU runner's own
        `_sample_verify` (the graph-safe sampler) and mtp_finalize's bookkeeping."""
        from vllm_moet_b200.engine.gpu_runner import NativeRunner
        kp1 = self.k + 1
        lg = torch.zeros(st.B * kp1, V)
        for r in range(st.B):
            toks, p = st.tokens[r].tolist(), int(st.seq_pos[r])
            for j in range(kp1):
                lg[r * kp1 + j] = self._onehot(f(toks[j], p + j))
        NativeRunner._sample_verify(self, st, lg)
        self.logits[st.B] = lg
        for r in range(st.B):
            if not int(st.active[r]):
                continue
            a, p = int(st.n_acc[r]), int(st.seq_pos[r])
            nxt = int(st.targets[r, a])
            st.tokens[r] = torch.tensor([nxt] + self._drafts(nxt, p + a + 1), dtype=torch.int32)
            st.seq_pos[r] = p + a + 1

    @staticmethod
    def _full_vocab(logits):                               # one rank: the whole vocabulary
        return logits

    _process = staticmethod(NativeRunner._process)         # the GPU runner's own processing step

    def main_logits(self, B):
        return self.logits.get(B)

    def route_ids(self, B):
        return []

    def check_status(self, where):
        pass


class _Stream:
    def synchronize(self):
        pass


@pytest.fixture
def engine(monkeypatch):
    zeros = torch.zeros

    def zeros_no_pin(*a, pin_memory=False, **kw):
        return zeros(*a, **kw)
    monkeypatch.setattr(torch, "zeros", zeros_no_pin)
    monkeypatch.setattr(torch.cuda, "current_stream", lambda *a, **k: _Stream())

    def make(max_num_seqs=4, k=2, prefix_caching=False, chunk=None):
        llm = object.__new__(LLM)
        cfg = tiny_config()
        llm.cfg, llm.k, llm.device = cfg, k, torch.device("cpu")
        llm.ecfg = EngineConfig(model=cfg, moet=MoetConfig(), max_num_seqs=max_num_seqs, max_model_len=512,
                                num_speculative_tokens=k, cuda_graphs=False)
        llm.max_blocks = -(-(512 + k + 2) // 64)
        llm.blocks = BlockManager(max_num_seqs * llm.max_blocks + 1, prefix_caching=prefix_caching)
        llm.tokenizer = ByteTokenizer(V)
        llm._states, llm._DecodeState, llm._ids = {}, DecodeState, itertools.count()
        llm.cache = llm.delta = llm.gate = llm.routing = llm.timers = None
        llm.spec_guard = llm.affinity = None
        llm._spec_draft = True
        llm._tp_group = llm._pp_group = llm._ep_group = None
        llm._decode_steps, llm.stats = 0, {}
        llm._chunk_budget = chunk
        llm.runner = FakeRunner(k)
        llm._run_torch = types.MethodType(LLM._run_native, llm)    # generate() dispatches by device type
        return llm
    return make


def test_batch_decodes_the_model_chain(engine):
    llm = engine()
    prompts = [[5, 6, 7], [40, 41], [9, 10, 11, 12]]
    lens = [9, 4, 13]
    out = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in lens])
    for o, p, n in zip(out, prompts, lens):
        assert o.outputs[0].token_ids == chain(p, n) and o.outputs[0].finish_reason == "length"
    assert llm.stats["accepted"] > 0
    assert llm.blocks.can_allocate(4 * 512 - 64)          # every request's blocks were released


def test_joins_grow_the_bucket_and_aborts_free_rows(engine):
    llm = engine(max_num_seqs=4)
    ev = {}

    def cb(name):
        return lambda ids, fin, lp=None: ev.setdefault(name, []).append((list(ids), fin))
    step = [0]
    joined = {"j1": [20, 21], "j2": [30, 31, 32], "j3": [50]}

    def between(n_free):
        step[0] += 1
        new = []
        if step[0] == 2:                                  # three requests while the 1-row bucket is busy
            new = [(rid, p, SamplingParams(max_tokens=40 if rid == "j2" else 6, ignore_eos=True), cb(rid))
                   for rid, p in joined.items()]
        return new[:max(0, n_free)], ({"j2"} if step[0] == 4 else set())
    out = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=14, ignore_eos=True), callbacks=[cb("a")],
                       request_ids=["a"], between_steps=between)
    assert out[0].outputs[0].token_ids == chain([5, 6, 7], 14)
    assert 4 in llm._states                               # the batch moved into the 4-row bucket
    for rid in ("j1", "j3"):
        assert sum((ids for ids, _ in ev[rid]), []) == chain(joined[rid], 6) and ev[rid][-1][1] == "length"
    got = sum((ids for ids, _ in ev["j2"]), [])
    assert ev["j2"][-1][1] == "abort" and got == chain(joined["j2"], len(got)) and len(got) < 40


def test_logprobs_read_from_the_verify_rows(engine):
    llm = engine()
    o = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=8, ignore_eos=True, logprobs=1))[0].outputs[0]
    assert len(o.logprobs) == 8
    want = -math.log1p((V - 1) * math.exp(-10.0))         # one-hot logit 10 over V tokens
    for t, d in zip(o.token_ids, o.logprobs):
        assert max(d, key=d.get) == t and abs(d[t] - want) < 1e-4   # the predicting row of each token


def test_gate_promotes_replays_and_logs(engine, tmp_path):
    """The confidence gate in the decode loop: an always-firing gate promotes the step's
    routed experts into a (CPU) delta tier, replays the step from its snapshot and logs
    each evaluation; the replayed steps still give the model's chain."""
    import json
    from vllm_moet_b200.residency import ConfidenceGate
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    from vllm_moet_b200.utils.observability import DeltaTrace, JsonlWriter
    llm = engine()
    L, E, H, I = 2, 8, 64, 64
    sb = delta_layout(H, I)[0]
    llm.delta = DeltaTier([torch.zeros(E, sb, dtype=torch.uint8) for _ in range(L)], H, I, 16, device="cpu",
                          policy="need")
    llm.gate = ConfidenceGate(tau=2.0, fp_max=2)          # max-prob <= 1 < tau: always fires
    llm.delta_trace = DeltaTrace(level=2, every=10 ** 6)
    llm.gate_log = JsonlWriter(str(tmp_path / "gate.jsonl"))
    llm.ecfg.moet.gate_fire_timing = False
    # the fake model routes each row to experts derived from its pending token, in every layer
    llm.runner.route_ids = lambda B, st=None: [torch.tensor([[int(t) % E, (int(t) + 1) % E] for t in
                                                             llm._states[B].tokens[:, 0].tolist()])] * L
    try:
        out = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=10, ignore_eos=True))[0].outputs[0].token_ids
    finally:
        llm.delta.close()
        llm.gate_log.close()
    assert out == chain([5, 6, 7], 10)
    assert llm.delta.stats["gate_replays"] > 0 and llm.delta.stats["fetched_rows"] > 0
    rows = [json.loads(x) for x in (tmp_path / "gate.jsonl").read_text().splitlines()]
    assert len(rows) == llm._decode_steps and rows[0]["fired"] >= 1 and rows[0]["iters"][0]["promoted"] > 0
    assert llm.delta_trace.snapshot(llm.delta)["resident"] > 0


def test_base_cache_misses_are_fetched_and_replayed(engine):
    """The expert-cache branch of the loop: the fake step counts routed experts whose slot
    is -1 into the cache's miss counter (as the expert kernels do); the loop fetches them,
    restores the step's state and replays until the step is miss-free."""
    from vllm_moet_b200.residency import ExpertCache, ReplayEngine, make_store
    from vllm_moet_b200.utils.observability import KpiLogger
    llm = engine()
    L, E, SB = 2, 8, 256
    st_ = make_store("pinned", L, E, SB)
    for li in range(L):
        st_.add_layer(li, torch.randint(0, 256, (E, SB), dtype=torch.uint8))
    cache = ExpertCache(st_, L, E, SB, 10, device="cpu", manager=False)   # one step needs <= 8 of 16
    llm.cache, llm.replay, llm.kpi = cache, ReplayEngine(cache, comm_device="cpu"), KpiLogger(every=10 ** 6)
    route = {}

    def route_ids(B):
        return route.get(B, [None] * L)
    llm.runner.route_ids = route_ids
    real_step = llm.runner.decode_body

    def step_with_routing(st):
        toks = st.tokens[:, 0].clone()
        real_step(st)
        ids = torch.tensor([[int(t) % E, (int(t) + 3) % E] for t in toks.tolist()])
        route[st.B] = [ids] * L
        for li in range(L):
            cache.miss_count += int((cache.slot_table[li, ids.reshape(-1)] < 0).sum())
    llm.runner.decode_body = step_with_routing
    out = llm.generate([[5, 6, 7], [9, 9]], SamplingParams(max_tokens=9, ignore_eos=True))
    assert [o.outputs[0].token_ids for o in out] == [chain([5, 6, 7], 9), chain([9, 9], 9)]
    assert llm.replay.stats["replayed_steps"] > 0 and cache.stats["fetched_rows"] > 0
    assert llm.kpi.snapshot()["replayed_steps"] == llm.replay.stats["replayed_steps"]
    snap = llm.kpi.snapshot()
    assert snap["pool_slots"] == 10 and abs(snap["pool_pct"] - 62.5) < 1e-9   # 10 of 2 x 8 experts
    assert "pool 10 slots = 62.5% of experts" in llm.kpi.line()


def test_spec_guard_and_draft_affinity_on_the_cache_loop(engine):
    """While the expert pool keeps replaying, the spec guard latches drafting off and the loop
    runs the no-draft step (one row per sequence); greedy output is still the model's chain.
    Draft-affinity learns token -> experts from each drafting step and prefetches the next
    step's drafts' experts."""
    from vllm_moet_b200.residency import ExpertCache, ReplayEngine, make_store
    from vllm_moet_b200.residency.control import DraftAffinity, SpecGuard
    from vllm_moet_b200.utils.observability import KpiLogger
    llm = engine()
    L, E, SB = 2, 64, 256          # 128 experts, 40 slots: a step's <= 36 fit, misses keep coming
    st_ = make_store("pinned", L, E, SB)
    for li in range(L):
        st_.add_layer(li, torch.randint(0, 256, (E, SB), dtype=torch.uint8))
    cache = ExpertCache(st_, L, E, SB, 40, device="cpu", manager=False)
    llm.cache, llm.replay, llm.kpi = cache, ReplayEngine(cache, comm_device="cpu"), KpiLogger(every=10 ** 6)
    llm.spec_guard = SpecGuard(alpha=0.6, hi=0.5, lo=0.05, patience=4)
    llm.affinity = DraftAffinity(cache)
    prefetched = []
    real_prefetch = cache.request_prefetch
    cache.request_prefetch = lambda pairs: (prefetched.append(list(pairs)), real_prefetch(pairs))[1]
    route = {}
    llm.runner.route_ids = lambda B: route.get(B, [None] * L)
    real_step = llm.runner.decode_body

    def step_with_routing(st, sample=False, draft=True):
        toks = (st.tokens if draft else st.tokens[:, :1]).clone()
        real_step(st, sample, draft)
        ids = torch.tensor([[int(t) % E, (int(t) * 5 + 3) % E] for t in toks.reshape(-1).tolist()])
        route[st.B] = [ids] * L
        for li in range(L):
            cache.miss_count += int((cache.slot_table[li, ids.reshape(-1)] < 0).sum())
    llm.runner.decode_body = step_with_routing
    prompts = [[5, 6, 7], [9, 9], [100, 3]]
    out = llm.generate(prompts, SamplingParams(max_tokens=24, ignore_eos=True))
    assert [o.outputs[0].token_ids for o in out] == [chain(p, 24) for p in prompts]
    assert llm.runner.nodraft_steps > 0                       # the guard suppressed drafting
    assert llm.runner.steps > llm.runner.nodraft_steps        # and let it resume
    # the learned table drives prefetches of a learned token's non-resident experts
    assert len(llm.affinity.table) > 0
    toks = list(llm.affinity.table)[:8]
    want = {(li, e) for t in toks for li, es in enumerate(llm.affinity.table[t]) for e in es
            if not cache.resident(li, e)}
    n = llm.affinity.prefetch(toks)
    assert n == len(want) and (not want or set(prefetched[-1]) == want)
    assert all(cache.resident(li, e) for li, e in want)


def test_sampling_rows_share_the_batch_with_greedy_rows(engine):
    """temperature > 0 on the GPU loop: the batch runs the sampling variant of the step;
    greedy rows in it still decode the model's chain, a seeded sampling row is reproducible
    and leaves the chain (T = 3 flattens the one-hot logits), and different seeds differ."""
    def run(seed):
        llm = engine()
        sp_s = SamplingParams(max_tokens=12, ignore_eos=True, temperature=3.0, seed=seed)
        sp_g = SamplingParams(max_tokens=12, ignore_eos=True)
        out = llm.generate([[5, 6, 7], [9, 10]], [sp_g, sp_s])
        return [o.outputs[0].token_ids for o in out]
    g1, s1 = run(7)
    g2, s2 = run(7)
    _, s3 = run(8)
    assert g1 == chain([5, 6, 7], 12) and g2 == g1
    assert s1 == s2 and len(s1) == 12 and s1 != chain([9, 10], 12) and s3 != s1


def test_penalties_in_the_gpu_loop(engine):
    """Penalties / logit bias on the GPU loop: the sampling variant processes the verify
    rows (drafts before row j count as generated) with device-side token counts kept by
    the host loop; a repetition penalty breaks the fake model's repetition and a large
    bias forces a token; greedy rows beside them keep the chain."""
    llm = engine()
    forced = SamplingParams(max_tokens=8, ignore_eos=True, logit_bias={77: 50.0})
    out = llm.generate([[5, 6, 7], [9, 10]], [SamplingParams(max_tokens=8, ignore_eos=True), forced])
    assert out[0].outputs[0].token_ids == chain([5, 6, 7], 8)
    assert out[1].outputs[0].token_ids == [77] * 8
    st = llm._states[2]
    assert st.proc is not None and float(st.proc["counts"][1, 77]) == 8.0
    # presence penalty 2 against a bias of 1.5 on token 77: once generated, 77 loses to the model
    pen = SamplingParams(max_tokens=6, ignore_eos=True, logit_bias={77: 11.0}, presence_penalty=2.0)
    got = llm.generate([[9, 10]], pen)[0].outputs[0].token_ids
    assert got[0] == 77 and 77 not in got[1:]


def test_prefix_sharing_in_the_gpu_loop(engine):
    """GPU prefix caching, host side: a second request sharing 2 full blocks (128 tokens)
    maps the first block, copies the second (copy-on-write) and prefills from position
    127; outputs are the model's chain and every block is accounted for at the end."""
    llm = engine(prefix_caching=True)
    prefix = [(7 * i) % 1000 + 3 for i in range(128)]
    a, b = prefix + [5, 6, 7], prefix + [9]
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    assert llm.generate([a], sp)[0].outputs[0].token_ids == chain(a, 6)
    assert llm.runner.starts_log[-1] == [0] and not llm.runner.copies
    assert llm.generate([b], sp)[0].outputs[0].token_ids == chain(b, 6)
    assert llm.runner.starts_log[-1] == [127] and len(llm.runner.copies) == 1
    bm = llm.blocks
    assert bm.stats["hit_blocks"] == 2 and not bm.owned
    bm.check_invariants()


def test_chunked_prefill_in_the_gpu_loop(engine):
    """GPU chunked prefill, host side: a 50-token prompt is prefilled 5 tokens a step
    (budget 8 minus the decoding row's k + 1 = 3) beside a decoding request; the last
    chunk is a prefill from its start position; both outputs are the model's chain."""
    llm = engine(chunk=8)
    short, long_ = [5, 6, 7], list(range(10, 60))
    out = llm.generate([short, long_], SamplingParams(max_tokens=30, ignore_eos=True))
    assert out[0].outputs[0].token_ids == chain(short, 30) and out[1].outputs[0].token_ids == chain(long_, 30)
    log = [c for c in llm._chunk_log if c[0] == out[1].request_id]
    assert log[0][1] == 0 and log[-1][2] == 50 and all(e - s <= 8 for _, s, e, _ in log)
    assert sum(1 for c in log if c[3] == 1) >= 5                   # chunks beside the decoding row
    assert llm.runner.chunks == [(s, e) for _, s, e, _ in log[:-1]]
    assert llm.runner.starts_log[-1] == [log[-1][1]]


def test_allowed_token_ids_in_the_gpu_loop(engine):
    """allowed_token_ids on the GPU loop: the row's dense bias keeps only the allowed
    tokens, so every emitted token is one of them; a greedy row beside it keeps the chain."""
    llm = engine()
    only = SamplingParams(max_tokens=6, ignore_eos=True, allowed_token_ids=[77, 78])
    out = llm.generate([[5, 6, 7], [9, 10]], [SamplingParams(max_tokens=6, ignore_eos=True), only])
    assert out[0].outputs[0].token_ids == chain([5, 6, 7], 6)
    assert set(out[1].outputs[0].token_ids) <= {77, 78} and len(out[1].outputs[0].token_ids) == 6


def test_gate_audit_spec_mask_and_trace(engine, tmp_path, caplog):
    """GATE_AUDIT = 1 with a gate that never fires: every step with experts to promote runs
    one audit fire (promote + replay) logged with its argmax flips; GATE_SPEC_MASK scores only the emitted verify
    rows; GATE_TRACE logs each fire.  Output is still the model's chain."""
    import json
    import logging
    from vllm_moet_b200.residency import ConfidenceGate
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    from vllm_moet_b200.utils.observability import JsonlWriter
    llm = engine()
    L, E, H, I = 2, 8, 64, 64
    sb = delta_layout(H, I)[0]
    llm.delta = DeltaTier([torch.zeros(E, sb, dtype=torch.uint8) for _ in range(L)], H, I, 16, device="cpu",
                          policy="need")
    llm.gate = ConfidenceGate(tau=-1.0, fp_max=2)          # never fires on its own
    llm.delta_trace = None
    llm.gate_log = JsonlWriter(str(tmp_path / "gate.jsonl"))
    m = llm.ecfg.moet
    m.gate_fire_timing, m.gate_audit, m.gate_spec_mask, m.gate_trace = False, 1.0, True, True
    llm.runner.route_ids = lambda B, st=None: [torch.tensor([[int(t) % E, (int(t) + 1) % E] for t in
                                                             llm._states[B].tokens[:, 0].tolist()])] * L
    scored = []
    real_score = llm.gate.score
    llm.gate.score = lambda lg, tp_group=None: (scored.append(lg.shape[0]), real_score(lg, tp_group=tp_group))[1]
    try:
        with caplog.at_level(logging.INFO, logger="vllm_moet_b200"):
            out = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=10, ignore_eos=True))[0].outputs[0].token_ids
    finally:
        llm.delta.close()
        llm.gate_log.close()
    assert out == chain([5, 6, 7], 10)
    rows = [json.loads(x) for x in (tmp_path / "gate.jsonl").read_text().splitlines()]
    # every fire is an audit (one per step; none once the step's experts are all resident)
    fired = [r for r in rows if r["fired"]]
    assert fired and all(r["audit"] and r["fired"] == 1 and "flips" in r for r in fired)
    assert all(not r["audit"] for r in rows if not r["fired"])
    assert llm.delta.stats["gate_audits"] == len(fired)
    assert max(scored) <= llm.k + 1 and min(scored) >= 1            # emitted rows of one sequence
    assert any("gate audit" in r.getMessage() for r in caplog.records)


@pytest.mark.parametrize("mode", ["capture", "no_reforward"])
def test_gate_capture_and_no_reforward(engine, tmp_path, mode):
    """GATE_CAPTURE: an always-firing gate only logs (no promotion, no replay).
    GATE_REFORWARD=0: a fire promotes for later steps but the step is not replayed."""
    import json
    from vllm_moet_b200.residency import ConfidenceGate
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    from vllm_moet_b200.utils.observability import JsonlWriter
    llm = engine()
    L, E, H, I = 2, 8, 64, 64
    sb = delta_layout(H, I)[0]
    llm.delta = DeltaTier([torch.zeros(E, sb, dtype=torch.uint8) for _ in range(L)], H, I, 16, device="cpu",
                          policy="need")
    llm.gate = ConfidenceGate(tau=2.0, fp_max=2)
    llm.delta_trace = None
    llm.gate_log = JsonlWriter(str(tmp_path / "gate.jsonl"))
    m = llm.ecfg.moet
    m.gate_fire_timing = False
    m.gate_capture, m.gate_reforward = mode == "capture", mode != "no_reforward"
    llm.runner.route_ids = lambda B, st=None: [torch.tensor([[int(t) % E, (int(t) + 1) % E] for t in
                                                             llm._states[B].tokens[:, 0].tolist()])] * L
    try:
        out = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=8, ignore_eos=True))[0].outputs[0].token_ids
    finally:
        llm.delta.close()
        llm.gate_log.close()
    assert out == chain([5, 6, 7], 8)
    rows = [json.loads(x) for x in (tmp_path / "gate.jsonl").read_text().splitlines()]
    assert llm.delta.stats["gate_replays"] == 0                     # neither mode replays a step
    if mode == "capture":
        assert rows and all(r["capture"] and r["would_fire"] for r in rows)
        assert llm.delta.stats["fetched_rows"] == 0
    else:
        fired = [r for r in rows if r["fired"]]
        assert fired and all(r["iters"][0]["reforward"] is False for r in fired)
        assert llm.delta.stats["fetched_rows"] > 0 and llm.delta.stats["gate_promote_only"] == len(fired)


def test_capped_gate_fire_promotes_the_most_needed_first(engine):
    """With more routed experts than gate max_promote, a fire promotes the ones the delta
    tier ranks highest (its decayed need / frequency)."""
    from vllm_moet_b200.residency import ConfidenceGate
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    llm = engine()
    L, E, H, I = 2, 8, 64, 64
    sb = delta_layout(H, I)[0]
    llm.delta = DeltaTier([torch.zeros(E, sb, dtype=torch.uint8) for _ in range(L)], H, I, 16, device="cpu",
                          policy="need")
    llm.gate = ConfidenceGate(tau=2.0, fp_max=1, max_promote=1)
    llm.delta_trace, llm.gate_log = None, None
    llm.ecfg.moet.gate_fire_timing = False
    llm.runner.route_ids = lambda B, st=None: [torch.tensor([[int(t) % E, (int(t) + 1) % E] for t in
                                                             llm._states[B].tokens[:, 0].tolist()])] * L
    llm.delta.freq[1, :] = torch.arange(E, dtype=torch.float32) * 100.0    # layer 1, higher ids hotter
    calls = []
    real = llm.delta.promote
    llm.delta.promote = lambda pairs, **kw: (calls.append(list(pairs)), real(pairs, **kw))[1]
    try:
        llm.generate([[5, 6, 7]], SamplingParams(max_tokens=2, ignore_eos=True))
    finally:
        llm.delta.close()
    first = calls[0]
    assert len(first) == 1 and first[0][0] == 1            # a layer-1 expert, the hottest routed one


def test_gate_hidden_capture_shards(engine, tmp_path):
    """GATE_HCAP_DIR with the gate dump: the scored rows' hidden states of every fired step
    go to hcap-NNNNN.pt shards (flushed every GATE_HCAP_FLUSH records and at close), keyed
    by the dump's step numbers."""
    import json
    from vllm_moet_b200.residency import ConfidenceGate
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    from vllm_moet_b200.utils.observability import HiddenCapture, JsonlWriter
    llm = engine()
    L, E, H, I = 2, 8, 64, 64
    sb = delta_layout(H, I)[0]
    llm.delta = DeltaTier([torch.zeros(E, sb, dtype=torch.uint8) for _ in range(L)], H, I, 16, device="cpu",
                          policy="need")
    llm.gate = ConfidenceGate(tau=2.0, fp_max=1)
    llm.delta_trace = None
    llm.gate_log = JsonlWriter(str(tmp_path / "gate.jsonl"))
    llm.hcap = HiddenCapture(str(tmp_path / "hcap"), flush=2)
    llm.ecfg.moet.gate_fire_timing = False
    llm.runner.main_hidden = lambda B: torch.arange(B * (llm.k + 1) * 4, dtype=torch.float32).view(-1, 4)
    llm.runner.route_ids = lambda B, st=None: [torch.tensor([[int(t) % E, (int(t) + 1) % E] for t in
                                                             llm._states[B].tokens[:, 0].tolist()])] * L
    try:
        llm.generate([[5, 6, 7]], SamplingParams(max_tokens=8, ignore_eos=True))
    finally:
        llm.delta.close()
        llm.gate_log.close()
        llm.hcap.close()
    fired = [r["step"] for r in map(json.loads, (tmp_path / "gate.jsonl").read_text().splitlines()) if r["fired"]]
    shards = sorted((tmp_path / "hcap").glob("hcap-*.pt"))
    got = [torch.load(p) for p in shards]
    steps = sum((g["steps"].tolist() for g in got), [])
    assert fired and steps == fired and len(shards) == (len(fired) + 1) // 2
    assert all(h.shape[1] == 4 for g in got for h in g["h"])


def test_capped_gate_fire_step_w_ranks_by_routing_weight(engine):
    """DELTA_RANK=step_w: a capped fire promotes the expert with this step's largest routing
    weight first, whatever the decayed rank says."""
    from vllm_moet_b200.residency import ConfidenceGate
    from vllm_moet_b200.residency.delta import DeltaTier, delta_layout
    llm = engine()
    L, E, H, I = 2, 8, 64, 64
    sb = delta_layout(H, I)[0]
    llm.delta = DeltaTier([torch.zeros(E, sb, dtype=torch.uint8) for _ in range(L)], H, I, 16, device="cpu",
                          policy="need")
    llm.gate = ConfidenceGate(tau=2.0, fp_max=1, max_promote=1)
    llm.delta_trace, llm.gate_log = None, None
    llm.ecfg.moet.gate_fire_timing = False
    llm.ecfg.moet.delta_rank = "step_w"
    ids_of = lambda B: [torch.tensor([[int(t) % E, (int(t) + 1) % E] for t in    # noqa: E731
                                      llm._states[B].tokens[:, 0].tolist()])] * L
    llm.runner.route_ids = lambda B, st=None: ids_of(B)
    # layer 0's second routed expert carries the heaviest weight; layer 1 the hottest rank
    llm.runner.route_weights = lambda B: [torch.tensor([[0.1, 0.9]] * B), torch.tensor([[0.2, 0.3]] * B)]
    llm.delta.freq[1, :] = 1000.0
    calls = []
    real = llm.delta.promote
    llm.delta.promote = lambda pairs, **kw: (calls.append(list(pairs)), real(pairs, **kw))[1]
    try:
        llm.generate([[5, 6, 7]], SamplingParams(max_tokens=2, ignore_eos=True))
    finally:
        llm.delta.close()
    (li, _), = calls[0]
    assert li == 0                                          # the heaviest weight beats the hottest rank


def test_one_token_bad_words_in_the_gpu_loop(engine):
    """One-token bad words on the GPU loop: the row's dense bias bans them."""
    llm = engine()
    want = chain([5, 6, 7], 6)
    out = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=6, ignore_eos=True, bad_word_ids=[[want[2]]]))
    got = out[0].outputs[0].token_ids
    assert want[2] not in got and got[:2] == want[:2]
