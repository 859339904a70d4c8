"""CPU engine: BASELINE config 1 (tiny MoE) end to end, config validation."""
import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import EngineConfig, MoetConfig, ParallelConfig, tiny_config
from vllm_moet_b200.engine.llm import LLM
from vllm_moet_b200.models import reference


@pytest.fixture(scope="module")
def tiny_llm():
    return LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)


def test_tiny_mtp_engine_matches_full_recompute(tiny_llm):
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(3, 1024, (32,), generator=g).tolist() for _ in range(4)]
    outs = tiny_llm.generate(prompts, SamplingParams(max_tokens=16, ignore_eos=True))
    for p, o in zip(prompts, outs):
        assert o.outputs[0].token_ids == reference.greedy_generate(tiny_llm.mw, p, 16)


def test_tiny_engine_without_mtp():
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=128)
    p = [5, 6, 7, 8]
    o = llm.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))
    assert o[0].outputs[0].token_ids == reference.greedy_generate(llm.mw, p, 6)


def test_string_prompt_and_stop_token(tiny_llm):
    o = tiny_llm.generate("hello", SamplingParams(max_tokens=5))
    assert 1 <= len(o[0].outputs[0].token_ids) <= 5
    first = o[0].outputs[0].token_ids[0]
    o2 = tiny_llm.generate("hello", SamplingParams(max_tokens=5, stop_token_ids=[first]))
    assert o2[0].outputs[0].token_ids == [first] and o2[0].outputs[0].finish_reason == "stop"


def test_config_validation():
    with pytest.raises(ValueError, match="ZERO_MODE"):
        MoetConfig(zero_mode="typo")
    with pytest.raises(ValueError, match="gate"):
        MoetConfig(gate=True)
    with pytest.raises(ValueError):
        ParallelConfig(tp=3)
    with pytest.raises(ValueError, match="nvfp4"):
        EngineConfig(model=tiny_config(), kv_cache_dtype="nvfp4")
    with pytest.raises(ValueError):
        SamplingParams(max_tokens=0)


def test_env_aliases(monkeypatch):
    monkeypatch.setenv("VLLM_MOE_W2_PREFILL_T", "128")
    monkeypatch.setenv("VLLM_MOE_W2_DELTA", "1")
    monkeypatch.setenv("VLLM_MOE_W2_GATE_TAU", "0.7")
    c = MoetConfig.from_env()
    assert c.prefill_t == 128 and c.delta is True and c.gate_tau == 0.7


def test_trace_env_aliases(monkeypatch):
    from vllm_moet_b200.config import MoetConfig
    monkeypatch.setenv("VLLM_PREFILL_TIMERS_FLUSH", "16")
    monkeypatch.setenv("VLLM_MOE_W2_DELTA_TRACE", "2")
    monkeypatch.setenv("VLLM_MOE_W2_GATE_FIRE_TIMING", "1")
    monkeypatch.setenv("VLLM_MOE_W2_GATE_DUMP", "/tmp/g.jsonl")
    m = MoetConfig.from_env()
    assert (m.prefill_timers_flush, m.delta_trace, m.gate_fire_timing, m.gate_dump) == (16, 2, True, "/tmp/g.jsonl")


def test_delta_trace_counts():
    import torch
    from vllm_moet_b200.utils.observability import DeltaTrace

    class FakeDelta:
        L, E = 2, 4
        mirror = torch.tensor([[0, -1, -1, -1], [-1, 1, -1, -1]])
        stats = {"fetched_rows": 2, "evictions": 0}

        def resident(self, li, e):
            return int(self.mirror[li, e]) >= 0
    lines = []
    t = DeltaTrace(level=2, every=2, sink=lines.append)
    d = FakeDelta()
    t.step(d, {(0, 0): 3, (0, 1): 1})
    t.step(d, {(1, 1): 2, (1, 2): 2})
    snap = t.snapshot(d)
    assert snap["hit_rate_distinct"] == 0.5 and snap["hit_rate_tokens"] == 5 / 8
    assert snap["coverage"] == 2 / 8 and snap["fp4_per_layer"] == [1, 1] and len(lines) == 1


def _stop_prompt():
    g = torch.Generator().manual_seed(5)
    return torch.randint(3, 259, (12,), generator=g).tolist()


def test_stop_strings_min_tokens_and_stop_ids():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    p = _stop_prompt()
    full = llm.generate([p], SamplingParams(max_tokens=16, ignore_eos=True))[0].outputs[0]
    stop = full.text[-2:]
    i = full.text.find(stop)
    cut = llm.generate([p], SamplingParams(max_tokens=16, ignore_eos=True, stop=[stop]))[0].outputs[0]
    assert cut.finish_reason == "stop" and cut.stop_reason == stop and cut.text == full.text[:i]
    assert cut.token_ids == full.token_ids[:len(cut.token_ids)] and len(cut.token_ids) <= len(full.token_ids)
    inc = llm.generate([p], SamplingParams(max_tokens=16, ignore_eos=True, stop=stop,
                                           include_stop_str_in_output=True))[0].outputs[0]
    assert inc.text == full.text[:i + len(stop)]
    # stop token ids apply even with ignore_eos (only EOS is ignored)
    sid = full.token_ids[2]
    k = full.token_ids.index(sid)
    o = llm.generate([p], SamplingParams(max_tokens=16, ignore_eos=True, stop_token_ids=[sid]))[0].outputs[0]
    assert o.finish_reason == "stop" and o.stop_reason == sid and o.token_ids == full.token_ids[:k + 1]
    # min_tokens: no stop condition before it
    first = full.token_ids[0]
    o = llm.generate([p], SamplingParams(max_tokens=16, ignore_eos=True, stop_token_ids=[first],
                                         min_tokens=4))[0].outputs[0]
    assert len(o.token_ids) >= 4 and o.token_ids == full.token_ids[:len(o.token_ids)]
    with pytest.raises(ValueError):
        SamplingParams(max_tokens=2, min_tokens=3)


def test_stop_stream_holds_back_partial_stops():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.tokenizer import ByteTokenizer
    from vllm_moet_b200.entrypoints.openai_server import _StopStream
    tok = ByteTokenizer(1024)
    ids = [ord(c) + 3 for c in "hello wor" "ld<END>tail"]
    ss = _StopStream(tok, SamplingParams(max_tokens=64, stop=["<END>"]))
    out = "".join(ss.push([t], False) for t in ids)
    assert out == "hello world" and ss.done
    ss = _StopStream(tok, SamplingParams(max_tokens=64, stop=["<END>"]))
    out = "".join(ss.push([t], i == 6) for i, t in enumerate(ids[:7]))
    assert out == "hello w"                    # finished without a stop: everything held back is flushed


def test_logprobs_match_reference():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    p = [5, 6, 7, 8, 9, 10]
    o = llm.generate([p], SamplingParams(max_tokens=7, ignore_eos=True, logprobs=3))[0].outputs[0]
    assert len(o.logprobs) == len(o.token_ids) == 7
    cs = reference.rope_cos_sin(llm.cfg, 64)
    toks = list(p)
    total = 0.0
    for t, d in zip(o.token_ids, o.logprobs):
        lg, _ = reference.forward(llm.mw, torch.tensor(toks), torch.arange(len(toks)), cs)
        lp = torch.log_softmax(lg[-1], -1)
        assert abs(d[t] - float(lp[t])) < 1e-4
        top = torch.topk(lp, 3).indices.tolist()
        assert set(top) <= set(d) and len(d) <= 4
        total += d[t]
        toks.append(t)
    assert abs(o.cumulative_logprob - total) < 1e-6
    got = []
    llm.generate([p], SamplingParams(max_tokens=3, ignore_eos=True, logprobs=0),
                 callbacks=[lambda ids, fin, lp=None: got.extend(lp or [])])
    assert len(got) == 3 and all(len(d) == 1 for d in got)
    assert llm.generate([p], SamplingParams(max_tokens=2))[0].outputs[0].logprobs is None


def test_requests_join_and_abort_between_steps():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, max_num_seqs=4)
    sp = SamplingParams(max_tokens=12, ignore_eos=True)
    solo = {n: llm.generate([p], s)[0].outputs[0].token_ids for n, p, s in
            (("b", [8, 9], sp), ("j", [9, 10, 11], SamplingParams(max_tokens=5, ignore_eos=True)))}
    ev = {}

    def cb(name):
        return lambda ids, fin, lp=None: ev.setdefault(name, []).append((list(ids), fin))
    step = [0]

    def between(n_free):
        step[0] += 1
        new = [("j", [9, 10, 11], SamplingParams(max_tokens=5, ignore_eos=True), cb("j"))] if step[0] == 3 else []
        return new, ({"a"} if step[0] == 2 else set())
    out = llm.generate([[5, 6, 7], [8, 9]], sp, callbacks=[cb("a"), cb("b")], request_ids=["a", "b"],
                       between_steps=between)
    a, b = (o.outputs[0] for o in out)
    assert a.finish_reason == "abort" and len(a.token_ids) < 12 and ev["a"][-1][1] == "abort"
    assert b.finish_reason == "length" and b.token_ids == solo["b"]
    joined = sum((ids for ids, _ in ev["j"]), [])
    assert joined == solo["j"] and ev["j"][-1][1] == "length"


def test_n_completions_and_chat():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    out = llm.generate([[5, 6, 7], [9, 10]], SamplingParams(max_tokens=5, ignore_eos=True, temperature=1.2, seed=4,
                                                             n=3))
    assert len(out) == 2 and all(len(o.outputs) == 3 for o in out)
    assert [c.index for c in out[0].outputs] == [0, 1, 2]
    seqs = [c.token_ids for c in out[0].outputs]
    assert len({tuple(x) for x in seqs}) > 1                      # different seeds, different samples
    again = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=5, ignore_eos=True, temperature=1.2, seed=4, n=3))
    assert [c.token_ids for c in again[0].outputs] == seqs         # seed + i per copy: reproducible
    greedy = llm.generate([[5, 6, 7]], SamplingParams(max_tokens=4, ignore_eos=True, n=2))[0].outputs
    assert greedy[0].token_ids == greedy[1].token_ids
    c = llm.chat([{"role": "user", "content": "hi"}], SamplingParams(max_tokens=3, ignore_eos=True))
    assert len(c) == 1 and len(c[0].outputs[0].token_ids) == 3
    assert c[0].prompt_token_ids[0] == llm.tokenizer.bos_token_id


def test_grow_state_moves_rows_to_a_larger_bucket():
    import types
    from vllm_moet_b200.engine.gpu_runner import DecodeState
    from vllm_moet_b200.engine.llm import LLM
    fake = types.SimpleNamespace(_states={}, _DecodeState=DecodeState, k=2, max_blocks=8, device="cpu")
    fake._state = types.MethodType(LLM._state, fake)
    st = fake._state(2)
    st.tokens.copy_(torch.arange(6, dtype=torch.int32).view(2, 3))
    st.seq_pos.copy_(torch.tensor([17, 40], dtype=torch.int32))
    st.block_table[1, :3] = torch.tensor([5, 6, 7], dtype=torch.int32)
    big = fake._state(4)
    big.tokens.fill_(99)                          # stale rows of an earlier use of the bucket
    st2 = LLM._grow_state(fake, st, 4)
    assert st2 is big and st2.B == 4
    assert torch.equal(st2.tokens[:2], st.tokens) and (st2.tokens[2:] == 0).all()
    assert st2.seq_pos.tolist() == [17, 40, 0, 0] and st2.block_table[1, :3].tolist() == [5, 6, 7]
    assert [LLM._bucket(n) for n in (1, 2, 3, 5, 32)] == [1, 2, 4, 8, 32]


def test_prompt_logprobs_match_reference():
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    p = [5, 6, 7, 8, 9, 10]
    o = llm.generate([p], SamplingParams(max_tokens=2, ignore_eos=True, prompt_logprobs=2))[0]
    assert o.prompt_logprobs[0] is None and len(o.prompt_logprobs) == len(p)
    lg, _ = reference.forward(llm.mw, torch.tensor(p), torch.arange(len(p)), reference.rope_cos_sin(llm.cfg, 64))
    lp = torch.log_softmax(lg, -1)
    for i in range(1, len(p)):
        d = o.prompt_logprobs[i]
        assert abs(d[p[i]] - float(lp[i - 1, p[i]])) < 1e-4 and len(d) <= 3
    assert llm.generate([p], SamplingParams(max_tokens=2))[0].prompt_logprobs is None


def test_prefix_caching_reuses_the_shared_prefix():
    """Automatic prefix caching: requests that share a block-aligned prompt prefix run the
    main model on the suffix only (and the MTP prefill from the prefix's last position),
    and give the same tokens, prompt logprobs and drafts-driven acceptance as a cold run."""
    from vllm_moet_b200 import SamplingParams
    sys_prompt = list(range(3, 3 + 40))
    prompts = [sys_prompt + [50, 51, 52], sys_prompt + [60, 61], sys_prompt + [50, 51, 52, 53, 54, 55]]
    sp = SamplingParams(max_tokens=10, ignore_eos=True, prompt_logprobs=1)
    cold = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    warm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256,
               enable_prefix_caching=True, prefix_block_size=16)
    want = [cold.generate([p], sp)[0] for p in prompts]
    got = [warm.generate([p], sp)[0] for p in prompts]
    for w, g in zip(want, got):
        assert g.outputs[0].token_ids == w.outputs[0].token_ids
        for a, b in zip(w.prompt_logprobs[1:], g.prompt_logprobs[1:]):
            assert a.keys() == b.keys() and all(abs(a[t] - b[t]) < 1e-3 for t in a)
    st = warm.runner.prefix_stats
    assert st["hits"] == 2 and st["hit_tokens"] == 32 + 32      # block 16: 32 of the 40 shared tokens
    assert cold.runner.prefix_stats["hits"] == 0


def test_hyper_connections_engine_matches_oracle():
    """mHC model (4 residual streams, Sinkhorn-mixed around every block): the CPU engine's
    MTP-speculative decode, with and without prefix caching, gives the full-recompute
    greedy chain; the streams really mix (the model differs from the hc_mult 1 model)."""
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.models import reference as ref
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, hc_mult=4,
              enable_prefix_caching=True, prefix_block_size=4)
    plain = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    prompts = [[5, 6, 7, 8, 9, 10], [5, 6, 7, 8, 20]]
    sp = SamplingParams(max_tokens=12, ignore_eos=True)
    outs = [llm.generate([p], sp)[0].outputs[0].token_ids for p in prompts]
    for p, o in zip(prompts, outs):
        assert o == ref.greedy_generate(llm.mw, p, 12)
    assert llm.runner.prefix_stats["hits"] == 1
    assert outs[0] != plain.generate([prompts[0]], sp)[0].outputs[0].token_ids
    with pytest.raises(NotImplementedError):
        LLM("tiny-moe", device="cpu", hc_mult=4, speculative_method="dspark", dspark={"model": "simple"})


def test_chunked_prefill_interleaves_with_decode():
    """Chunked prefill: a long prompt is prefilled a token budget at a time while a short
    request keeps decoding (its decode rows take (k + 1) tokens of each step's budget);
    tokens and prompt logprobs equal the unchunked engine's, with and without prefix caching."""
    from vllm_moet_b200 import SamplingParams
    short, long_ = [5, 6, 7, 8], list(range(3, 63))
    sp = SamplingParams(max_tokens=10, ignore_eos=True, prompt_logprobs=0)
    plain = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    want = plain.generate([short, long_], sp)
    for prefix in (False, True):
        llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256,
                  enable_chunked_prefill=True, max_num_batched_tokens=8, enable_prefix_caching=prefix,
                  prefix_block_size=16)
        got = llm.generate([short, long_], sp)
        for w, g in zip(want, got):
            assert g.outputs[0].token_ids == w.outputs[0].token_ids
            for a, b in zip(w.prompt_logprobs[1:], g.prompt_logprobs[1:]):
                assert a.keys() == b.keys() and all(abs(a[t] - b[t]) < 1e-3 for t in a)
        log = [c for c in llm._chunk_log if c[0] == got[1].request_id]
        assert len(log) >= 10 and log[-1][2] == len(long_)
        assert all(d - b <= 8 for _, b, d, _ in log)
        assert sum(1 for c in log if c[3] == 1) >= 5             # chunks that ran beside a decoding row
        assert llm.stats["prefill_chunks"] == len(llm._chunk_log)


def test_reference_dsa_selection():
    """The oracle's DSA indexer: no selection while the context fits in index_topk (the
    forward equals the dense one); with a small top-k every query keeps exactly top-k keys
    at or before its position (fewer when fewer exist), and the logits change."""
    import torch
    from vllm_moet_b200.config import glm52_config
    from vllm_moet_b200.models import reference
    from vllm_moet_b200.models.weights import random_weights
    cfg = glm52_config(num_layers=2, hidden=256, vocab=512, num_experts=8, moe_intermediate=64,
                       dense_intermediate=128, num_dense_layers=1, num_heads=4, q_lora_rank=64, top_k=2,
                       index_heads=4, index_head_dim=32, index_topk=4096)
    mw = random_weights(cfg, "cpu", seed=3, with_mtp=False)
    T = 40
    toks = torch.randint(3, 512, (T,), generator=torch.Generator().manual_seed(1))
    cs = reference.rope_cos_sin(cfg, 128)
    dense, _ = reference.forward(mw, toks, torch.arange(T), cs)
    lw = mw.layers[0]
    x = torch.randn(T, cfg.hidden)
    qa = torch.randn(T, cfg.q_lora_rank)
    assert reference.dsa_select(cfg, lw, x, qa, torch.arange(T)) is None
    small = cfg.replace(index_topk=8)
    keep = reference.dsa_select(small, lw, x, qa, torch.arange(T))
    assert keep.shape == (T, T)
    # causal keys kept per query: all of them up to 8, then exactly 8 (the attention masks the rest)
    assert all(int(keep[t, :t + 1].sum()) == min(t + 1, 8) for t in range(T))
    mw.cfg = small
    sparse, _ = reference.forward(mw, toks, torch.arange(T), cs)
    assert not torch.allclose(sparse, dense)


def test_allowed_token_ids_match_masked_greedy(tiny_llm):
    """allowed_token_ids (vLLM's field): greedy decoding over the allowed tokens only, the
    first token included, equal to a greedy loop over the oracle's masked logits."""
    allowed = [11, 200, 345, 678, 901]
    p = [5, 9, 17, 33]
    got = tiny_llm.generate([p], SamplingParams(max_tokens=5, ignore_eos=True, allowed_token_ids=allowed))
    got = got[0].outputs[0].token_ids
    cs = reference.rope_cos_sin(tiny_llm.mw.cfg, 64)
    seq, want = list(p), []
    for _ in range(5):
        lg, _ = reference.forward(tiny_llm.mw, torch.tensor(seq), torch.arange(len(seq)), cs)
        m = torch.full_like(lg[-1], float("-inf"))
        m[allowed] = 0
        t = int(torch.argmax(lg[-1] + m))
        want.append(t)
        seq.append(t)
    assert got == want and set(got) <= set(allowed)
    with pytest.raises(ValueError):
        SamplingParams(allowed_token_ids=[])


def test_get_tokenizer(tiny_llm):
    tok = tiny_llm.get_tokenizer()
    assert tok is tiny_llm.tokenizer and tok.decode(tok.encode("ab")) == "ab"


def test_request_acceptance_metrics(tiny_llm):
    """Per-request acceptance length: tokens emitted per decode step after the first token."""
    o = tiny_llm.generate([[5, 9, 17, 33]], SamplingParams(max_tokens=10, ignore_eos=True))[0]
    m = o.metrics
    assert m["decode_steps"] >= 1 and 1.0 <= m["tokens_per_step"] <= tiny_llm.k + 1
    assert abs(m["tokens_per_step"] * m["decode_steps"] - (len(o.outputs[0].token_ids) - 1)) < 1e-9


def test_bad_words(tiny_llm):
    """bad_words / bad_word_ids (vLLM's fields): a one-token word never appears; a
    two-token word's second token is banned only right after its first."""
    p = [5, 9, 17, 33]
    sp = SamplingParams(max_tokens=6, ignore_eos=True)
    g = tiny_llm.generate([p], sp)[0].outputs[0].token_ids
    one = tiny_llm.generate([p], SamplingParams(max_tokens=6, ignore_eos=True, bad_word_ids=[[g[1]]]))
    one = one[0].outputs[0].token_ids
    assert g[1] not in one and one[0] == g[0]
    two = tiny_llm.generate([p], SamplingParams(max_tokens=6, ignore_eos=True, bad_word_ids=[[g[0], g[1]]]))
    two = two[0].outputs[0].token_ids
    assert two[0] == g[0] and two[1] != g[1]
    assert all(not (a == g[0] and b == g[1]) for a, b in zip(two, two[1:]))
    # words are tokenized by the engine (the word and its leading-space form)
    sw = SamplingParams(max_tokens=2, ignore_eos=True, bad_words=["ab"])
    tiny_llm.generate([p], sw)
    assert sw.bad_word_ids and all(isinstance(t, int) for w in sw.bad_word_ids for t in w)
