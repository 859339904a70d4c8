"""GPU expert cache end to end: a decode served from a host store through a
small GPU cache (misses counted in-graph, fetched, replayed to a fixed point)
emits exactly the tokens of the fully resident engine."""
import pytest
import torch

from vllm_moet_b200 import SamplingParams
from vllm_moet_b200.config import ds4_flash_config
from vllm_moet_b200.engine.llm import LLM

pytestmark = pytest.mark.gpu


def _cfg():
    return ds4_flash_config(num_layers=3, hidden=1024, vocab=2048, num_experts=16, moe_intermediate=256,
                            dense_intermediate=512, num_heads=8, q_lora_rank=256, top_k=4)


def _prompts():
    g = torch.Generator().manual_seed(5)
    return [torch.randint(3, 2048, (n,), generator=g).tolist() for n in (29, 50)]


@pytest.fixture(scope="module")
def resident_tokens():
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2)
    out = [o.outputs[0].token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    del llm
    torch.cuda.empty_cache()
    return out


@pytest.mark.parametrize("kind", ["pinned", "tiered"])
def test_cached_experts_match_resident(resident_tokens, kind, tmp_path, monkeypatch):
    # 3 MoE layers (2 main + MTP) x 16 experts = 48; a 40-slot cache (below the conservative
    # working-set floor, hence FORCE_POOL) forces evictions and replays
    monkeypatch.setenv("VLLM_MOE_W2_FORCE_POOL", "1")
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              expert_cache_slots=40, expert_store=kind, expert_store_dir=str(tmp_path))
    out = [o.outputs[0].token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    assert out == resident_tokens
    st = llm.cache.stats
    assert st["fetched_rows"] > 0
    assert llm.replay.stats["steps"] > 0
    llm.shutdown()


def test_delta_tier_and_gate(resident_tokens):
    """Gate never firing: tokens equal the base engine.  Gate always firing with a pool
    that holds every expert: every decode step replays on FP4 experts, and the
    tokens track an oracle whose experts are the FP4 (MXFP4) weights."""
    from vllm_moet_b200.models import reference
    from vllm_moet_b200.residency.delta import dequant_delta_slot
    quiet = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
                delta_slots=48, gate=True)
    quiet.gate.tau = -1.0           # never fires
    out = [o.outputs[0].token_ids for o in quiet.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    assert out == resident_tokens
    del quiet
    torch.cuda.empty_cache()
    loud = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
               delta_slots=48, gate=True)
    loud.gate.tau = 2.0             # always fires (max-prob <= 1)
    p = _prompts()[0]
    toks = loud.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids
    assert loud.delta.stats["gate_replays"] > 0 and loud.delta.stats["fetched_rows"] > 0
    # oracle over FP4 experts for the decode part (the first token comes from prefill on the base)
    from vllm_moet_b200.residency import moe_layers
    lay = moe_layers(loud.mw)[0].experts.layout
    for li, lw in enumerate(moe_layers(loud.mw)):
        rows = loud.delta.store.layers[li]
        d = [dequant_delta_slot(rows[e].cpu(), lay.H, lay.I) for e in range(rows.shape[0])]
        lw.experts.dense_w13 = torch.stack([a for a, _ in d]).cuda()
        lw.experts.dense_w2 = torch.stack([b for _, b in d]).cuda()
    cs = reference.rope_cos_sin(loud.cfg, 256, "cuda")
    seq = list(p) + [toks[0]]
    for tok in toks[1:]:
        lg, _ = reference.forward(loud.mw, torch.tensor(seq, device="cuda"), torch.arange(len(seq), device="cuda"), cs)
        row = lg[-1]
        assert float(row[tok]) >= float(row.max()) - 0.5 * (float(row.std()) + 1e-6), (tok, int(row.argmax()))
        seq.append(tok)


def test_split_fp4_delta_and_gate(resident_tokens, monkeypatch):
    """Split FP4 delta slots (quintal refinement over the resident 2-bit base): with the
    gate quiet the tokens equal the base engine; with the gate always firing every decode
    step replays on FP4 experts rebuilt from base codes + refinement digits, and the tokens
    track an oracle whose experts are those exact MXFP4 values."""
    from vllm_moet_b200.formats import planes as pl
    from vllm_moet_b200.models import reference
    from vllm_moet_b200.residency import moe_layers
    from vllm_moet_b200.residency.delta import dequant_split_slot
    monkeypatch.setenv("VLLM_MOE_W2_DELTA_SPLIT", "1")
    quiet = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
                delta_slots=48, gate=True)
    assert quiet.delta.split
    quiet.gate.tau = -1.0
    out = [o.outputs[0].token_ids for o in quiet.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    assert out == resident_tokens
    quiet.shutdown()
    del quiet
    torch.cuda.empty_cache()
    loud = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
               delta_slots=48, gate=True)
    loud.gate.tau = 2.0
    p = _prompts()[0]
    toks = loud.generate([p], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids
    assert loud.delta.stats["gate_replays"] > 0 and loud.delta.stats["fetched_rows"] > 0
    loud.runner.check_status("split fp4")
    lay = moe_layers(loud.mw)[0].experts.layout
    H, I = lay.H, lay.I
    for li, lw in enumerate(moe_layers(loud.mw)):
        rows = loud.delta.store.layers[li]
        w13s, w2s = [], []
        for e in range(rows.shape[0]):
            c13, s13, c2, s2 = lay.split(lw.experts.pool[e].cpu())
            a, b = dequant_split_slot(rows[e].cpu(), pl.unpack_codes(c13, 2 * I, H), pl.unpack_scales(s13, 2 * I, H),
                                      pl.unpack_codes(c2, H, I), pl.unpack_scales(s2, H, I), H, I)
            w13s.append(a), w2s.append(b)
        lw.experts.dense_w13 = torch.stack(w13s).cuda()
        lw.experts.dense_w2 = torch.stack(w2s).cuda()
    cs = reference.rope_cos_sin(loud.cfg, 256, "cuda")
    seq = list(p) + [toks[0]]
    for tok in toks[1:]:
        lg, _ = reference.forward(loud.mw, torch.tensor(seq, device="cuda"), torch.arange(len(seq), device="cuda"), cs)
        row = lg[-1]
        assert float(row[tok]) >= float(row.max()) - 0.5 * (float(row.std()) + 1e-6), (tok, int(row.argmax()))
        seq.append(tok)
    loud.shutdown()


def test_traces_and_dumps(tmp_path, monkeypatch):
    """Prefill span timers, routing capture, the delta trace / precision-map dump and the
    gate JSONL with fire timing, all switched on by the reference's env names."""
    import json
    import numpy as np
    monkeypatch.setenv("VLLM_PREFILL_TIMERS_FLUSH", "4")
    monkeypatch.setenv("VLLM_MOE_W2_DELTA_TRACE", "2")
    monkeypatch.setenv("VLLM_MOE_W2_DELTA_DUMP", str(tmp_path / "prec.json"))
    monkeypatch.setenv("VLLM_MOE_W2_DELTA_CAPTURE", str(tmp_path / "routes.npy"))
    monkeypatch.setenv("VLLM_MOE_W2_GATE_FIRE_TIMING", "1")
    monkeypatch.setenv("VLLM_MOE_W2_GATE_DUMP", str(tmp_path / "gate.jsonl"))
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              delta_slots=48, gate=True)
    llm.gate.tau = 2.0
    llm.generate(_prompts(), SamplingParams(max_tokens=6, ignore_eos=True))
    summary = llm.timers.summary()
    assert {"prefill", "prefill.attention", "prefill.moe"} <= set(summary) and summary["prefill"]["total_ms"] > 0
    llm.shutdown()
    prec = json.loads((tmp_path / "prec.json").read_text())
    assert prec["delta"]["tier"] == "fp4-direct8" and len(prec["delta"]["resident"]) > 0
    assert 0 < prec["trace"]["coverage"] <= 1 and len(prec["trace"]["fp4_per_layer"]) == 3
    routes = np.load(tmp_path / "routes.npy")
    assert routes.ndim == 3 and routes.shape[1] == 3 and routes.shape[0] == llm._decode_steps
    rows = [json.loads(x) for x in (tmp_path / "gate.jsonl").read_text().splitlines()]
    assert len(rows) == llm._decode_steps and any(r["fired"] > 0 for r in rows)
    fired = [it for r in rows for it in r["iters"]]
    assert fired and all(it["promote_ms"] >= 0 and it["replay_ms"] > 0 for it in fired)


@pytest.mark.parametrize("pf4", ["1", "0"])
def test_prefill_fp4(pf4, monkeypatch):
    """Prefill-FP4 (VLLM_MOE_W2_PREFILL_FP4, default on): with every expert holding a direct-8
    delta slot, the prefill's last logits track the fp32 oracle over the FP4 (MXFP4) experts
    and not the one over the 2-bit base; with it off, the other way round."""
    from vllm_moet_b200.models import reference
    from vllm_moet_b200.residency import moe_layers
    from vllm_moet_b200.residency.delta import dequant_delta_slot
    monkeypatch.setenv("VLLM_MOE_W2_PREFILL_FP4", pf4)
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              delta_slots=48, gate=True)
    llm.gate.tau = -1.0
    layers = moe_layers(llm.mw)
    llm.delta.promote([(li, e) for li in range(len(layers)) for e in range(16)])
    p = _prompts()[1]
    llm.generate([p], SamplingParams(max_tokens=1, ignore_eos=True))
    lg = llm.runner.ws_prefill.bufs[("main.logits", torch.float32)][: llm.cfg.vocab].clone()
    cs = reference.rope_cos_sin(llm.cfg, 256, "cuda")
    t = torch.tensor(p, device="cuda")
    base = reference.forward(llm.mw, t, torch.arange(len(p), device="cuda"), cs)[0][-1]
    lay = layers[0].experts.layout
    for li, lw in enumerate(layers):
        rows = llm.delta.store.layers[li]
        d = [dequant_delta_slot(rows[e].cpu(), lay.H, lay.I) for e in range(rows.shape[0])]
        lw.experts.dense_w13 = torch.stack([a for a, _ in d]).cuda()
        lw.experts.dense_w2 = torch.stack([b for _, b in d]).cuda()
    fp4 = reference.forward(llm.mw, t, torch.arange(len(p), device="cuda"), cs)[0][-1]
    rel = lambda a, b: float((a - b).norm() / b.norm())     # noqa: E731
    e_fp4, e_base = rel(lg, fp4), rel(lg, base)
    if pf4 == "1":
        assert e_fp4 < e_base, (e_fp4, e_base)
    else:
        assert e_base < e_fp4, (e_fp4, e_base)
    llm.shutdown()


def test_router_lookahead_and_pilot_keep_tokens(resident_tokens, monkeypatch):
    """LOOKA + PILOT over a small expert cache: the in-graph predictions and the host
    prefetches never change the emitted tokens; the recall counters are rates, the
    lookahead predictor scores every main-stack layer after the first."""
    monkeypatch.setenv("VLLM_MOE_W2_FORCE_POOL", "1")
    monkeypatch.setenv("VLLM_MOE_W2_LOOKA", "1")
    monkeypatch.setenv("VLLM_MOE_W2_PILOT", "1")
    monkeypatch.setenv("VLLM_MOE_W2_PILOT_K", "8")
    llm = LLM(_cfg(), device="cuda", num_speculative_tokens=2, max_model_len=512, max_num_seqs=2,
              expert_cache_slots=40, expert_store="pinned")
    out = [o.outputs[0].token_ids for o in llm.generate(_prompts(), SamplingParams(max_tokens=12, ignore_eos=True))]
    assert out == resident_tokens
    r = llm.stats["looka_recall"]
    assert r["routed"] > 0 and 0 <= r["previous_step"] <= 1 and 0 < r["router_lookahead"] <= 1
    assert llm.stats["pilot"].get("requested", 0) + llm.stats["pilot"].get("warm_skips", 0) > 0
    llm.shutdown()
