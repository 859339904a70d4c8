"""Trellis (EXL3-style) base tier on the CPU: format, Viterbi encoder, the decode kernel's
bit arithmetic restated in Python, decode groups, the tier and the engine hook.

The reference tests its EXL3 tier for parity against pack reconstruction
(tools/test_moe_w2_exl3.py, patch/vllm-moet-v0.24.0.patch:1736-1933) and checks the M8
group builder's invariants against its host builder (P:10456-10510); these are the same
checks for our format."""
import itertools
import math
import struct

import pytest
import torch

from vllm_moet_b200.formats import trellis as tf
from vllm_moet_b200.residency import trellis_tier as tt


def _f16(bits: int) -> float:
    return struct.unpack("<e", struct.pack("<H", bits & 0xFFFF))[0]


def test_codebooks_match_scalar_definitions():
    states = list(range(0, 1 << 16, 997)) + [0, 1, 65535]
    got3 = tf.codebook_raw(torch.tensor(states), "3inst")
    got1 = tf.codebook_raw(torch.tensor(states), "1mad")
    for i, s in enumerate(states):
        x = (s * 89226354 + 64248484) & 0xFFFFFFFF
        m = (x & 0x8FFF8FFF) ^ 0x3B603B60
        assert float(got3[i]) == pytest.approx(_f16(m) + _f16(m >> 16), abs=0)
        x = (s * 34038481 + 76625530) & 0xFFFFFFFF
        tot = sum((x >> (8 * b)) & 0xFF for b in range(4))
        assert float(got1[i]) == pytest.approx((tot - 510) / 147.8, rel=1e-6)
    for cb in tf.CODEBOOKS:     # unit RMS after normalisation, near-zero mean
        v = tf.codebook_table(16, cb).double()
        assert float(v.pow(2).mean().sqrt()) == pytest.approx(1.0, rel=1e-5)
        assert abs(float(v.mean())) < 0.01


def test_fwht_is_block_sylvester_hadamard():
    from scipy.linalg import hadamard
    for n in (16, 96, 256, 384):
        b = tf.hadamard_block(n)
        assert b == min(128, n & -n)
        H = torch.block_diag(*[torch.tensor(hadamard(b), dtype=torch.float64)] * (n // b)) / math.sqrt(b)
        x = torch.randn(5, n, dtype=torch.float64)
        assert torch.allclose(tf.fwht(x), x @ H, atol=1e-12)
        assert torch.allclose(tf.fwht(tf.fwht(x)), x, atol=1e-12)


def test_viterbi_is_optimal_on_short_walks():
    torch.manual_seed(0)
    K, L, n = 1, 3, 6
    cbv = tf.codebook_table(L)
    target = torch.randn(4, n)
    _, cost = tf._viterbi(target, cbv, K, L, None)
    for b in range(4):
        best = float("inf")
        for s0 in range(1 << L):
            for codes in itertools.product(range(1 << K), repeat=n - 1):
                s, c = s0, float((target[b, 0] - cbv[s0]) ** 2)
                for i, code in enumerate(codes, 1):
                    s = ((s << K) | code) & ((1 << L) - 1)
                    c += float((target[b, i] - cbv[s]) ** 2)
                best = min(best, c)
        assert float(cost[b]) == pytest.approx(best, rel=1e-5)


@pytest.mark.parametrize("K,L", [(1, 6), (2, 8), (2, 12), (3, 10), (4, 9)])
def test_encoded_stream_is_the_tail_biting_walk(K, L):
    torch.manual_seed(K * 100 + L)
    v = torch.randn(8, 256)
    words = tf.encode_tiles(v, K, L)
    assert words.shape == (8, 16 * K) and words.dtype == torch.int16
    st = tf.tile_states(words, K, L)
    # consecutive states overlap in L-K bits, cyclically (the stream is one closed walk)
    mask = (1 << (L - K)) - 1
    assert torch.equal(st >> K, torch.roll(st, 1, dims=1) & mask)
    dec = tf.decode_tiles(words, K, L)
    # the decoded values are the tail-biting Viterbi optimum of the second pass
    cbv = tf.codebook_table(L)
    st2, cost = tf._viterbi(v, cbv, K, L, tf._viterbi(v, cbv, K, L, None)[0][:, -1] & mask)
    assert torch.equal(st2, st)
    assert torch.allclose(((dec - v) ** 2).sum(1), cost, rtol=1e-4)
    mse = float(((dec - v) ** 2).mean())
    assert mse < {1: 0.4, 2: 0.11, 3: 0.035, 4: 0.012}[K]


def _kernel_states(words: torch.Tensor, K: int, L: int) -> torch.Tensor:
    """The trellis_gemv kernel's window extraction, restated: lane (kk, nn0) holds words
    w0..w0+3 of the tile (cyclic), shifts out 8 windows."""
    NW, NB = 16 * K, 256 * K
    out = torch.empty(words.shape[0], 256, dtype=torch.int64)
    w = words.to(torch.int64) & 0xFFFF
    for lane in range(32):
        kk, nn0 = lane >> 1, (lane & 1) * 8
        i0 = kk * 16 + nn0
        start = (i0 + 1) * K - L
        if start < 0:
            start += NB
        w0, sh = start >> 4, start & 15
        u = torch.zeros(words.shape[0], dtype=torch.int64)
        parts = [w[:, (w0 + q) % NW] for q in range(4)]
        for j in range(8):
            shift = 64 - sh - j * K - L
            assert 0 <= shift <= 64 - L
            # (u >> shift) & mask without 64-bit unsigned arithmetic: bits [64-shift-L, 64-shift)
            lo = 64 - shift - L
            val = torch.zeros_like(u)
            for b in range(L):
                pos = lo + b                   # bit position from the MSB of u
                wq, bit = pos // 16, 15 - pos % 16
                val = (val << 1) | ((parts[wq] >> bit) & 1)
            out[:, i0 + j] = val
    return out


@pytest.mark.parametrize("K,L", [(1, 2), (1, 16), (2, 8), (2, 16), (3, 12), (3, 16), (4, 5), (4, 16)])
def test_kernel_window_extraction_matches_format(K, L):
    g = torch.Generator().manual_seed(K * 31 + L)
    words = torch.randint(-32768, 32768, (3, 16 * K), generator=g, dtype=torch.int64).to(torch.int16)
    assert torch.equal(_kernel_states(words, K, L), tf.tile_states(words, K, L))


def test_quantize_linear_round_trip():
    torch.manual_seed(1)
    w = torch.randn(64, 128) * 0.02
    w[3] *= 8                                   # an outlier row
    x = torch.randn(5, 128)
    prev = None
    for K in (2, 3, 4):
        t = tf.quantize_linear(w, K, L=10, seed=3)
        assert t["trellis"].shape == (8, 4, 16 * K)
        assert t["suh"].dtype == torch.float16 and t["svh"].shape == (64,)
        wd = tf.dequant_linear(t, K, 10)
        rel = float((wd - w).norm() / w.norm())
        assert rel < {2: 0.33, 3: 0.18, 4: 0.1}[K]
        assert prev is None or rel < prev
        prev = rel
        # the transform route (what the kernels compute) equals the dense reconstruction
        assert torch.allclose(tf.apply_linear(x, t, K, 10), x @ wd.t(), rtol=1e-4, atol=1e-5)
        assert tf.linear_bytes(64, 128, K) == t["trellis"].numel() * 2 + 2 * (64 + 128)


def _groups_brute(ids, rows=8):
    T, k = ids.shape
    per = {}
    for p, e in enumerate(ids.reshape(-1).tolist()):
        per.setdefault(e, []).append(p)
    groups = []
    for e in sorted(per):
        ps = per[e]
        for g0 in range(0, len(ps), rows):
            groups.append((e, ps[g0:g0 + rows] + [-1] * (rows - len(ps[g0:g0 + rows]))))
    return groups


@pytest.mark.parametrize("T,k,E", [(1, 8, 256), (3, 8, 16), (9, 2, 4), (20, 4, 6), (17, 1, 1)])
def test_group_pairs_matches_brute_force(T, k, E):
    g = torch.Generator().manual_seed(T * 7 + k)
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]) if k <= E else None
    experts, row_map = tt.group_pairs(ids)
    want = _groups_brute(ids)
    P = T * k
    assert experts.shape == (P,) and row_map.shape == (P, 8)
    for gi, (e, rows) in enumerate(want):
        assert int(experts[gi]) == e and row_map[gi].tolist() == rows
    assert (row_map[len(want):] == -1).all() and (experts[len(want):] == 0).all()
    # every pair exactly once, never more than min(T, 8) rows per group
    got = sorted(x for x in row_map.reshape(-1).tolist() if x >= 0)
    assert got == list(range(P))
    assert int((row_map >= 0).sum(1).max()) <= min(T, 8)


@pytest.fixture(scope="module")
def tiny_tier(tmp_path_factory):
    from vllm_moet_b200.engine.llm import LLM
    d = str(tmp_path_factory.mktemp("trellis"))
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=128)
    layers = tt.write_model_packs(llm.mw, d, w13_k=3, w2_k=3, L=8)
    return llm, d, layers


def test_tier_forward_matches_pack_reconstruction(tiny_tier):
    llm, d, layers = tiny_tier
    cfg = llm.mw.cfg
    tier = tt.TrellisBaseTier(d, layers, w13_k=3, w2_k=3, act_limit=cfg.swiglu_limit)
    assert tier.L == 8 and tier.E == cfg.num_experts
    torch.manual_seed(0)
    li = layers[0]
    x = torch.randn(6, cfg.hidden)
    ids = torch.stack([torch.randperm(cfg.num_experts)[:cfg.top_k] for _ in range(6)])
    w = torch.rand(6, cfg.top_k)
    y = tier.forward_topk(li, x, ids, w)
    want = torch.zeros(6, cfg.hidden)
    from vllm_moet_b200.models.reference import swiglu
    for t in range(6):
        for j in range(cfg.top_k):
            w13, w2 = tier.dequant_expert(li, int(ids[t, j]))
            want[t] += w[t, j] * (swiglu(x[t:t + 1] @ w13.t(), cfg.swiglu_limit) @ w2.t())[0]
    assert torch.allclose(y, want, rtol=1e-4, atol=1e-5)
    # the served weights are close to the model's own experts
    w13, w2 = tier.dequant_expert(li, 0)
    o13, o2 = llm.mw.layers[li].experts.dequant_expert(0)
    assert float((w13 - o13).norm() / o13.norm()) < 0.2 and float((w2 - o2).norm() / o2.norm()) < 0.2
    # fp4_mask: the masked pairs are left out, and adding them back gives the full block
    mask = torch.zeros(6, cfg.top_k, dtype=torch.bool)
    mask[::2, 0] = True
    ym = tier.forward_topk(li, x, ids, w, fp4_mask=mask)
    add = torch.zeros_like(ym)
    for t, j in mask.nonzero().tolist():
        w13, w2 = tier.dequant_expert(li, int(ids[t, j]))
        add[t] += w[t, j] * (swiglu(x[t:t + 1] @ w13.t(), cfg.swiglu_limit) @ w2.t())[0]
    assert torch.allclose(ym + add, y, rtol=1e-4, atol=1e-5)
    assert tier.total_bytes() == sum(
        tf.linear_bytes(n, k_, 3) for n, k_ in ((cfg.moe_intermediate, cfg.hidden),) * 2
        + ((cfg.hidden, cfg.moe_intermediate),)) * cfg.num_experts * len(layers)


def test_engine_serves_from_trellis_tier(tiny_tier):
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference as ref
    _, d, layers = tiny_tier
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=128, trellis_pack=d)
    assert llm.trellis is not None and sorted(llm.trellis.layers) == layers
    assert (llm.trellis.w13_k, llm.trellis.w2_k) == (3, 3)      # from the pack's metadata
    g = torch.Generator().manual_seed(5)
    p = torch.randint(3, 1024, (24,), generator=g).tolist()
    out = llm.generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0].outputs[0].token_ids
    with ref.moe_context(llm.trellis.moe_fn(llm.mw)):
        want = ref.greedy_generate(llm.mw, p, 8)
    assert out == want
    plain = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=128)
    assert plain.generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0].outputs[0].token_ids \
        == ref.greedy_generate(plain.mw, p, 8)


def test_tier_rejects_foreign_packs(tmp_path):
    from safetensors.torch import save_file
    save_file({"e0.w1.k2.trellis": torch.zeros(1, dtype=torch.int16)}, str(tmp_path / "exl3-l00.safetensors"))
    with pytest.raises(ValueError, match="moet-trellis-v1"):
        tt.TrellisBaseTier(str(tmp_path), [0])


def test_pack_builder_cli(tmp_path, capsys):
    import json
    from vllm_moet_b200.tools.build_trellis_pack import main
    assert main([str(tmp_path), "--model", "tiny-moe", "--layers", "1", "--L", "6", "--w13-k", "2",
                 "--w2-k", "3", "--codebook", "1mad"]) == 0
    rec = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert rec["layer"] == 1 and rec["bits"] == [2, 3] and rec["format"] == tf.FORMAT
    assert 0 < rec["rel_err_w13_e0"] < 0.5 and 0 < rec["rel_err_w2_e0"] < 0.4
    tier = tt.TrellisBaseTier(str(tmp_path), [1])
    assert (tier.w13_k, tier.w2_k, tier.L, tier.codebook) == (2, 3, 6, "1mad")


def test_delta_pool_serves_base_plus_residual(tiny_tier):
    from vllm_moet_b200.models.reference import swiglu
    llm, d, layers = tiny_tier
    cfg = llm.mw.cfg
    li = layers[0]
    tier = tt.TrellisBaseTier(d, layers, act_limit=cfg.swiglu_limit)
    pool = tt.TrellisDeltaPool(tier, slots=2, dk13=3, dk2=3, L=8)
    true = [llm.mw.layers[li].experts.dequant_expert(e) for e in range(cfg.num_experts)]
    for e in (1, 4):
        assert pool.promote(li, e, *true[e]) in (0, 1)
    # the pooled experts are served closer to their true weights than by the base alone
    for e in (1, 4):
        b13, b2 = tier.dequant_expert(li, e)
        p13, p2 = pool.dequant_expert(li, e)
        assert (p13 - true[e][0]).norm() < 0.5 * (b13 - true[e][0]).norm()
        assert (p2 - true[e][1]).norm() < 0.5 * (b2 - true[e][1]).norm()
    assert torch.equal(pool.dequant_expert(li, 0)[0], tier.dequant_expert(li, 0)[0])
    torch.manual_seed(2)
    T = 5
    x = torch.randn(T, cfg.hidden)
    ids = torch.stack([torch.randperm(cfg.num_experts)[:cfg.top_k] for _ in range(T)])
    ids[0, 0], ids[1, 1] = 1, 4
    w = torch.rand(T, cfg.top_k)
    y = tier.forward_topk(li, x, ids, w, delta=pool)
    want = torch.zeros(T, cfg.hidden)
    for t in range(T):
        for j in range(cfg.top_k):
            w13, w2 = pool.dequant_expert(li, int(ids[t, j]))
            want[t] += w[t, j] * (swiglu(x[t:t + 1] @ w13.t(), cfg.swiglu_limit) @ w2.t())[0]
    assert torch.allclose(y, want, rtol=1e-4, atol=1e-5)
    # FIFO eviction once the slots are full; re-promotion keeps the expert's slot
    s4 = int(pool.slot_of[li][4])
    assert pool.promote(li, 4, *true[4]) == s4
    pool.promote(li, 6, *true[6])                 # evicts expert 1, the oldest promotion
    assert int(pool.slot_of[li][1]) == -1 and int(pool.slot_of[li][6]) >= 0
    assert pool.stats == {"promoted": 4, "evicted": 1}
    pool.evict(li, 6)
    assert int(pool.slot_of[li][6]) == -1
    y0 = tier.forward_topk(li, x, ids, w, delta=pool)     # only expert 4 is still pooled
    want0 = tier.forward_topk(li, x, ids, w)
    m = (ids == 4)
    assert torch.allclose(y0[~m.any(1)], want0[~m.any(1)], rtol=1e-5, atol=1e-6)
    assert not torch.allclose(y0[m.any(1)], want0[m.any(1)], rtol=1e-3, atol=1e-5)


def test_engine_with_delta_pool_matches_oracle(tiny_tier):
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.models import reference as ref
    _, d, layers = tiny_tier
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=128, trellis_pack=d)
    pool = tt.TrellisDeltaPool(llm.trellis, slots=3, L=8)
    for li in layers:
        for e in range(3):
            pool.promote(li, e, *llm.mw.layers[li].experts.dequant_expert(e))
    llm.trellis.attach_delta(pool)
    p = list(range(40, 64))
    out = llm.generate([p], SamplingParams(max_tokens=8, ignore_eos=True))[0].outputs[0].token_ids
    with ref.moe_context(llm.trellis.moe_fn(llm.mw)):
        assert out == ref.greedy_generate(llm.mw, p, 8)


def test_pack_builder_codes_checkpoint_experts_from_the_source(tmp_path, capsys):
    import json
    import sys as _sys
    _sys.path.insert(0, str(__import__("pathlib").Path(__file__).parent))
    from test_loader_cpu import _make_ckpt
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.tools.build_trellis_pack import main
    ck = str(tmp_path / "ckpt")
    _make_ckpt(ck, quant=True)
    out = str(tmp_path / "packs")
    assert main([out, "--checkpoint", ck, "--L", "8", "--w13-k", "3", "--w2-k", "3"]) == 0
    recs = [json.loads(x) for x in capsys.readouterr().out.strip().splitlines() if x.startswith("{")]
    llm = LLM(ck, device="cpu", num_speculative_tokens=0, max_model_len=64)
    moe = [li for li, lw in enumerate(llm.mw.layers) if lw.is_moe]
    assert [r["layer"] for r in recs] == moe
    tier = tt.TrellisBaseTier(out, moe)
    for li in moe:
        src13, src2 = next(tt.checkpoint_experts(ck, li, 1))
        t13, t2 = tier.dequant_expert(li, 0)
        c13, c2 = llm.mw.layers[li].experts.dequant_expert(0)       # the engine's 2-bit copy
        # 3-bit trellis from the source beats the 2-bit codebook on the same weights
        assert (t13 - src13).norm() < (c13 - src13).norm() and (t2 - src2).norm() < (c2 - src2).norm()
    # the tier serves the checkpoint through the engine
    eng = LLM(ck, device="cpu", num_speculative_tokens=0, max_model_len=64, trellis_pack=out)
    assert sorted(eng.trellis.layers) == moe
    assert len(eng.generate([[5, 6, 7]], __import__("vllm_moet_b200").SamplingParams(max_tokens=3,
                                                                                 ignore_eos=True))[0]
               .outputs[0].token_ids) == 3


def test_trellis_bench_cli_runs_on_cpu(capsys):
    import json
    from vllm_moet_b200.utils.trellis_bench import main
    assert main(["--hidden", "128", "--inter", "64", "--experts", "8", "--top-k", "2", "--tokens", "1,2",
                 "--iters", "1", "--warmup", "1", "--device", "cpu", "--L", "8"]) == 0
    recs = [json.loads(x) for x in capsys.readouterr().out.strip().splitlines()]
    assert [r["tokens"] for r in recs] == [1, 2] and all(r["us_per_block"] > 0 for r in recs)
