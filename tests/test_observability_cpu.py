import json

import numpy as np
import torch

from vllm_moet_b200.utils.observability import KpiLogger, RoutingCapture, SpanTimers, percentiles, precision_map


def test_kpi_line_and_dump(tmp_path):
    lines = []
    k = KpiLogger(every=2, path=str(tmp_path / "kpi.json"), sink=lines.append)
    k.record_read(100.0)
    k.record_read(300.0)
    k.step(replayed=True, misses=3, fetched_rows=3, fetched_bytes=3 << 20)
    k.step()
    assert len(lines) == 1 and lines[0].startswith("[moet] KPI: steps 2 replay 50.0% misses 3")
    d = json.loads((tmp_path / "kpi.json").read_text())
    assert d["steps"] == 2 and d["read_us"]["p99"] == 300.0
    assert percentiles([1, 2, 3, 4])["p50"] in (2, 3)
    k.gauge(pool_slots=40, pool_pct=12.5, replay_ema=3.25, looka={"previous_step": 0.5, "router_lookahead": 0.75})
    k.c["draft_prefetched"] += 7
    ln = k.line()
    assert ln.endswith("; pool 40 slots = 12.5% of experts; draft-prefetched 7; replay EMA 3.2%; "
                       "LOOKA recall prev/router 0.50/0.75") or ln.endswith(
        "; pool 40 slots = 12.5% of experts; draft-prefetched 7; replay EMA 3.3%; LOOKA recall prev/router 0.50/0.75")
    assert k.snapshot()["pool_slots"] == 40


def test_routing_capture_and_precision_map(tmp_path):
    rc = RoutingCapture()
    rc.record([torch.tensor([[1, 2]]), None])
    rc.record([torch.tensor([[3, 4]]), torch.tensor([[5, 6]])])
    rc.save(str(tmp_path / "r.npy"))
    arr = np.load(tmp_path / "r.npy")
    assert arr.shape == (2, 2, 2) and arr[1, 1].tolist() == [5, 6] and arr[0, 1].tolist() == [-1, -1]

    class C:
        L, E = 2, 3
        mirror = torch.tensor([[-1, 4, -1], [0, -1, -1]])
    assert sorted(map(tuple, precision_map(C)["resident"])) == [(0, 1, 4), (1, 0, 0)]


def test_span_timers_cpu():
    t = SpanTimers()
    with t.span("prefill"):
        sum(range(1000))
    assert t.summary()["prefill"]["n"] == 1


def test_decode_roofline_model():
    from vllm_moet_b200.config import ds4_flash_config
    from vllm_moet_b200.utils.roofline import roofline, step_bytes
    cfg = ds4_flash_config()
    one = step_bytes(cfg, streams=1)
    many = step_bytes(cfg, streams=32)
    assert 20 < one["experts_distinct_per_layer"] < 24 and 230 < many["experts_distinct_per_layer"] <= 256
    assert many["experts"] > 9 * one["experts"] and many["dense"] == one["dense"]
    assert abs(step_bytes(cfg, streams=1, tp=2)["lm_head"] * 2 - one["lm_head"]) < 1
    r = roofline(cfg, 6549.1, streams=1, measured_ms=6.17)
    assert 1.0 < r["floor_ms"] < 1.3 and 0.15 < r["fraction_of_roofline"] < 0.25


def test_delta_policy_simulator(tmp_path):
    import numpy as np
    from vllm_moet_b200.tools.delta_sim import main, simulate
    rng = np.random.default_rng(0)
    steps, L, rows, E = 200, 3, 6, 32
    # a hot set of 4 experts per layer gets 80 % of the routing, the rest is uniform noise
    hot = rng.integers(0, E, (L, 4))
    routes = np.where(rng.random((steps, L, rows)) < 0.8, hot[None, :, rng.integers(0, 4, rows)].squeeze(),
                      rng.integers(0, E, (steps, L, rows))).astype(np.int32)
    routes[:, :, -1] = -1                                    # padding rows are ignored
    big = simulate(routes, slots=L * E, policy="lru")
    assert big["evictions_per_step"] == 0 and big["hit_rate_distinct"] > 0.9
    small_lru = simulate(routes, slots=16, policy="lru")
    small_freq = simulate(routes, slots=16, policy="freq")
    assert small_freq["hit_rate_tokens"] >= small_lru["hit_rate_tokens"] - 0.02   # frequency keeps the hot set
    assert 0 < small_freq["hit_rate_tokens"] <= 1 and small_lru["evictions_per_step"] > 0
    np.save(tmp_path / "r.npy", routes)
    main([str(tmp_path / "r.npy"), "--slots", "16", "--policy", "lru"])
