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
