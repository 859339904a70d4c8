"""The delta-tier demo drives the real manager and trace: the slots fill, every resident
pair is unique, hit rates are rates, the trace line comes every `every` steps, and under
Zipf routing the token-weighted hit rate exceeds the distinct-pair rate."""
from vllm_moet_b200.tools.delta_trace_demo import run


def test_delta_trace_demo():
    lines = []
    snap = run(layers=6, experts=32, slots=20, steps=60, tokens=3, top_k=4, zipf=1.2, every=20, sink=lines.append)
    assert len(lines) == 3 and all("delta" in x for x in lines)
    assert snap["steps"] == 60 and snap["resident"] == 20
    res = snap["resident_map"]["resident"]
    assert len(res) == 20 and len({(li, e) for li, e, _ in res}) == 20 and len({s for _, _, s in res}) == 20
    assert 0 <= snap["hit_rate_distinct"] <= 1 and 0 <= snap["hit_rate_tokens"] <= 1
    assert snap["hit_rate_tokens"] > snap["hit_rate_distinct"]
    assert sum(snap["fp4_per_layer"]) == 20
