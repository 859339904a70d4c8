"""Inter-host PP prototype over localhost TCP: stage chains reproduce the
single-process greedy tokens, the injected RTT shows up as link time, and the
wire format round-trips tensors bit-exactly."""
import socket
import threading

import pytest
import torch

from vllm_moet_b200.config import tiny_config
from vllm_moet_b200.models import reference
from vllm_moet_b200.models.weights import random_weights
from vllm_moet_b200.parallel.interhost_pp import Driver, Stage, recv_frame, send_frame, serve_stage


def _cfg(hc=1):
    return tiny_config(num_layers=4, hc_mult=hc)


def _chain(stages, rtt_ms=0.0, hc=1):
    """Start stages 1..n-1 (listeners, last first) in threads; -> (driver, threads)."""
    cfg = _cfg(hc)
    listeners = [socket.create_server(("127.0.0.1", 0)) for _ in range(stages - 1)]
    ports = [ls.getsockname()[1] for ls in listeners]
    threads = []
    for s in range(stages - 1, 0, -1):
        nxt = ("127.0.0.1", ports[s]) if s < stages - 1 else None
        th = threading.Thread(target=serve_stage, args=(Stage(cfg, s, stages), listeners[s - 1], nxt, rtt_ms),
                              daemon=True)
        th.start()
        threads.append(th)
    return Driver(Stage(cfg, 0, stages), ("127.0.0.1", ports[0]), rtt_ms), threads, listeners


@pytest.mark.parametrize("stages,hc", [(2, 1), (3, 1), (2, 4)])
def test_chain_matches_single_process(stages, hc):
    """(hc 4: hyper-connection streams [T, 4, H] cross the links.)"""
    cfg = _cfg(hc)
    full = random_weights(cfg, "cpu", seed=0, with_mtp=False)
    prompt = [5, 9, 17, 33, 65, 129, 257, 513]
    want = reference.greedy_generate(full, prompt, 6)
    d, threads, listeners = _chain(stages, hc=hc)
    try:
        res = d.generate(prompt, 6)
        assert res["tokens"] == want
        again = d.generate(prompt, 6)                 # reset clears every stage's KV cache
        assert again["tokens"] == want
    finally:
        d.close()
        for th in threads:
            th.join(timeout=30)
        for ls in listeners:
            ls.close()


def test_injected_rtt_is_link_time():
    d, threads, listeners = _chain(2, rtt_ms=30.0)
    try:
        res = d.generate([3, 4, 5, 6], 5)
        assert res["per_token_ms"] >= 30.0                      # one round trip per token
        assert res["link_ms"] >= 25.0 and res["stage_compute_ms"] >= 0
        assert abs(res["per_token_ms"] - res["link_ms"] - res["stage_compute_ms"]) < 1e-6
    finally:
        d.close()
        for th in threads:
            th.join(timeout=30)
        for ls in listeners:
            ls.close()


def test_wire_format_roundtrip():
    a, b = socket.socketpair()
    try:
        t = {"h": torch.randn(3, 5).to(torch.bfloat16), "ids": torch.arange(7, dtype=torch.int64),
             "e": torch.empty(0, 4)}
        send_frame(a, {"op": "fwd", "positions": [1, 2, 3]}, t)
        hdr, got = recv_frame(b)
        assert hdr == {"op": "fwd", "positions": [1, 2, 3]}
        assert torch.equal(got["h"].view(torch.int16), t["h"].view(torch.int16)) and got["h"].dtype == torch.bfloat16
        assert torch.equal(got["ids"], t["ids"]) and got["e"].shape == (0, 4)
        with pytest.raises(TypeError):
            send_frame(a, {}, {"c": torch.zeros(2, dtype=torch.complex64)})
    finally:
        a.close()
        b.close()


def test_chain_with_trellis_served_experts(tmp_path):
    """Each stage serves its MoE layers from the trellis packs (global layer ids); the chain
    equals the single-process oracle under the same tier."""
    from vllm_moet_b200.residency import trellis_tier as tt
    cfg = _cfg()
    full = random_weights(cfg, "cpu", seed=0, with_mtp=False)
    layers = tt.write_model_packs(full, str(tmp_path), L=6)
    tier = tt.TrellisBaseTier(str(tmp_path), layers, act_limit=cfg.swiglu_limit)
    prompt = [5, 9, 17, 33, 65, 129]
    with reference.moe_context(tier.moe_fn(full)):
        want = reference.greedy_generate(full, prompt, 5)
    ls = socket.create_server(("127.0.0.1", 0))
    th = threading.Thread(target=serve_stage, args=(Stage(cfg, 1, 2, trellis_pack=str(tmp_path)), ls, None, 0.0),
                          daemon=True)
    th.start()
    d = Driver(Stage(cfg, 0, 2, trellis_pack=str(tmp_path)), ("127.0.0.1", ls.getsockname()[1]))
    try:
        assert d.st.moe_fn is not None
        assert d.generate(prompt, 5)["tokens"] == want
    finally:
        d.close()
        th.join(timeout=30)
        ls.close()
