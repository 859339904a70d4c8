"""Data-parallel serving: replica choice, health, failover, launch commands (CPU)."""
import json
import socket
import threading
import time

import pytest
import requests

from vllm_moet_b200.entrypoints.dp_router import DPRouter, build_router_app
from vllm_moet_b200.entrypoints.dp_serve import replica_commands


def test_pick_least_in_flight_round_robin_and_health():
    r = DPRouter(["http://a", "http://b", "http://c"], fail_after=2)
    a, b, c = r.replicas
    first = [r.pick().url for _ in range(3)]
    assert sorted(first) == ["http://a", "http://b", "http://c"]      # ties rotate
    a.in_flight, b.in_flight, c.in_flight = 2, 0, 1
    assert r.pick() is b
    assert r.pick(exclude=[b]) is c
    r.mark(b, False)
    assert b.healthy                                                   # one failed poll is tolerated
    r.mark(b, False)
    assert not b.healthy and r.pick() is c
    r.mark(b, True)
    assert b.healthy and r.pick() is b
    for rep in r.replicas:
        r.mark(rep, False), r.mark(rep, False)
    assert r.pick() is None
    with pytest.raises(ValueError):
        DPRouter([])


def test_metrics_aggregate():
    r = DPRouter(["http://a", "http://b"])
    text = r.metrics_text(["moet_requests_total 3\nmoet_generated_tokens_total 10\n",
                           "moet_requests_total 4\nother 1\n"])
    assert "moet_requests_total 7" in text and "moet_generated_tokens_total 10" in text
    assert "moet_router_healthy_replicas 2" in text and "other" not in text


def test_replica_commands_gpu_slices_and_ports():
    cmds = replica_commands("ds4-flash-shape", dp=2, tp=2, port=8000, extra=["--max-num-seqs", "8"],
                            gpus=[0, 1, 2, 3], python="py")
    (a0, e0, u0), (a1, e1, u1) = cmds
    assert e0["CUDA_VISIBLE_DEVICES"] == "0,1" and e1["CUDA_VISIBLE_DEVICES"] == "2,3"
    assert u0.endswith(":8001") and u1.endswith(":8002")
    assert a0[:3] == ["py", "-m", "torch.distributed.run"] and "--nproc-per-node=2" in a0
    assert "127.0.0.1" in a0 and a0[a0.index("--master-port") + 1] != a1[a1.index("--master-port") + 1]
    assert a0[-2:] == ["--max-num-seqs", "8"]
    single = replica_commands("tiny-moe", dp=3, tp=1, port=9000, extra=[], gpus=None, python="py")
    assert [c[0][:3] for c in single] == [["py", "-m", "vllm_moet_b200.entrypoints.openai_server"]] * 3
    assert all(c[1] == {} for c in single)
    with pytest.raises(ValueError):
        replica_commands("m", dp=2, tp=2, port=1, extra=[], gpus=[0, 1, 2])


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _serve(app):
    import uvicorn
    port = _free_port()
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(200):
        try:
            requests.get(url + "/health", timeout=1)
            break
        except requests.ConnectionError:
            time.sleep(0.05)
    return srv, th, url


@pytest.fixture(scope="module")
def dp_cluster():
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.entrypoints.openai_server import EngineWorker, build_app
    reps = []
    for _ in range(2):
        llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
        w = EngineWorker(llm, "tiny-moe")
        srv, th, url = _serve(build_app(w))
        reps.append((srv, th, url, w, llm))
    router = DPRouter([r[2] for r in reps], fail_after=1)
    rsrv, rth, rurl = _serve(build_router_app(router, poll_s=0.2))
    yield rurl, router, reps
    rsrv.should_exit = True
    rth.join(timeout=10)
    for srv, th, _, w, _ in reps:
        srv.should_exit = True
        th.join(timeout=10)
        w.close()


def test_router_results_spread_and_streaming(dp_cluster):
    url, router, reps = dp_cluster
    from vllm_moet_b200.models import reference
    want = reference.greedy_generate(reps[0][4].mw, [5, 6, 7, 8], 6)
    outs = []

    def one():
        r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 6,
                                                         "ignore_eos": True}, timeout=120)
        outs.append(r)
    ths = [threading.Thread(target=one) for _ in range(4)]
    [t.start() for t in ths]
    [t.join() for t in ths]
    assert all(r.ok for r in outs), [r.text for r in outs]
    assert all(r.json()["choices"][0]["token_ids"] == want for r in outs)
    assert all(rep.served >= 1 for rep in router.replicas)            # both replicas took requests
    r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 5, "stream": True,
                                                     "ignore_eos": True}, stream=True, timeout=120)
    events = [ln[6:] for ln in r.iter_lines(decode_unicode=True) if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    assert sum((json.loads(e)["choices"][0]["token_ids"] for e in events[:-1]), []) == want[:5]
    assert requests.get(url + "/v1/models").json()["data"][0]["id"] == "tiny-moe"
    m = requests.get(url + "/metrics").text
    assert "moet_requests_total" in m and "moet_router_requests_total" in m
    assert requests.get(url + "/health").json()["healthy_replicas"] == 2
    assert requests.post(url + "/v1/completions", json={"prompt": "x", "temperature": -1}).status_code == 400


def test_router_fails_over_when_a_replica_stops(dp_cluster):
    url, router, reps = dp_cluster
    srv, th, rep_url, _, _ = reps[1]
    srv.should_exit = True            # replica 1 goes away between requests
    th.join(timeout=10)
    for _ in range(100):
        if requests.get(url + "/health").json()["healthy_replicas"] == 1:
            break
        time.sleep(0.1)
    assert requests.get(url + "/health").json()["healthy_replicas"] == 1
    for _ in range(3):
        r = requests.post(url + "/v1/completions", json={"prompt": [9, 10], "max_tokens": 3, "ignore_eos": True},
                          timeout=120)
        assert r.ok, r.text
        assert len(r.json()["choices"][0]["token_ids"]) == 3
    # a connection refused by the stopped replica is retried on the live one (the health
    # poller may take the replica out again first, so try a few times)
    for _ in range(10):
        before = router.stats["router_retries"]
        router.replicas[1].healthy, router.replicas[1].failures = True, 0
        router.replicas[0].in_flight += 5          # make the dead replica the first choice
        try:
            r = requests.post(url + "/v1/completions", json={"prompt": [9, 10], "max_tokens": 2,
                                                             "ignore_eos": True}, timeout=120)
        finally:
            router.replicas[0].in_flight -= 5
        assert r.ok, r.text
        if router.stats["router_retries"] > before:
            break
    assert router.stats["router_retries"] > before and not router.replicas[1].healthy


def test_dp_serve_launches_replicas_and_router():
    """`openai_server --data-parallel-size 2` on CPU: two replica processes and the router."""
    import os
    import signal
    import subprocess
    import sys
    port = _free_port()
    argv = [sys.executable, "-m", "vllm_moet_b200.entrypoints.openai_server", "--model", "tiny-moe",
            "--data-parallel-size", "2", "--gpus", "cpu", "--device", "cpu", "--port", str(port),
            "--max-model-len", "256", "--max-num-seqs", "4"]
    env = dict(os.environ, MOET_SKIP_BUILD_CHECK="1")
    proc = subprocess.Popen(argv, env=env, start_new_session=True, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    url = f"http://127.0.0.1:{port}"
    try:
        ok = False
        for _ in range(600):
            if proc.poll() is not None:
                break
            try:
                if requests.get(url + "/health", timeout=1).ok:
                    ok = True
                    break
            except requests.RequestException:
                time.sleep(0.2)
        assert ok, proc.stdout.read().decode()[-2000:] if proc.poll() is not None else "router not healthy"
        assert requests.get(url + "/health").json()["replicas"] == 2
        r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 3, "ignore_eos": True},
                          timeout=120)
        assert r.ok and len(r.json()["choices"][0]["token_ids"]) == 3
    finally:
        os.killpg(proc.pid, signal.SIGTERM)       # the launcher's own group; it stops its replicas
        try:
            proc.wait(timeout=60)
        except subprocess.TimeoutExpired:
            os.killpg(proc.pid, signal.SIGKILL)
    # the launcher stopped its replicas on the way out
    for p in (port + 1, port + 2):
        with pytest.raises(requests.ConnectionError):
            requests.get(f"http://127.0.0.1:{p}/health", timeout=2)
