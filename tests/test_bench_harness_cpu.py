import json
import shutil

from vllm_moet_b200.bench.harness import lint, render, resolve_recipe, run_recipe
from vllm_moet_b200.ops.fingerprint import source_fingerprint


def test_tiny_recipe_run_lint_render(tmp_path):
    src = resolve_recipe("tiny_cpu")
    rec = tmp_path / "tiny_cpu.yaml"
    shutil.copy(src, rec)
    res = run_recipe(str(rec))
    assert res["source_fingerprint"] == source_fingerprint()
    assert not lint(res, str(rec))
    kinds = [r["probe"] for r in res["results"]]
    assert kinds.count("decode") == 2 and {"probe": "coherence", "identical": True, "tokens": 8, "degenerate": False} in res["results"]
    table = render([res])
    assert "| tiny_cpu | cpu | coherence | 8 tokens | identical |" in table
    rec.write_text(rec.read_text() + "\n# edited\n")
    assert any("sha256" in e for e in lint(res, str(rec)))
    bad = dict(res)
    del bad["git_commit"]
    assert "missing field git_commit" in lint(bad, str(rec))
    json.dumps(res)


def test_multi_rank_recipe_under_torchrun(tmp_path):
    """A `parallel: {tp: 2}` recipe launched with torchrun (gloo on CPU): rank 0 writes one
    result that lints; a multi-rank recipe started as one process is refused."""
    import json
    import os
    import socket
    import subprocess
    import sys
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    out = tmp_path / "res"
    env = dict(os.environ, MOET_SKIP_BUILD_CHECK="1")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", str(port), "-m", "vllm_moet_b200.bench", "run",
                        "tiny_cpu_tp2", "--out", str(out)], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    files = list(out.iterdir())
    assert len(files) == 1
    from vllm_moet_b200.bench.harness import lint
    res = json.loads(files[0].read_text())
    assert lint(res) == [] and res["world"] == 2 and res["parallel"] == {"tp": 2}
    assert any(x["probe"] == "coherence" and x["identical"] for x in res["results"])
    r1 = subprocess.run([sys.executable, "-m", "vllm_moet_b200.bench", "run", "tiny_cpu_tp2", "--out", str(out)],
                        capture_output=True, text=True, timeout=300, env=env)
    assert r1.returncode != 0 and "needs tp * pp = 2 ranks" in (r1.stderr + r1.stdout)


def test_every_recipe_is_well_formed():
    import inspect
    import os
    import yaml
    from vllm_moet_b200.bench.harness import RECIPE_DIR
    from vllm_moet_b200.engine.llm import LLM
    params = set(inspect.signature(LLM.__init__).parameters) - {"self", "model"}
    for fn in sorted(os.listdir(RECIPE_DIR)):
        rec = yaml.safe_load(open(os.path.join(RECIPE_DIR, fn)))
        assert rec["name"] == fn[:-5], fn
        assert set(rec.get("engine", {})) <= params | {"device"}, (fn, set(rec["engine"]) - params)
        assert all(p["kind"] in ("decode", "prefill", "coherence", "shared_prefix", "needle", "arithmetic",
                                 "quality") for p in rec["probes"]), fn
        assert set(rec.get("parallel") or {}) <= {"tp", "pp", "ep"}, fn


def test_recipe_probes_over_http(tmp_path):
    """`bench run <recipe> --url ...`: the same probes against a running server."""
    import json
    import socket
    import threading
    import time
    import requests
    import uvicorn
    from vllm_moet_b200.bench.harness import lint, main
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.entrypoints.openai_server import EngineWorker, build_app
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256, max_num_seqs=4)
    w = EngineWorker(llm, "tiny-moe")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    srv = uvicorn.Server(uvicorn.Config(build_app(w), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{port}"
    try:
        for _ in range(100):
            try:
                if requests.get(url + "/health", timeout=1).ok:
                    break
            except requests.ConnectionError:
                time.sleep(0.1)
        main(["run", "tiny_cpu", "--out", str(tmp_path), "--url", url])
        (f,) = list(tmp_path.iterdir())
        res = json.loads(f.read_text())
        assert lint(res) == [] and res["mode"] == "http"
        dec = [r for r in res["results"] if r["probe"] == "decode"]
        assert [r["streams"] for r in dec] == [1, 4] and all(r["tok_s"] > 0 for r in dec)
        assert any(r["probe"] == "coherence" and r["identical"] for r in res["results"])
    finally:
        srv.should_exit = True
        th.join(timeout=10)
        w.close()


def test_shared_prefix_probe_reports_cache_hits():
    from vllm_moet_b200.bench.harness import lint, resolve_recipe, run_recipe
    res = run_recipe(resolve_recipe("tiny_cpu_prefix"))
    row = [r for r in res["results"] if r["probe"] == "shared_prefix"][0]
    assert row["hits"] == 3 and row["cold_ms"] > 0 and row["warm_ms"] > 0
    assert not lint(res)


def test_quality_needle_and_arithmetic_probes():
    """The quality probe pairs the recipe's engine (MTP k=2) with a baseline (no
    speculation) against the oracle: both exact, so McNemar finds nothing and the gates
    pass; needle and arithmetic report structured results (random weights fail them)."""
    from vllm_moet_b200.bench.harness import lint, resolve_recipe, run_recipe
    res = run_recipe(resolve_recipe("tiny_cpu_quality"))
    q = [r for r in res["results"] if r["probe"] == "quality"][0]
    assert q["pass"] and q["vs_baseline"]["acc_cand"] == q["vs_baseline"]["acc_base"] == 1.0
    a = [r for r in res["results"] if r["probe"] == "arithmetic"][0]
    n = [r for r in res["results"] if r["probe"] == "needle"][0]
    assert a["of"] == 4 and 0 <= a["score"] <= 4 and n["cases"][0]["words"] == 60
    assert not lint(res)
