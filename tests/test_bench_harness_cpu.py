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
    assert kinds.count("decode") == 2 and {"probe": "coherence", "identical": True, "tokens": 8} in res["results"]
    table = render([res])
    assert "| tiny_cpu | cpu | coherence | 8 tokens | identical |" in table
    rec.write_text(rec.read_text() + "\n# edited\n")
    assert any("sha256" in e for e in lint(res, str(rec)))
    bad = dict(res)
    del bad["git_commit"]
    assert "missing field git_commit" in lint(bad, str(rec))
    json.dumps(res)
