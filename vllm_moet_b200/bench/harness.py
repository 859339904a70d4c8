"""Recipe runner, result lint and renderer (see the package docstring)."""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import time
from typing import List

import torch
import yaml

SCHEMA = 2
RECIPE_DIR = os.path.join(os.path.dirname(__file__), "recipes")
REQUIRED = ("schema", "recipe", "recipe_sha256", "git_commit", "source_fingerprint", "device", "results", "time")


def resolve_recipe(arg: str) -> str:
    if os.path.exists(arg):
        return arg
    p = os.path.join(RECIPE_DIR, arg if arg.endswith(".yaml") else arg + ".yaml")
    if not os.path.exists(p):
        raise FileNotFoundError(f"no recipe {arg!r} (have {sorted(os.listdir(RECIPE_DIR))})")
    return p


def file_sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def git_commit() -> str:
    try:
        return subprocess.run(["git", "rev-parse", "HEAD"], capture_output=True, text=True, timeout=10,
                              cwd=os.path.dirname(os.path.abspath(__file__))).stdout.strip() or "unknown"
    except (OSError, subprocess.SubprocessError):
        return "unknown"


def _sync(dev):
    if dev.type == "cuda":
        torch.cuda.synchronize()


def _parallel(rec: dict) -> dict:
    """Launch under torchrun for multi-rank recipes: `parallel: {tp, pp, ep}` -> LLM arguments.
    Ranks are laid out stage-major (rank = stage * tp + tp_rank); every group is created on
    every rank in the same order."""
    par = rec.get("parallel") or {}
    tp, pp, ep = int(par.get("tp", 1)), int(par.get("pp", 1)), bool(par.get("ep", False))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if tp * pp != world:
        raise SystemExit(f"recipe {rec['name']} needs tp * pp = {tp * pp} ranks, launched with {world} "
                         f"(torchrun --nproc-per-node {tp * pp} -m vllm_moet_b200.bench run ...)")
    if world == 1:
        return {}
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    cuda = torch.cuda.is_available() and rec.get("engine", {}).get("device", "cuda") != "cpu"
    if cuda:
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    if not dist.is_initialized():
        dist.init_process_group("nccl" if cuda else "gloo")
    stage, tr = divmod(rank, tp)
    tp_groups = [dist.new_group([s * tp + t for t in range(tp)]) for s in range(pp)] if tp > 1 else None
    pp_groups = [dist.new_group([s * tp + t for s in range(pp)]) for t in range(tp)] if pp > 1 else None
    kw = {}
    if tp > 1:
        kw.update(tensor_parallel_size=tp, tp_group=tp_groups[stage], tp_rank=tr, expert_parallel=ep)
    if pp > 1:
        kw.update(pipeline_parallel_size=pp, pp_group=pp_groups[tr], pp_rank=stage)
    return kw


def run_recipe_http(path: str, url: str) -> dict:
    """The recipe's probes against a running OpenAI-compatible server (`serve` mode):
    decode = concurrent streams of /v1/completions (wall-clock tok/s), prefill = one
    request with max_tokens 1 (prompt tok/s, i.e. time to first token), coherence = the
    same greedy request twice."""
    import concurrent.futures as cf
    import requests
    from ..ops.fingerprint import source_fingerprint
    with open(path) as f:
        rec = yaml.safe_load(f)
    url = url.rstrip("/")
    info = requests.get(url + "/v1/models", timeout=30).json()["data"][0]
    V = int(rec.get("vocab") or 259)            # token ids 3..V-1 exist in every preset (byte range)
    g = torch.Generator().manual_seed(0)

    def prompt(n):
        return torch.randint(3, V, (n,), generator=g).tolist()

    def complete(p, n):
        r = requests.post(url + "/v1/completions", json={"prompt": p, "max_tokens": n, "ignore_eos": True},
                          timeout=3600)
        r.raise_for_status()
        return r.json()["choices"][0]["token_ids"]
    results: List[dict] = []
    for pr in rec.get("probes", []):
        kind = pr["kind"]
        if kind == "decode":
            for S in pr["streams"]:
                ps = [prompt(pr["prompt_len"]) for _ in range(S)]
                with cf.ThreadPoolExecutor(S) as ex:
                    list(ex.map(lambda p: complete(p, 2), ps))              # warm
                    t0 = time.perf_counter()
                    outs = list(ex.map(lambda p: complete(p, pr["tokens"]), ps))
                    dt = time.perf_counter() - t0
                results.append({"probe": "decode", "streams": S, "tok_s": sum(map(len, outs)) / dt,
                                "wall_s": dt})
        elif kind == "prefill":
            for n in pr["lengths"]:
                p = prompt(n)
                complete(p, 1)
                t0 = time.perf_counter()
                complete(p, 1)
                dt = time.perf_counter() - t0
                results.append({"probe": "prefill", "length": n, "tok_s": n / dt, "ms": dt * 1e3})
        elif kind == "coherence":
            p = prompt(pr["prompt_len"])
            a, b = complete(p, pr["tokens"]), complete(p, pr["tokens"])
            results.append({"probe": "coherence", "identical": a == b, "tokens": len(a)})
        else:
            raise ValueError(f"unknown probe kind {kind!r}")
    return {"schema": SCHEMA, "recipe": rec["name"], "recipe_sha256": file_sha(path), "git_commit": git_commit(),
            "source_fingerprint": source_fingerprint(), "device": f"http {url} ({info['id']})", "results": results,
            "world": 1, "parallel": rec.get("parallel") or {}, "mode": "http",
            "time": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}


def run_recipe(path: str) -> dict:
    from ..engine.llm import LLM
    from ..engine.sampling_params import SamplingParams
    from ..ops.fingerprint import source_fingerprint
    with open(path) as f:
        rec = yaml.safe_load(f)
    eng = dict(rec.get("engine", {}))
    par = _parallel(rec)
    llm = LLM(rec["model"], **eng, **par, **rec.get("overrides", {}))
    g = torch.Generator().manual_seed(0)
    V = llm.cfg.vocab

    def prompt(n):
        return torch.randint(3, V, (n,), generator=g).tolist()
    results: List[dict] = []
    for pr in rec.get("probes", []):
        kind = pr["kind"]
        if kind == "decode":
            for S in pr["streams"]:
                ps = [prompt(pr["prompt_len"]) for _ in range(S)]
                sp = SamplingParams(max_tokens=pr["tokens"], ignore_eos=True)
                llm.generate(ps, SamplingParams(max_tokens=2, ignore_eos=True))
                outs = llm.generate(ps, sp)
                st = llm.stats
                gen = sum(len(o.outputs[0].token_ids) - 1 for o in outs)
                secs = st.get("decode_s") or 1e-9
                results.append({"probe": "decode", "streams": S, "tok_s": gen / secs if "decode_s" in st else None,
                                "steps": st.get("steps"), "accepted": st.get("accepted")})
        elif kind == "prefill":
            for n in pr["lengths"]:
                p = prompt(n)
                llm.generate([p], SamplingParams(max_tokens=1, ignore_eos=True))
                t0 = time.perf_counter()
                llm.generate([p], SamplingParams(max_tokens=1, ignore_eos=True))
                _sync(llm.device)
                dt = time.perf_counter() - t0
                results.append({"probe": "prefill", "length": n, "tok_s": n / dt, "ms": dt * 1e3})
        elif kind == "coherence":
            p = prompt(pr["prompt_len"])
            sp = SamplingParams(max_tokens=pr["tokens"], ignore_eos=True)
            a = llm.generate([p], sp)[0].outputs[0]
            b = llm.generate([p], sp)[0].outputs[0].token_ids
            from .stats import degenerate
            results.append({"probe": "coherence", "identical": a.token_ids == b, "tokens": len(a.token_ids),
                            "degenerate": degenerate(a.text)})
        elif kind == "needle":
            results.append(_needle(llm, pr))
        elif kind == "arithmetic":
            results.append(_arithmetic(llm, pr))
        elif kind == "quality":
            results.append(_quality(llm, rec, pr, prompt))
        elif kind == "shared_prefix":
            # requests sharing a long prefix: time to first token of the first (cold) and of
            # the later ones (prefix cache warm when the engine has it on)
            pre = prompt(pr["prefix_len"])
            ttft = []
            for i in range(pr["requests"]):
                p = pre + prompt(pr["suffix_len"])
                t0 = time.perf_counter()
                llm.generate([p], SamplingParams(max_tokens=1, ignore_eos=True))
                _sync(llm.device)
                ttft.append((time.perf_counter() - t0) * 1e3)
            bm = getattr(llm, "blocks", None)
            hits = (bm.stats["hit_blocks"] if bm is not None and getattr(bm, "prefix_caching", False)
                    else getattr(llm.runner, "prefix_stats", {}).get("hits"))
            results.append({"probe": "shared_prefix", "prefix_len": pr["prefix_len"], "cold_ms": ttft[0],
                            "warm_ms": sum(ttft[1:]) / max(1, len(ttft) - 1), "hits": hits})
        else:
            raise ValueError(f"unknown probe kind {kind!r}")
    dev = torch.cuda.get_device_name(0) if torch.cuda.is_available() and llm.device.type == "cuda" else "cpu"
    return {"schema": SCHEMA, "recipe": rec["name"], "recipe_sha256": file_sha(path), "git_commit": git_commit(),
            "source_fingerprint": source_fingerprint(), "device": dev, "results": results,
            "world": int(os.environ.get("WORLD_SIZE", "1")), "parallel": rec.get("parallel") or {},
            "time": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}


_FILLER = ("river stone lantern copper meadow violet harbor quiet thunder maple orbit canvas velvet "
           "pepper glacier saddle willow ember falcon marble").split()
_SECRET = "cobalt-heron-7319"
_ARITH = [("What is 219 * 37? Reply with only the number.", 8103),
          ("What is 64 * 58? Reply with only the number.", 3712),
          ("What is 1200 + 345 + 78 + 9? Reply with only the number.", 1632),
          ("What is 9081 - 4567? Reply with only the number.", 4514)]


def _needle(llm, pr) -> dict:
    """A passphrase at `depth` inside `words` filler words; pass if the answer holds it."""
    import random
    from ..engine.sampling_params import SamplingParams
    cases = []
    for n in pr.get("words", [200]):
        rnd = random.Random(11)
        filler = [rnd.choice(_FILLER) for _ in range(n)]
        at = int(n * pr.get("depth", 0.5))
        text = " ".join(filler[:at]) + f"\n\nThe vault passphrase is {_SECRET}.\n\n" + " ".join(filler[at:])
        msg = [{"role": "user", "content": text + "\n\nWhat is the vault passphrase? Reply with it only."}]
        out = llm.chat(msg, SamplingParams(max_tokens=pr.get("max_tokens", 24)))[0].outputs[0].text
        cases.append({"words": n, "pass": _SECRET in out})
    return {"probe": "needle", "cases": cases, "all_pass": all(c["pass"] for c in cases)}


def _arithmetic(llm, pr) -> dict:
    import re
    from ..engine.sampling_params import SamplingParams
    rows = []
    for q, gold in _ARITH:
        out = llm.chat([{"role": "user", "content": q}], SamplingParams(max_tokens=pr.get("max_tokens", 32)))
        nums = re.findall(r"-?\d+", out[0].outputs[0].text.replace(",", ""))
        got = int(nums[-1]) if nums else None
        rows.append({"gold": gold, "got": got, "ok": got == gold})
    return {"probe": "arithmetic", "score": sum(r["ok"] for r in rows), "of": len(rows), "rows": rows}


def _quality(llm, rec, pr, prompt) -> dict:
    """Paired A/B of the recipe's engine against `baseline` engine settings: an item is
    correct when the engine's greedy tokens equal the fp32 oracle's; McNemar and the
    paired token statistics decide the recipe's `gates`."""
    from ..engine.llm import LLM
    from ..engine.sampling_params import SamplingParams
    from ..models import reference
    from .stats import compare, passes
    eng = dict(rec.get("engine", {}), **pr.get("baseline", {}))
    base = LLM(rec["model"], **eng, **_parallel(rec), **rec.get("overrides", {}))
    sp = SamplingParams(max_tokens=pr["tokens"], ignore_eos=True)
    rows_c, rows_b = {}, {}
    for i in range(pr["items"]):
        p = prompt(pr["prompt_len"])
        want = reference.greedy_generate(llm.mw, p, pr["tokens"])
        for eng_, rows in ((llm, rows_c), (base, rows_b)):
            got = eng_.generate([p], sp)[0].outputs[0].token_ids
            rows[f"item{i}"] = {"correct": got == want, "tokens": len(got)}
    cmp_ = compare(rows_b, rows_c)
    return {"probe": "quality", "items": pr["items"], "vs_baseline": cmp_,
            "pass": passes(cmp_, pr.get("gates", {}))}


def lint(result: dict, recipe_path: str = None) -> List[str]:
    errs = [f"missing field {k}" for k in REQUIRED if k not in result]
    if result.get("schema") != SCHEMA:
        errs.append(f"schema {result.get('schema')} != {SCHEMA}")
    if recipe_path is None and "recipe" in result:
        try:
            recipe_path = resolve_recipe(result["recipe"])
        except FileNotFoundError:
            errs.append(f"recipe {result['recipe']} not found")
    if recipe_path and "recipe_sha256" in result and file_sha(recipe_path) != result["recipe_sha256"]:
        errs.append("recipe changed since the result was produced (sha256 mismatch)")
    for r in result.get("results", []):
        if "probe" not in r:
            errs.append("a result row without a probe kind")
    return errs


def render(results: List[dict]) -> str:
    rows = ["| recipe | device | probe | setting | value |", "|---|---|---|---|---|"]
    for res in results:
        for r in res["results"]:
            if r["probe"] == "decode":
                rows.append(f"| {res['recipe']} | {res['device']} | decode | {r['streams']} streams | "
                            f"{(r['tok_s'] or 0):.1f} tok/s |")
            elif r["probe"] == "prefill":
                rows.append(f"| {res['recipe']} | {res['device']} | prefill | {r['length']} tokens | "
                            f"{r['tok_s']:.0f} tok/s |")
            else:
                rows.append(f"| {res['recipe']} | {res['device']} | coherence | {r['tokens']} tokens | "
                            f"{'identical' if r['identical'] else 'DIFFERENT'} |")
    return "\n".join(rows)


def main(argv=None):
    ap = argparse.ArgumentParser(prog="python -m vllm_moet_b200.bench")
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run"); r.add_argument("recipe"); r.add_argument("--out", default="bench_results")
    r.add_argument("--url", default=None, help="run the probes against a running server instead of in-process")
    li = sub.add_parser("lint"); li.add_argument("files", nargs="+")
    rn = sub.add_parser("render"); rn.add_argument("files", nargs="+")
    a = ap.parse_args(argv)
    if a.cmd == "run":
        path = resolve_recipe(a.recipe)
        res = run_recipe_http(path, a.url) if a.url else run_recipe(path)
        if int(os.environ.get("RANK", "0")) == 0:
            os.makedirs(a.out, exist_ok=True)
            out = os.path.join(a.out, f"{res['recipe']}.{int(time.time())}.json")
            with open(out, "w") as f:
                json.dump(res, f, indent=1)
            print(out)
    elif a.cmd == "lint":
        bad = 0
        for fn in a.files:
            with open(fn) as f:
                errs = lint(json.load(f))
            for e in errs:
                print(f"{fn}: {e}")
            bad += bool(errs)
        sys.exit(1 if bad else 0)
    else:
        res = []
        for fn in a.files:
            with open(fn) as f:
                res.append(json.load(f))
        print(render(res))
