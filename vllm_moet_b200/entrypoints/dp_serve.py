"""Launch ``dp`` engine replicas of ``tp`` GPUs each, plus the request router.

    python -m vllm_moet_b200.entrypoints.dp_serve --model ds4-flash-shape \\
        --data-parallel-size 4 --tensor-parallel-size 2 --port 8000

Replica ``i`` gets GPUs ``[i*tp, (i+1)*tp)`` (through ``CUDA_VISIBLE_DEVICES``)
and serves on ``port + 1 + i``; a replica of more than one GPU is a torchrun
group (rendezvous on 127.0.0.1, its own master port).  The router listens on
``port``.  Children are stopped by their own process ids when the router exits.
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time
from typing import List, Optional


def replica_commands(model: str, dp: int, tp: int, port: int, extra: List[str], gpus: Optional[List[int]] = None,
                     master_port: int = 29600, python: str = sys.executable):
    """-> [(argv, env_overrides, url)] for every replica (no process started)."""
    out = []
    for i in range(dp):
        p = port + 1 + i
        env = {}
        if gpus is not None:
            sl = gpus[i * tp:(i + 1) * tp]
            if len(sl) != tp:
                raise ValueError(f"{dp} replicas x {tp} GPUs need {dp * tp} GPUs, have {len(gpus)}")
            env["CUDA_VISIBLE_DEVICES"] = ",".join(map(str, sl))
        server = ["-m", "vllm_moet_b200.entrypoints.openai_server", "--model", model, "--port", str(p)] + extra
        if tp > 1:
            argv = [python, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={tp}",
                    "--master-addr", "127.0.0.1", "--master-port", str(master_port + i)] + server
        else:
            argv = [python] + server
        out.append((argv, env, f"http://127.0.0.1:{p}"))
    return out


def wait_healthy(urls: List[str], timeout_s: float = 1800.0, procs=None) -> None:
    import requests
    t0 = time.time()
    pending = list(urls)
    while pending:
        if procs is not None:
            dead = [p.args for p in procs if p.poll() is not None]
            if dead:
                raise RuntimeError(f"replica exited during startup: {dead[0]}")
        for u in list(pending):
            try:
                if requests.get(u + "/health", timeout=1).ok:
                    pending.remove(u)
            except requests.RequestException:
                pass
        if pending and time.time() - t0 > timeout_s:
            raise TimeoutError(f"replicas not healthy after {timeout_s:.0f} s: {pending}")
        if pending:
            time.sleep(1.0)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="ds4-flash-shape")
    ap.add_argument("--data-parallel-size", type=int, default=1)
    ap.add_argument("--tensor-parallel-size", type=int, default=1)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--gpus", default=None, help="comma-separated GPU ids (default: 0..dp*tp-1; 'cpu' for none)")
    args, extra = ap.parse_known_args(argv)
    extra = [a for a in extra if not a.startswith("--data-parallel-size")]
    dp, tp = args.data_parallel_size, args.tensor_parallel_size
    gpus = None if args.gpus == "cpu" else (
        [int(x) for x in args.gpus.split(",")] if args.gpus else list(range(dp * tp)))
    cmds = replica_commands(args.model, dp, tp, args.port, extra, gpus)
    procs = []

    def _on_term(signum, frame):       # SIGTERM ends the launcher through the cleanup below
        raise SystemExit(128 + signum)
    signal.signal(signal.SIGTERM, _on_term)
    try:
        for argv_i, env_i, _ in cmds:
            env = dict(os.environ)
            env.update(env_i)
            procs.append(subprocess.Popen(argv_i, env=env, start_new_session=True))
        urls = [u for _, _, u in cmds]
        wait_healthy(urls, procs=procs)
        from .dp_router import main as router_main
        router_main(["--backends", ",".join(urls), "--host", args.host, "--port", str(args.port)])
    finally:
        for p in procs:
            if p.poll() is None:
                try:
                    os.killpg(p.pid, signal.SIGTERM)      # the replica's own process group (torchrun + ranks)
                except ProcessLookupError:
                    pass
        for p in procs:
            try:
                p.wait(timeout=30)
            except subprocess.TimeoutExpired:
                os.killpg(p.pid, signal.SIGKILL)


if __name__ == "__main__":
    main()
