"""Data parallelism for serving: replicated engines behind a request router.

Each data-parallel replica is a complete engine -- one process on one GPU, or a
torchrun group of ``tp`` ranks over a slice of the GPUs -- serving the
OpenAI-compatible API of :mod:`.openai_server` on its own port.  The router is a
small HTTP front end that forwards every request to one replica and streams the
answer back unchanged:

* choice: the healthy replica with the fewest requests in flight (ties go
  round-robin), so long generations do not pile up on one engine;
* health: every replica's ``/health`` is polled; a replica that fails
  ``fail_after`` polls in a row (or refuses a connection) leaves the rotation
  until a poll succeeds again;
* failover: a request whose replica cannot be reached is retried on the next
  replica, as long as no byte of the answer has gone to the client;
* ``/metrics`` sums the replicas' counters and adds the router's own.

Upstream vLLM runs DP as replicated engine cores behind one API server
(``--data-parallel-size``); the reference inherits that and adds nothing of its
own.  Here the replicas are whole servers, so a replica is started, stopped and
health-checked on the host without touching the others' GPUs.

    python -m vllm_moet_b200.entrypoints.dp_router --backends http://127.0.0.1:8001,http://127.0.0.1:8002
"""
from __future__ import annotations

import argparse
import asyncio
import itertools
import json
from typing import Any, Dict, List, Optional

_COUNTER_PREFIX = "moet_"


class Replica:
    def __init__(self, url: str):
        self.url = url.rstrip("/")
        self.in_flight = 0
        self.served = 0
        self.failures = 0          # consecutive failed health polls
        self.healthy = True

    def __repr__(self):
        return f"Replica({self.url}, in_flight={self.in_flight}, healthy={self.healthy})"


class DPRouter:
    """Least-in-flight choice over healthy replicas (pure host logic)."""

    def __init__(self, urls: List[str], fail_after: int = 2):
        if not urls:
            raise ValueError("at least one replica URL is required")
        self.replicas = [Replica(u) for u in urls]
        self.fail_after = fail_after
        self._rr = itertools.count()
        self.stats = {"router_requests": 0, "router_retries": 0, "router_errors": 0}

    def healthy(self) -> List[Replica]:
        return [r for r in self.replicas if r.healthy]

    def pick(self, exclude=()) -> Optional[Replica]:
        cands = [r for r in self.healthy() if r not in exclude]
        if not cands:
            return None
        low = min(r.in_flight for r in cands)
        best = [r for r in cands if r.in_flight == low]
        return best[next(self._rr) % len(best)]

    def mark(self, rep: Replica, ok: bool):
        if ok:
            rep.failures, rep.healthy = 0, True
        else:
            rep.failures += 1
            if rep.failures >= self.fail_after:
                rep.healthy = False

    def metrics_text(self, replica_texts: List[str]) -> str:
        agg: Dict[str, float] = {}
        for text in replica_texts:
            for ln in text.splitlines():
                parts = ln.split()
                if len(parts) == 2 and parts[0].startswith(_COUNTER_PREFIX):
                    try:
                        agg[parts[0]] = agg.get(parts[0], 0.0) + float(parts[1])
                    except ValueError:
                        pass
        lines = [f"{k} {int(v) if float(v).is_integer() else v}" for k, v in sorted(agg.items())]
        lines += [f"moet_{k}_total {v}" for k, v in self.stats.items()]
        lines.append(f"moet_router_healthy_replicas {len(self.healthy())}")
        for i, r in enumerate(self.replicas):
            lines.append(f'moet_router_replica_in_flight{{replica="{i}"}} {r.in_flight}')
            lines.append(f'moet_router_replica_served_total{{replica="{i}"}} {r.served}')
        return "\n".join(lines) + "\n"


def build_router_app(router: DPRouter, poll_s: float = 2.0, timeout_s: float = 600.0):
    import aiohttp
    import contextlib
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, Response, StreamingResponse

    state: Dict[str, object] = {}

    async def session() -> "aiohttp.ClientSession":
        s = state.get("session")
        if s is None:
            s = aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=timeout_s))
            state["session"] = s
        return s

    async def poll_once():
        s = await session()
        for rep in router.replicas:
            try:
                async with s.get(rep.url + "/health", timeout=aiohttp.ClientTimeout(total=2.0)) as r:
                    router.mark(rep, r.status == 200)
            except (aiohttp.ClientError, asyncio.TimeoutError):
                router.mark(rep, False)

    async def poller():
        while True:
            await poll_once()
            await asyncio.sleep(poll_s)

    @contextlib.asynccontextmanager
    async def lifespan(_app):
        state["poller"] = asyncio.create_task(poller())
        yield
        state["poller"].cancel()
        s = state.get("session")
        if s is not None:
            await s.close()

    app = FastAPI(title="vllm_moet_b200 data-parallel router", lifespan=lifespan)

    async def forward(path: str, body: Dict):
        """POST to one replica; retry on another while nothing has been sent back."""
        router.stats["router_requests"] += 1
        tried: List[Replica] = []
        s = await session()
        while True:
            rep = router.pick(exclude=tried)
            if rep is None:
                router.stats["router_errors"] += 1
                raise HTTPException(503, "no healthy data-parallel replica")
            tried.append(rep)
            rep.in_flight += 1
            try:
                resp = await s.post(rep.url + path, json=body)
            except (aiohttp.ClientError, asyncio.TimeoutError):
                rep.in_flight -= 1
                rep.failures, rep.healthy = router.fail_after, False   # a refused connection takes it out at once
                router.stats["router_retries"] += 1
                continue
            rep.served += 1
            if body.get("stream") and resp.status == 200:
                async def relay():
                    try:
                        async for chunk in resp.content.iter_any():
                            yield chunk
                    finally:
                        resp.release()
                        rep.in_flight -= 1
                return StreamingResponse(relay(), media_type="text/event-stream")
            try:
                data = await resp.read()
            finally:
                resp.release()
                rep.in_flight -= 1
            return Response(content=data, status_code=resp.status,
                            media_type=resp.headers.get("content-type", "application/json"))

    @app.post("/v1/completions")
    async def completions(body: Dict[str, Any]):
        return await forward("/v1/completions", body)

    @app.post("/v1/chat/completions")
    async def chat(body: Dict[str, Any]):
        return await forward("/v1/chat/completions", body)

    @app.get("/health")
    async def health():
        n = len(router.healthy())
        if n == 0:
            raise HTTPException(503, "no healthy data-parallel replica")
        return {"status": "ok", "healthy_replicas": n, "replicas": len(router.replicas)}

    @app.get("/v1/models")
    async def models():
        s = await session()
        for rep in router.healthy():
            try:
                async with s.get(rep.url + "/v1/models") as r:
                    if r.status == 200:
                        return JSONResponse(json.loads(await r.read()))
            except aiohttp.ClientError:
                router.mark(rep, False)
        raise HTTPException(503, "no healthy data-parallel replica")

    @app.get("/metrics")
    async def metrics():
        s = await session()
        texts = []
        for rep in router.replicas:
            try:
                async with s.get(rep.url + "/metrics", timeout=aiohttp.ClientTimeout(total=2.0)) as r:
                    if r.status == 200:
                        texts.append((await r.read()).decode())
            except (aiohttp.ClientError, asyncio.TimeoutError):
                pass
        return PlainTextResponse(router.metrics_text(texts))

    app.state.router = router
    app.state.poll_once = poll_once
    return app


def main(argv=None):
    ap = argparse.ArgumentParser(description="data-parallel request router")
    ap.add_argument("--backends", required=True, help="comma-separated replica base URLs")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--poll-s", type=float, default=2.0)
    args = ap.parse_args(argv)
    import uvicorn
    router = DPRouter([u for u in args.backends.split(",") if u])
    uvicorn.run(build_router_app(router, poll_s=args.poll_s), host=args.host, port=args.port, log_level="warning")


if __name__ == "__main__":
    main()
