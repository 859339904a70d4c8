"""OpenAI-compatible HTTP server over the engine.

    python -m vllm_moet_b200.entrypoints.openai_server --model ds4-flash-shape --port 8000
    torchrun --nproc-per-node 8 -m vllm_moet_b200.entrypoints.openai_server --model ds4-flash-shape
    python -m vllm_moet_b200.entrypoints.openai_server --data-parallel-size 4 --tensor-parallel-size 2

Endpoints: ``GET /health``, ``GET /v1/models``, ``POST /v1/completions``,
``POST /v1/chat/completions`` (DeepSeek-V4 chat encoding, ``reasoning_effort``,
tools; ``stream: true`` sends server-sent events ending in ``data: [DONE]``),
``GET /metrics`` (Prometheus text).

Requests are queued to one engine thread that batches whatever is waiting
into a single ``LLM.generate`` call (the engine refills finished rows while
decoding).  Under tensor parallelism rank 0 serves HTTP and broadcasts each
batch to the other ranks (``torch.distributed.broadcast_object_list``), which
run the same ``generate`` call in lock step.
"""
from __future__ import annotations

import argparse
import asyncio
import itertools
import json
import os
import queue
import threading
import time
import uuid
from typing import Any, Dict, List, Optional

from ..engine.sampling_params import SamplingParams, cut_at_stop
from . import chat_encoding


class EngineWorker:
    """Owns the LLM on one thread; requests come in through a queue.  A request that
    arrives while a batch is decoding joins it between steps (up to the running batch
    size); `abort(request_id)` finishes a request at the next step."""

    def __init__(self, llm, model_name: str, tp_group=None, max_batch: int = 32):
        self.llm, self.model_name, self.group = llm, model_name, tp_group
        self.max_batch = max_batch
        self.q: "queue.Queue" = queue.Queue()
        self.stats = {"requests": 0, "prompt_tokens": 0, "generated_tokens": 0, "batches": 0, "joined": 0,
                      "aborted": 0, "decode_steps": 0, "accepted_draft_tokens": 0}
        self._ids = itertools.count()
        self._aborts: set = set()
        self._lock = threading.Lock()
        self._stop = False
        self.thread = threading.Thread(target=self._loop, name="engine", daemon=True)
        self.thread.start()

    def submit(self, prompt_ids: List[int], params: SamplingParams, on_tokens) -> str:
        rid = f"srv-{next(self._ids)}"
        self.q.put((rid, prompt_ids, params, on_tokens))
        return rid

    def abort(self, rid: str) -> None:
        with self._lock:
            self._aborts.add(rid)
        self.stats["aborted"] += 1

    def _loop(self):
        while not self._stop:
            item = self.q.get()
            if item is None:
                break
            batch = [item]
            while len(batch) < self.max_batch:
                try:
                    nxt = self.q.get_nowait()
                except queue.Empty:
                    break
                if nxt is None:
                    self._stop = True
                    break
                batch.append(nxt)
            self._run(batch)
        if self.group is not None:
            import torch.distributed as dist
            dist.broadcast_object_list([None], src=0, group=self.group)

    def _between(self, n_free: int):
        """Serving hook of LLM.generate: requests that arrived meanwhile, aborts."""
        items = []
        while len(items) < n_free and not self._stop:
            try:
                it = self.q.get_nowait()
            except queue.Empty:
                break
            if it is None:              # shutdown: finish the running batch first
                self._stop = True
                break
            items.append(it)
        with self._lock:
            aborts, self._aborts = self._aborts, set()
        self.stats["joined"] += len(items)
        self.stats["requests"] += len(items)
        self.stats["prompt_tokens"] += sum(len(it[1]) for it in items)
        if self.group is not None:
            import torch.distributed as dist
            dist.broadcast_object_list([([it[:3] for it in items], aborts)], src=0, group=self.group)
        return items, aborts

    def _run(self, batch):
        rids = [b[0] for b in batch]
        prompts = [b[1] for b in batch]
        params = [b[2] for b in batch]
        if self.group is not None:
            import torch.distributed as dist
            dist.broadcast_object_list([(prompts, params, rids)], src=0, group=self.group)
        self.stats["batches"] += 1
        self.stats["requests"] += len(batch)
        self.stats["prompt_tokens"] += sum(len(p) for p in prompts)
        try:
            outs = self.llm.generate(prompts, params, callbacks=[b[3] for b in batch], request_ids=rids,
                                     between_steps=self._between)
            self.stats["generated_tokens"] += sum(len(o.outputs[0].token_ids) for o in outs)
            self._engine_counters()
        except Exception as e:  # noqa: BLE001 - report to every waiting request
            for b in batch:
                b[3]([], "error:" + str(e))

    def _engine_counters(self):
        """Speculative-decoding and prefix-cache counters of the run that just ended."""
        st = getattr(self.llm, "stats", {}) or {}
        self.stats["decode_steps"] += int(st.get("steps") or 0)
        self.stats["accepted_draft_tokens"] += int(st.get("accepted") or 0)
        bm = getattr(self.llm, "blocks", None)
        if bm is not None and getattr(bm, "prefix_caching", False):
            self.stats["prefix_cache_hit_blocks"] = bm.stats["hit_blocks"]
        ps = getattr(getattr(self.llm, "runner", None), "prefix_stats", None)
        if ps is not None:
            self.stats["prefix_cache_hits"] = ps["hits"]

    def close(self):
        self.q.put(None)
        self.thread.join(timeout=10)


def follower_loop(llm, tp_group):
    """Ranks > 0 under TP: run each broadcast batch in lock step with rank 0, including
    the requests that join it and the aborts (received at the same points of the loop)."""
    import torch.distributed as dist

    def between(n_free):
        box = [None]
        dist.broadcast_object_list(box, src=0, group=tp_group)
        items, aborts = box[0]
        return [(rid, p, sp, None) for rid, p, sp in items], aborts
    while True:
        box = [None]
        dist.broadcast_object_list(box, src=0, group=tp_group)
        if box[0] is None:
            return
        prompts, params, rids = box[0]
        llm.generate(prompts, params, request_ids=rids, between_steps=between)


UNSUPPORTED_FIELDS = ("guided_json", "guided_regex", "guided_choice", "guided_grammar", "structured_outputs")


def _params_from(body: Dict[str, Any], default_max: int = 16) -> SamplingParams:
    # constrained decoding is not served: refuse it instead of answering unconstrained
    rf = body.get("response_format")
    if isinstance(rf, dict) and rf.get("type", "text") != "text":
        raise ValueError(f"response_format {rf.get('type')!r} is not supported (plain text only)")
    bad = [k for k in UNSUPPORTED_FIELDS if body.get(k) is not None]
    if bad:
        raise ValueError(f"constrained decoding is not supported: {', '.join(bad)}")
    temp = float(body.get("temperature", 0.0) or 0.0)
    if temp < 0:
        raise ValueError("temperature must be >= 0")
    stop_ids = list(body.get("stop_token_ids") or [])
    stop = body.get("stop") or []
    seed = body.get("seed")
    lp = body.get("logprobs")
    if isinstance(lp, bool):          # chat: logprobs true + top_logprobs n
        lp = int(body.get("top_logprobs") or 0) if lp else None
    elif lp is not None:
        lp = int(lp)
    return SamplingParams(max_tokens=int(body.get("max_tokens") or body.get("max_completion_tokens") or default_max),
                          temperature=temp, top_p=float(body.get("top_p", 1.0) or 1.0),
                          top_k=int(body.get("top_k") or 0), seed=None if seed is None else int(seed),
                          stop_token_ids=stop_ids, ignore_eos=bool(body.get("ignore_eos", False)),
                          stop=[stop] if isinstance(stop, str) else list(stop),
                          include_stop_str_in_output=bool(body.get("include_stop_str_in_output", False)),
                          min_tokens=int(body.get("min_tokens") or 0), logprobs=lp, n=int(body.get("n") or 1),
                          presence_penalty=float(body.get("presence_penalty") or 0.0),
                          frequency_penalty=float(body.get("frequency_penalty") or 0.0),
                          repetition_penalty=float(body.get("repetition_penalty") or 1.0),
                          min_p=float(body.get("min_p") or 0.0),
                          logit_bias={int(k): float(v) for k, v in (body.get("logit_bias") or {}).items()} or None,
                          allowed_token_ids=body.get("allowed_token_ids"), bad_words=body.get("bad_words"))


class _ChatParseStream:
    """Incremental DS4 chat parsing for streamed chat completions: text before ``</think>``
    goes out as ``reasoning_content`` deltas (thinking mode), then ``content`` deltas; a
    tail that could still be the start of a marker is held back; from the DSML tool-call
    block on, text is buffered and parsed at the end into one ``tool_calls`` delta."""

    def __init__(self, thinking: bool, tools: bool):
        self.mode = "reasoning_content" if thinking else "content"
        self.thinking, self.tools = thinking, tools
        self.buf, self.full, self.tool_buf = "", "", ""
        self.tool_calls = None
        self.call_start = f"\n\n<{chat_encoding.DSML}{chat_encoding.CALLS_BLOCK}>"

    def _marker(self):
        if self.mode == "reasoning_content":
            return chat_encoding.THINK_END
        return self.call_start if self.tools and self.mode == "content" else None

    def push(self, text: str, finished: bool) -> Dict[str, Any]:
        self.full += text
        delta: Dict[str, Any] = {}

        def emit(key, piece):
            if piece:
                delta[key] = delta.get(key, "") + piece
        if self.mode == "tools":
            self.tool_buf += text
        else:
            self.buf += text
        while self.mode != "tools":
            m = self._marker()
            if m is not None and m in self.buf:
                before, after = self.buf.split(m, 1)
                emit(self.mode, before)
                if self.mode == "reasoning_content":
                    self.mode, self.buf = "content", after
                else:
                    self.mode, self.tool_buf, self.buf = "tools", m + after, ""
                continue
            hold = 0 if finished or m is None else len(m) - 1
            cut = max(0, len(self.buf) - hold)
            emit(self.mode, self.buf[:cut].replace(chat_encoding.EOS, "") if finished else self.buf[:cut])
            self.buf = self.buf[cut:]
            break
        if finished and self.mode == "tools":
            try:
                msg = chat_encoding.parse_completion(self.full, thinking=self.thinking)
                self.tool_calls = msg.get("tool_calls") or []
                delta["tool_calls"] = [dict(c, index=i) for i, c in enumerate(self.tool_calls)]
            except ValueError:
                emit("content", self.tool_buf)          # not a valid tool-call block: plain text
        return delta


class _StopStream:
    """Incremental text for streaming with stop strings: a tail that could still be the
    start of a stop string is held back until it is resolved (as vLLM streams)."""

    def __init__(self, tok, params: SamplingParams):
        self.tok, self.p = tok, params
        self.ids, self.sent = [], 0
        self.hold = max((len(x) for x in params.stop), default=1) - 1
        self.done = False

    def push(self, new_ids, finished: bool) -> str:
        if self.done:
            return ""
        self.ids += list(new_ids)
        text = self.tok.decode(self.ids)
        cut, hit = cut_at_stop(text, self.p.stop, self.p.include_stop_str_in_output)
        if hit is not None or finished:
            self.done = True
            out, self.sent = cut[self.sent:], len(cut)
            return out
        upto = max(self.sent, len(text) - self.hold)
        out, self.sent = text[self.sent:upto], upto
        return out


def build_app(worker: EngineWorker, reasoning_parser: Optional[str] = "deepseek_v4",
              tool_call_parser: Optional[str] = "deepseek_v4"):
    """The HTTP app.  Parsers (the reference's --reasoning-parser / --tool-call-parser):
    "deepseek_v4" splits chat output into reasoning_content / content / tool_calls with the
    DS4 encoding; None returns the raw completion text as content."""
    from fastapi import FastAPI, HTTPException
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="vllm_moet_b200 OpenAI-compatible server")
    tok = worker.llm.tokenizer
    name = worker.model_name

    from prometheus_client import CollectorRegistry, Histogram, generate_latest
    registry = CollectorRegistry()
    buckets = (0.005, 0.01, 0.02, 0.05, 0.1, 0.2, 0.5, 1, 2, 5, 10, 30, 60)
    h_ttft = Histogram("moet_time_to_first_token_seconds", "time to first token", registry=registry,
                       buckets=buckets)
    h_tpot = Histogram("moet_time_per_output_token_seconds", "time per output token after the first",
                       registry=registry, buckets=(0.001, 0.002, 0.005, 0.01, 0.02, 0.05, 0.1, 0.2, 0.5, 1))
    h_e2e = Histogram("moet_e2e_request_latency_seconds", "end-to-end request latency", registry=registry,
                      buckets=buckets)
    h_acc = Histogram("moet_request_tokens_per_step", "tokens emitted per decode step of a request "
                      "(1 + accepted draft tokens on average)", registry=registry,
                      buckets=(1.0, 1.25, 1.5, 1.75, 2.0, 2.5, 3.0, 4.0, 5.0, 8.0))

    def run_request(prompt_ids, params):
        """-> (asyncio.Queue of (ids, finish, logprobs)) fed from the engine thread."""
        loop = asyncio.get_running_loop()
        aq: "asyncio.Queue" = asyncio.Queue()
        t0, seen = time.perf_counter(), {"first": None, "n": 0}

        def cb(ids, finish, lp=None):
            now = time.perf_counter()
            if ids and seen["first"] is None:
                seen["first"] = now
                h_ttft.observe(now - t0)
            seen["n"] += len(ids)
            seen["calls"] = seen.get("calls", 0) + (1 if ids else 0)
            if finish is not None and not finish.startswith("error:"):
                h_e2e.observe(now - t0)
                if seen["calls"] > 1:        # one call per engine step after the first token
                    h_acc.observe((seen["n"] - 1) / (seen["calls"] - 1))
                if seen["first"] is not None and seen["n"] > 1:
                    h_tpot.observe((now - seen["first"]) / (seen["n"] - 1))
            loop.call_soon_threadsafe(aq.put_nowait, (list(ids), finish, lp))
        aq.rid = worker.submit(prompt_ids, params, cb)
        return aq

    async def guard(agen, aq):
        """Stream `agen`; a client that goes away before the end aborts its request."""
        done = False
        try:
            async for chunk in agen:
                yield chunk
            done = True
        finally:
            if not done:
                worker.abort(aq.rid)

    async def collect(aq):
        ids, finish, lps = [], None, []
        while finish is None:
            new, finish, lp = await aq.get()
            ids += new
            lps += lp or []
        if finish.startswith("error:"):
            raise HTTPException(500, finish[6:])
        return ids, finish, lps

    def completion_logprobs(ids, lps):
        """OpenAI completions format: tokens, token_logprobs, top_logprobs, text_offset."""
        toks = [tok.decode([t]) for t in ids]
        offs, o = [], 0
        for t in toks:
            offs.append(o)
            o += len(t)
        return {"tokens": toks, "token_logprobs": [d.get(t) for d, t in zip(lps, ids)],
                "top_logprobs": [{tok.decode([k]): v for k, v in d.items()} for d in lps], "text_offset": offs}

    def chat_logprobs(ids, lps, top_n):
        """OpenAI chat format: content[] of {token, logprob, bytes, top_logprobs[]}."""
        out = []
        for t, d in zip(ids, lps):
            s = tok.decode([t])
            alts = sorted(d.items(), key=lambda kv: -kv[1])[:top_n]
            out.append({"token": s, "logprob": d.get(t), "bytes": list(s.encode("utf-8")),
                        "top_logprobs": [{"token": tok.decode([k]), "logprob": v,
                                          "bytes": list(tok.decode([k]).encode("utf-8"))} for k, v in alts]})
        return {"content": out}

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": name, "object": "model", "owned_by": "vllm_moet_b200",
                                            "max_model_len": worker.llm.ecfg.max_model_len}]}

    @app.post("/tokenize")
    async def tokenize(body: Dict[str, Any]):
        if "messages" in body:
            text = chat_encoding.render(body["messages"], tools=body.get("tools"),
                                        reasoning_effort=body.get("reasoning_effort", "none"))
            ids = [tok.bos_token_id] + tok.encode(text)
        else:
            ids = _prompt_ids(body.get("prompt", "")) if body.get("add_special_tokens", True) \
                else tok.encode(body.get("prompt", ""))
        return {"tokens": ids, "count": len(ids), "max_model_len": worker.llm.ecfg.max_model_len}

    @app.post("/detokenize")
    async def detokenize(body: Dict[str, Any]):
        return {"prompt": tok.decode(list(body.get("tokens", [])))}

    @app.get("/version")
    async def version():
        from .. import __version__
        return {"version": __version__}

    @app.get("/metrics")
    async def metrics():
        lines = [f"moet_{k}_total {v}" for k, v in worker.stats.items()]
        return PlainTextResponse("\n".join(lines) + "\n" + generate_latest(registry).decode())

    def copies(params):
        """n completions -> n engine requests (copy j samples with seed + j when seeded)."""
        import dataclasses
        return [dataclasses.replace(params, n=1, seed=None if params.seed is None else params.seed + j)
                for j in range(params.n)]

    def _servable(params):
        """Refuse what the engine would refuse (e.g. penalties with SP prefill) with a 400."""
        check = getattr(worker.llm, "_check_request", None)
        if check is None:
            return
        try:
            check([0], params)
        except (NotImplementedError, ValueError) as e:
            raise HTTPException(400, str(e))

    def _usage_chunk(rid, created, obj, n_prompt, n_out):
        return {"id": rid, "object": obj, "created": created, "model": name, "choices": [],
                "usage": {"prompt_tokens": n_prompt, "completion_tokens": n_out, "total_tokens": n_prompt + n_out}}

    def _prompt_text(p, ids):
        return p if isinstance(p, str) else tok.decode([t for t in ids if t != tok.bos_token_id])

    def _prompt_ids(p):
        if isinstance(p, str):
            return [tok.bos_token_id] + tok.encode(p)
        if isinstance(p, list) and all(isinstance(t, int) for t in p):
            return list(p)
        raise HTTPException(400, "prompt must be a string or a list of token ids")

    async def run_beams(plist, bp):
        """The beam search over the engine queue: each step's beams are one-token requests."""
        from ..engine.beam_search import search_steps, step_params
        gen = search_steps(plist, bp, tok.eos_token_id, tok.decode)
        sp = step_params(bp)
        try:
            batch = next(gen)
            while True:
                res = await asyncio.gather(*[collect(run_request(b, sp)) for b in batch])
                batch = gen.send([r[2][0] for r in res])
        except StopIteration as stop:
            return stop.value

    def beam_params(body, params):
        from ..engine.beam_search import BeamSearchParams
        if body.get("stream"):
            raise HTTPException(400, "beam search does not stream")
        try:
            return BeamSearchParams(beam_width=int(body.get("best_of") or params.n), max_tokens=params.max_tokens,
                                    ignore_eos=params.ignore_eos,
                                    length_penalty=float(body.get("length_penalty", 1.0)))
        except ValueError as e:
            raise HTTPException(400, str(e))

    async def beam_completion(body, params, plist, rid, created):
        """``use_beam_search``: beam width = ``n`` (or ``best_of``), the search driven through
        the engine queue -- each step's beams are one-token requests served concurrently."""
        bp = beam_params(body, params)
        outs = await run_beams(plist, bp)
        choices, n_out = [], 0
        for j, o in enumerate(outs):
            for s_ in o.sequences[:params.n]:
                n_out += len(s_.generated)
                choices.append({"index": len(choices), "text": s_.text, "token_ids": s_.generated,
                                "finish_reason": s_.finish_reason, "cumulative_logprob": s_.cum_logprob,
                                "logprobs": None})
        return JSONResponse({"id": rid, "object": "text_completion", "created": created, "model": name,
                             "choices": choices,
                             "usage": {"prompt_tokens": sum(map(len, plist)), "completion_tokens": n_out,
                                       "total_tokens": sum(map(len, plist)) + n_out}})

    @app.post("/v1/completions")
    async def completions(body: Dict[str, Any]):
        try:
            params = _params_from(body)
        except ValueError as e:
            raise HTTPException(400, str(e))
        _servable(params)
        prompts = body.get("prompt")
        echo = bool(body.get("echo", False))
        if isinstance(prompts, list) and prompts and not isinstance(prompts[0], int):
            plist = [_prompt_ids(p) for p in prompts]
            raw = list(prompts)
        else:
            plist = [_prompt_ids(prompts)]
            raw = [prompts]
        rid, created = f"cmpl-{uuid.uuid4().hex[:24]}", int(time.time())
        if body.get("use_beam_search"):
            return await beam_completion(body, params, plist, rid, created)
        if body.get("stream"):
            if len(plist) != 1 or params.n != 1:
                raise HTTPException(400, "streaming serves one prompt and one completion per request")
            aq = run_request(plist[0], params)
            usage = bool((body.get("stream_options") or {}).get("include_usage"))

            async def gen():
                finish, n_out = None, 0
                ss = _StopStream(tok, params)
                if echo:
                    first = {"id": rid, "object": "text_completion", "created": created, "model": name,
                             "choices": [{"index": 0, "text": _prompt_text(prompts if isinstance(prompts, (str, list))
                                                                           else "", plist[0]),
                                          "token_ids": [], "logprobs": None, "finish_reason": None}]}
                    yield f"data: {json.dumps(first)}\n\n"
                while finish is None:
                    ids, finish, lp = await aq.get()
                    if finish and finish.startswith("error:"):
                        yield f"data: {json.dumps({'error': finish[6:]})}\n\n"
                        break
                    n_out += len(ids)
                    text = ss.push(ids, finish is not None) if params.stop else tok.decode(ids)
                    chunk = {"id": rid, "object": "text_completion", "created": created, "model": name,
                             "choices": [{"index": 0, "text": text, "token_ids": ids,
                                          "logprobs": completion_logprobs(ids, lp) if lp else None,
                                          "finish_reason": finish}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                if usage:
                    yield f"data: {json.dumps(_usage_chunk(rid, created, 'text_completion', len(plist[0]), n_out))}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(guard(gen(), aq), media_type="text/event-stream")
        qs = [run_request(p, c) for p in plist for c in copies(params)]
        choices, n_out = [], 0
        for i, aq in enumerate(qs):
            ids, finish, lps = await collect(aq)
            n_out += len(ids)
            text, hit = cut_at_stop(tok.decode(ids), params.stop, params.include_stop_str_in_output)
            if echo:                                       # the prompt text before the completion
                j = i // params.n
                text = _prompt_text(raw[j], plist[j]) + text
            choices.append({"index": i, "text": text, "token_ids": ids, "finish_reason": finish,
                            "stop_reason": hit,
                            "logprobs": completion_logprobs(ids, lps) if params.logprobs is not None else None})
        return JSONResponse({"id": rid, "object": "text_completion", "created": created, "model": name,
                             "choices": choices,
                             "usage": {"prompt_tokens": sum(map(len, plist)), "completion_tokens": n_out,
                                       "total_tokens": sum(map(len, plist)) + n_out}})

    @app.post("/v1/chat/completions")
    async def chat(body: Dict[str, Any]):
        try:
            params = _params_from(body)
        except ValueError as e:
            raise HTTPException(400, str(e))
        _servable(params)
        effort = body.get("reasoning_effort", "none")
        text = chat_encoding.render(body.get("messages", []), tools=body.get("tools"), reasoning_effort=effort)
        prompt = [tok.bos_token_id] + tok.encode(text)
        rid, created = f"chatcmpl-{uuid.uuid4().hex[:24]}", int(time.time())
        thinking = chat_encoding.normalize_effort(effort) is not None
        if body.get("use_beam_search"):       # beam search: n best beams as n choices
            outs = await run_beams([prompt], beam_params(body, params))
            seqs = outs[0].sequences[:params.n]
            n_out = sum(len(q.generated) for q in seqs)
            return JSONResponse({"id": rid, "object": "chat.completion", "created": created, "model": name,
                                 "choices": [{"index": i, "message": {"role": "assistant", "content": q.text},
                                              "finish_reason": q.finish_reason,
                                              "cumulative_logprob": q.cum_logprob} for i, q in enumerate(seqs)],
                                 "usage": {"prompt_tokens": len(prompt), "completion_tokens": n_out,
                                           "total_tokens": len(prompt) + n_out}})
        if body.get("stream") and params.n != 1:
            raise HTTPException(400, "streaming serves one completion per request")
        qs = [run_request(prompt, c) for c in copies(params)]
        aq = qs[0]
        if body.get("stream"):
            usage = bool((body.get("stream_options") or {}).get("include_usage"))

            async def gen():
                finish, n_out = None, 0
                first = True
                ss = _StopStream(tok, params)
                cps = _ChatParseStream(thinking and bool(reasoning_parser), bool(tool_call_parser)) \
                    if (reasoning_parser or tool_call_parser) else None
                while finish is None:
                    ids, finish, _ = await aq.get()
                    n_out += len(ids)
                    text = ss.push(ids, finish is not None) if params.stop else tok.decode(ids)
                    delta = cps.push(text, finish is not None) if cps is not None else {"content": text}
                    if first:
                        delta["role"] = "assistant"
                        first = False
                    fr = "tool_calls" if finish and cps is not None and cps.tool_calls else finish
                    chunk = {"id": rid, "object": "chat.completion.chunk", "created": created, "model": name,
                             "choices": [{"index": 0, "delta": delta, "finish_reason": fr}]}
                    yield f"data: {json.dumps(chunk)}\n\n"
                if usage:
                    yield f"data: {json.dumps(_usage_chunk(rid, created, 'chat.completion.chunk', len(prompt), n_out))}\n\n"
                yield "data: [DONE]\n\n"
            return StreamingResponse(guard(gen(), aq), media_type="text/event-stream")
        choices, n_out = [], 0
        for j, q in enumerate(qs):
            ids, finish, lps = await collect(q)
            n_out += len(ids)
            out_text = cut_at_stop(tok.decode(ids), params.stop, params.include_stop_str_in_output)[0]
            msg = {"role": "assistant", "content": out_text}
            if reasoning_parser or tool_call_parser:
                try:
                    msg = chat_encoding.parse_completion(out_text, thinking=thinking and bool(reasoning_parser))
                    if not tool_call_parser and msg.get("tool_calls"):
                        msg = {"role": "assistant", "content": out_text}
                except ValueError:
                    pass        # a free-form completion (random-init models): returned as content
            choices.append({"index": j, "message": msg, "finish_reason": finish,
                            "logprobs": chat_logprobs(ids, lps, params.logprobs)
                            if params.logprobs is not None else None})
        return JSONResponse({"id": rid, "object": "chat.completion", "created": created, "model": name,
                             "choices": choices,
                             "usage": {"prompt_tokens": len(prompt), "completion_tokens": n_out,
                                       "total_tokens": len(prompt) + n_out}})

    return app


_PARSERS = ("deepseek_v4", "none")


def build_parser():
    ap = argparse.ArgumentParser(description="OpenAI-compatible server over the engine")
    ap.add_argument("--model", default="ds4-flash-shape", help="a preset name or a local checkpoint directory")
    ap.add_argument("--served-model-name", default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--num-layers", type=int, default=None)
    ap.add_argument("--max-model-len", type=int, default=8192)
    ap.add_argument("--max-num-seqs", type=int, default=32)
    ap.add_argument("--num-speculative-tokens", type=int, default=2)
    ap.add_argument("--speculative-config", default=None,
                    help='JSON, e.g. {"method": "mtp", "num_speculative_tokens": 2}')
    ap.add_argument("--kv-cache-dtype", default="auto", choices=("auto", "bf16", "bfloat16", "nvfp4"))
    ap.add_argument("--device", default=None)
    ap.add_argument("--data-parallel-size", type=int, default=1,
                    help="replicated engines behind a request router (see dp_serve)")
    ap.add_argument("--tensor-parallel-size", type=int, default=None,
                    help="GPUs per replica with --data-parallel-size; otherwise torchrun's WORLD_SIZE")
    ap.add_argument("--pipeline-parallel-size", type=int, default=1)
    ap.add_argument("--decode-context-parallel-size", type=int, default=1)
    ap.add_argument("--enable-expert-parallel", action="store_true")
    ap.add_argument("--enable-prefix-caching", action="store_true",
                    help="reuse the K/V of shared block-aligned prompt prefixes")
    ap.add_argument("--block-size", type=int, default=16, help="prefix-cache block of the CPU engine, in tokens (GPU: 64-token KV blocks)")
    ap.add_argument("--enable-chunked-prefill", action="store_true",
                    help="prefill long prompts a token budget per step beside the decoding rows")
    ap.add_argument("--max-num-batched-tokens", type=int, default=None, help="per-step token budget (chunked prefill)")
    ap.add_argument("--gpus", default=None, help="GPU ids for the replicas of --data-parallel-size ('cpu': none)")
    ap.add_argument("--reasoning-parser", default="deepseek_v4", choices=_PARSERS)
    ap.add_argument("--tool-call-parser", default="deepseek_v4", choices=_PARSERS)
    ap.add_argument("--enable-auto-tool-choice", action="store_true", help="accepted (tools are always parsed)")
    ap.add_argument("--gpu-memory-utilization", type=float, default=None, help="accepted; KV blocks are sized "
                    "from the free memory after the weights")
    ap.add_argument("--trust-remote-code", action="store_true", help="accepted; no remote code is run")
    ap.add_argument("--dtype", default="auto", help="accepted; activations are bf16")
    ap.add_argument("--trellis-pack", default=None,
                    help="serve the routed experts from these trellis (EXL3-style) packs (one rank)")
    return ap


def llm_kwargs(args, world: int = 1, rank: int = 0, group=None) -> dict:
    """Server flags -> LLM keyword arguments (refusing what the GPU server path does not serve)."""
    k = args.num_speculative_tokens
    method = "mtp"
    if args.speculative_config:
        spec = json.loads(args.speculative_config)
        method = spec.get("method", "mtp")
        if method in ("mtp", "deepseek_mtp", "deepseek_v4_mtp"):
            method = "mtp"
        elif method not in ("eagle3", "dspark", "dflash"):       # these three: CPU engine
            raise SystemExit(f"speculative method {method!r}: mtp | eagle3 | dspark | dflash")
        k = int(spec.get("num_speculative_tokens", k))
    if args.pipeline_parallel_size != 1:
        raise SystemExit("--pipeline-parallel-size: the server runs TP ranks; use the LLM API for pipeline stages")
    if args.decode_context_parallel_size != 1:
        raise SystemExit("--decode-context-parallel-size: the server runs TP ranks; use the LLM API with dcp_group")
    kv = "nvfp4" if args.kv_cache_dtype == "nvfp4" else "bf16"
    return dict(device=args.device, num_speculative_tokens=0 if method in ("dspark", "dflash") else k,
                max_model_len=args.max_model_len,
                max_num_seqs=args.max_num_seqs, num_layers=args.num_layers, kv_cache_dtype=kv,
                tensor_parallel_size=world, tp_group=group, tp_rank=rank,
                expert_parallel=bool(args.enable_expert_parallel), speculative_method=method,
                **({"dspark": {"block": k}} if method in ("dspark", "dflash") else {}),
                enable_prefix_caching=bool(getattr(args, "enable_prefix_caching", False)),
                prefix_block_size=int(getattr(args, "block_size", 16)),
                enable_chunked_prefill=bool(getattr(args, "enable_chunked_prefill", False)),
                max_num_batched_tokens=getattr(args, "max_num_batched_tokens", None),
                **({"trellis_pack": args.trellis_pack} if getattr(args, "trellis_pack", None) else {}))


def main(argv=None):
    args = build_parser().parse_args(argv)
    if args.data_parallel_size > 1:
        import sys
        from .dp_serve import main as dp_main
        dp_main(list(sys.argv[1:] if argv is None else argv))
        return
    import torch
    from ..engine.llm import LLM
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.tensor_parallel_size not in (None, world):
        raise SystemExit(f"--tensor-parallel-size {args.tensor_parallel_size} without --data-parallel-size: "
                         f"launch with torchrun --nproc-per-node {args.tensor_parallel_size}")
    kw = llm_kwargs(args, world, rank)
    group = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl")
        group = dist.group.WORLD
        kw["tp_group"] = group
    llm = LLM(args.model, **kw)
    if rank != 0:
        follower_loop(llm, group)
        return
    import uvicorn
    name = args.served_model_name or args.model
    worker = EngineWorker(llm, name, group, max_batch=args.max_num_seqs)
    parse = lambda v: None if v == "none" else v      # noqa: E731
    uvicorn.run(build_app(worker, parse(args.reasoning_parser), parse(args.tool_call_parser)), host=args.host,
                port=args.port, log_level="warning")


if __name__ == "__main__":
    main()
