"""OpenAI-compatible server (tiny CPU model) and the DeepSeek-V4 chat encoding."""
import json
import socket
import threading
import time

import pytest
import requests

from vllm_moet_b200.entrypoints import chat_encoding as ce


def test_effort_normalisation():
    assert ce.normalize_effort("none") is None
    assert ce.normalize_effort(None) == "low"
    assert ce.normalize_effort("xhigh") == "max" and ce.normalize_effort("max") == "max"
    assert ce.normalize_effort("medium") == "high" and ce.normalize_effort("low") == "low"


def test_render_and_parse_roundtrip():
    tools = [{"type": "function", "function": {"name": "get_weather", "description": "d",
                                               "parameters": {"type": "object"}}}]
    msgs = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "weather?"},
            {"role": "assistant", "content": "", "reasoning_content": "need a tool",
             "tool_calls": [{"type": "function", "function": {"name": "get_weather",
                                                               "arguments": '{"city": "Oslo", "days": 3}'}}]},
            {"role": "tool", "content": "sunny"}]
    text = ce.render(msgs, tools=tools, reasoning_effort="high")
    assert text.startswith(ce.BOS + ce.EFFORT_PROMPTS["high"])
    assert "<tool_result>sunny</tool_result>" in text and "## Tools" in text
    assert f'<{ce.DSML}parameter name="city" string="true">Oslo</{ce.DSML}parameter>' in text
    assert f'<{ce.DSML}parameter name="days" string="false">3</{ce.DSML}parameter>' in text
    assert "need a tool" in text and text.endswith(ce.ASSISTANT + ce.THINK_START)
    # earlier-turn reasoning is dropped once a later user turn exists
    t2 = ce.render(msgs + [{"role": "user", "content": "thanks"}], reasoning_effort="low")
    assert "need a tool" not in t2
    assert ce.render([{"role": "user", "content": "x"}], reasoning_effort="none").endswith(ce.ASSISTANT + ce.THINK_END)
    comp = "let me check" + ce.THINK_END + "Sure." + ce.encode_tool_calls(
        [{"function": {"name": "f", "arguments": {"a": 1, "b": "x"}}}]) + ce.EOS
    msg = ce.parse_completion(comp, thinking=True)
    assert msg["reasoning_content"] == "let me check" and msg["content"] == "Sure."
    assert json.loads(msg["tool_calls"][0]["function"]["arguments"]) == {"a": 1, "b": "x"}
    with pytest.raises(ValueError):
        ce.parse_completion("no end of thinking", thinking=True)
    with pytest.raises(ValueError):
        ce.parse_completion("a" + ce.THINK_END + "b" + ce.BOS, thinking=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def server():
    import uvicorn
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.entrypoints.openai_server import EngineWorker, build_app
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    worker = EngineWorker(llm, "tiny-moe")
    port = _free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(worker), host="127.0.0.1", port=port, log_level="warning"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    url = f"http://127.0.0.1:{port}"
    for _ in range(100):
        try:
            if requests.get(url + "/health", timeout=1).ok:
                break
        except requests.ConnectionError:
            time.sleep(0.1)
    yield url, llm
    srv.should_exit = True
    th.join(timeout=10)
    worker.close()


def test_completions_match_engine(server):
    url, llm = server
    r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 6, "ignore_eos": True},
                      timeout=120)
    assert r.ok, r.text
    body = r.json()
    from vllm_moet_b200.models import reference
    assert body["choices"][0]["token_ids"] == reference.greedy_generate(llm.mw, [5, 6, 7, 8], 6)
    assert body["usage"]["completion_tokens"] == 6
    assert requests.get(url + "/v1/models").json()["data"][0]["id"] == "tiny-moe"
    m = requests.get(url + "/metrics").text
    assert "moet_requests_total" in m
    assert "moet_time_to_first_token_seconds_count" in m and "moet_e2e_request_latency_seconds_bucket" in m
    count = [ln for ln in m.splitlines() if ln.startswith("moet_e2e_request_latency_seconds_count")][0]
    assert float(count.split()[-1]) >= 1
    assert "moet_decode_steps_total" in m and "moet_accepted_draft_tokens_total" in m
    acc = [ln for ln in m.splitlines() if ln.startswith("moet_request_tokens_per_step_count")][0]
    assert float(acc.split()[-1]) >= 1


def test_streaming_and_chat(server):
    url, _ = server
    r = requests.post(url + "/v1/completions", json={"prompt": "hi", "max_tokens": 5, "stream": True,
                                                     "ignore_eos": True}, stream=True, timeout=120)
    events = [ln[6:] for ln in r.iter_lines(decode_unicode=True) if ln.startswith("data: ")]
    assert events[-1] == "[DONE]"
    ids = sum((json.loads(e)["choices"][0]["token_ids"] for e in events[:-1]), [])
    assert len(ids) == 5 and json.loads(events[-2])["choices"][0]["finish_reason"] == "length"
    r = requests.post(url + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hello"}],
                                                          "max_tokens": 4, "ignore_eos": True}, timeout=120)
    assert r.ok and r.json()["choices"][0]["message"]["role"] == "assistant"
    assert requests.post(url + "/v1/completions", json={"prompt": "x", "temperature": -1}).status_code == 400
    body = {"prompt": [5, 6, 7, 8], "max_tokens": 6, "ignore_eos": True, "temperature": 0.8, "seed": 3}
    a = requests.post(url + "/v1/completions", json=body, timeout=120).json()["choices"][0]["token_ids"]
    b = requests.post(url + "/v1/completions", json=body, timeout=120).json()["choices"][0]["token_ids"]
    assert a == b and len(a) == 6                     # seeded sampling is reproducible


def _tp_serving(rank, world):
    """Rank 0 serves (EngineWorker batches broadcast to followers); rank 1 follows."""
    import torch.distributed as dist
    from vllm_moet_b200 import SamplingParams
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.entrypoints.openai_server import EngineWorker, follower_loop
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=128,
              tensor_parallel_size=world, tp_group=dist.group.WORLD, tp_rank=rank)
    if rank != 0:
        follower_loop(llm, dist.group.WORLD)
        return None
    import threading
    done = threading.Event()
    got = {}

    def cb(ids, finish):
        got.setdefault("ids", []).extend(ids)
        if finish:
            done.set()
    w = EngineWorker(llm, "tiny-moe", tp_group=dist.group.WORLD)
    w.submit([5, 6, 7, 8], SamplingParams(max_tokens=6, ignore_eos=True), cb)
    done.wait(120)
    w.close()
    return got["ids"]


def test_tp2_serving_followers_match_single_rank():
    from mp_util import run_ranks
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200 import SamplingParams
    ids = run_ranks(_tp_serving, 2)[0]
    one = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=128)
    want = one.generate([[5, 6, 7, 8]], SamplingParams(max_tokens=6, ignore_eos=True))[0].outputs[0].token_ids
    assert ids == want


def test_stop_strings_over_http(server):
    url, _ = server
    g = __import__("torch").Generator().manual_seed(5)
    p = __import__("torch").randint(3, 259, (12,), generator=g).tolist()
    body = {"prompt": p, "max_tokens": 16, "ignore_eos": True}
    full = requests.post(url + "/v1/completions", json=body, timeout=120).json()["choices"][0]["text"]
    stop = full[-2:]
    want = full[: full.find(stop)]
    r = requests.post(url + "/v1/completions", json=dict(body, stop=stop), timeout=120).json()["choices"][0]
    assert r["text"] == want and r["finish_reason"] == "stop" and r["stop_reason"] == stop
    s = requests.post(url + "/v1/completions", json=dict(body, stop=[stop], stream=True), stream=True, timeout=120)
    events = [ln[6:] for ln in s.iter_lines(decode_unicode=True) if ln.startswith("data: ")]
    assert "".join(json.loads(e)["choices"][0]["text"] for e in events[:-1]) == want


def test_logprobs_over_http(server):
    url, _ = server
    r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 4, "ignore_eos": True,
                                                     "logprobs": 2}, timeout=120).json()["choices"][0]
    lp = r["logprobs"]
    assert len(lp["token_logprobs"]) == 4 and all(x <= 0 for x in lp["token_logprobs"])
    assert len(lp["top_logprobs"]) == 4 and lp["text_offset"][0] == 0
    c = requests.post(url + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                          "max_tokens": 3, "ignore_eos": True, "logprobs": True,
                                                          "top_logprobs": 2}, timeout=120).json()["choices"][0]
    content = c["logprobs"]["content"]
    assert len(content) == 3 and all(len(e["top_logprobs"]) == 2 and e["logprob"] <= 0 for e in content)
    plain = requests.post(url + "/v1/completions", json={"prompt": [5, 6], "max_tokens": 2}, timeout=120).json()
    assert plain["choices"][0]["logprobs"] is None


def test_cli_flags_map_to_engine_arguments():
    from vllm_moet_b200.entrypoints.openai_server import build_parser, llm_kwargs
    a = build_parser().parse_args(["--model", "tiny-moe", "--speculative-config",
                                   '{"method": "deepseek_mtp", "num_speculative_tokens": 3}',
                                   "--kv-cache-dtype", "nvfp4", "--enable-expert-parallel", "--reasoning-parser",
                                   "none", "--served-model-name", "moet", "--gpu-memory-utilization", "0.9"])
    kw = llm_kwargs(a)
    assert kw["num_speculative_tokens"] == 3 and kw["kv_cache_dtype"] == "nvfp4" and kw["expert_parallel"]
    assert a.reasoning_parser == "none" and a.served_model_name == "moet"
    kw = llm_kwargs(build_parser().parse_args(["--enable-prefix-caching", "--block-size", "32",
                                               "--enable-chunked-prefill", "--max-num-batched-tokens", "512"]))
    assert kw["enable_prefix_caching"] and kw["prefix_block_size"] == 32
    assert kw["enable_chunked_prefill"] and kw["max_num_batched_tokens"] == 512
    assert "trellis_pack" not in kw
    assert llm_kwargs(build_parser().parse_args(["--trellis-pack", "/packs"]))["trellis_pack"] == "/packs"
    from vllm_moet_b200.entrypoints.openai_server import _params_from
    sp = _params_from({"presence_penalty": 0.5, "frequency_penalty": 0.25, "repetition_penalty": 1.1,
                       "min_p": 0.05, "logit_bias": {"42": -100}})
    assert (sp.presence_penalty, sp.frequency_penalty, sp.repetition_penalty, sp.min_p) == (0.5, 0.25, 1.1, 0.05)
    assert sp.logit_bias == {42: -100.0} and sp.processes_logits
    kw = llm_kwargs(build_parser().parse_args(["--speculative-config",
                                               '{"method": "eagle3", "num_speculative_tokens": 3}']))
    assert kw["speculative_method"] == "eagle3" and kw["num_speculative_tokens"] == 3
    kw = llm_kwargs(build_parser().parse_args(["--speculative-config", '{"method": "dspark", "num_speculative_tokens": 4}']))
    assert kw["speculative_method"] == "dspark" and kw["dspark"] == {"block": 4}
    for bad in (["--speculative-config", '{"method": "ngram"}'], ["--pipeline-parallel-size", "2"],
                ["--decode-context-parallel-size", "2"]):
        with pytest.raises(SystemExit):
            llm_kwargs(build_parser().parse_args(bad))


def test_raw_content_without_parsers():
    """--reasoning-parser none / --tool-call-parser none: chat content is the raw completion."""
    import uvicorn
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.entrypoints.openai_server import EngineWorker, build_app
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=2, max_model_len=256)
    w = EngineWorker(llm, "raw")
    port = _free_port()
    srv = uvicorn.Server(uvicorn.Config(build_app(w, None, None), host="127.0.0.1", port=port, log_level="warning"))
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
        r = requests.post(url + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                              "max_tokens": 4, "ignore_eos": True}, timeout=120)
        msg = r.json()["choices"][0]["message"]
        assert msg["role"] == "assistant" and "reasoning_content" not in msg and "tool_calls" not in msg
        assert r.json()["model"] == "raw"
    finally:
        srv.should_exit = True
        th.join(timeout=10)
        w.close()


def test_requests_join_running_batch_and_disconnect_aborts(server):
    url, _ = server
    order = []

    def run(name, n):
        r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": n, "ignore_eos": True},
                          timeout=120)
        assert r.ok
        order.append(name)
    long = threading.Thread(target=run, args=("long", 120))
    long.start()
    time.sleep(0.3)
    run("short", 2)                  # joins the running batch instead of waiting for it
    long.join()
    assert order == ["short", "long"]
    # a streaming client that goes away aborts its request
    s = requests.post(url + "/v1/completions", json={"prompt": [5, 6], "max_tokens": 200, "ignore_eos": True,
                                                     "stream": True}, stream=True, timeout=120)
    it = s.iter_lines()
    next(it)
    s.close()
    m = ""
    for _ in range(100):
        m = requests.get(url + "/metrics").text
        if "moet_aborted_total 1" in m:
            break
        time.sleep(0.1)
    assert "moet_aborted_total 1" in m


def test_n_choices_over_http(server):
    url, _ = server
    body = {"prompt": [5, 6, 7], "max_tokens": 4, "ignore_eos": True, "temperature": 1.3, "seed": 2, "n": 3}
    ch = requests.post(url + "/v1/completions", json=body, timeout=120).json()["choices"]
    assert [c["index"] for c in ch] == [0, 1, 2] and len({tuple(c["token_ids"]) for c in ch}) > 1
    chat = requests.post(url + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                             "max_tokens": 3, "ignore_eos": True, "n": 2},
                         timeout=120).json()
    assert len(chat["choices"]) == 2 and chat["usage"]["completion_tokens"] == 6
    assert requests.post(url + "/v1/completions", json=dict(body, stream=True), timeout=120).status_code == 400


def test_tokenize_detokenize_version(server):
    url, _ = server
    t = requests.post(url + "/tokenize", json={"prompt": "hi"}).json()
    assert t["tokens"][0] == 1 and t["count"] == 3
    assert requests.post(url + "/detokenize", json={"tokens": t["tokens"][1:]}).json()["prompt"] == "hi"
    c = requests.post(url + "/tokenize", json={"messages": [{"role": "user", "content": "hi"}]}).json()
    assert c["count"] > 3
    assert requests.get(url + "/version").json()["version"]


def test_chat_stream_parser_splits_reasoning_content_and_tool_calls():
    from vllm_moet_b200.entrypoints import chat_encoding as ce
    from vllm_moet_b200.entrypoints.openai_server import _ChatParseStream
    text = "let me think" + ce.THINK_END + "Sure." + ce.encode_tool_calls(
        [{"function": {"name": "get_weather", "arguments": {"city": "Oslo"}}}]) + ce.EOS
    for step in (1, 3, 7, len(text)):            # any chunking gives the same deltas
        ps = _ChatParseStream(thinking=True, tools=True)
        pieces = [text[i:i + step] for i in range(0, len(text), step)]
        out = [ps.push(p, i == len(pieces) - 1) for i, p in enumerate(pieces)]
        assert "".join(d.get("reasoning_content", "") for d in out) == "let me think"
        assert "".join(d.get("content", "") for d in out) == "Sure."
        calls = [c for d in out for c in d.get("tool_calls", [])]
        assert len(calls) == 1 and calls[0]["function"]["name"] == "get_weather" and calls[0]["index"] == 0
        assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Oslo"}
    plain = _ChatParseStream(thinking=False, tools=True)
    d = [plain.push("no tools here", False), plain.push("", True)]
    assert "".join(x.get("content", "") for x in d) == "no tools here" and plain.tool_calls is None


def test_chat_stream_over_http(server):
    url, _ = server
    r = requests.post(url + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                          "max_tokens": 4, "ignore_eos": True, "stream": True},
                      stream=True, timeout=120)
    events = [json.loads(ln[6:]) for ln in r.iter_lines(decode_unicode=True)
              if ln.startswith("data: ") and ln != "data: [DONE]"]
    assert events[0]["choices"][0]["delta"]["role"] == "assistant"
    assert events[-1]["choices"][0]["finish_reason"] == "length"


def test_echo_and_stream_usage(server):
    url, _ = server
    body = {"prompt": "abc", "max_tokens": 4, "ignore_eos": True, "echo": True}
    r = requests.post(url + "/v1/completions", json=body, timeout=120).json()
    assert r["choices"][0]["text"].startswith("abc")
    r = requests.post(url + "/v1/completions", json=dict(body, stream=True, stream_options={"include_usage": True}),
                      stream=True, timeout=120)
    events = [json.loads(ln[6:]) for ln in r.iter_lines(decode_unicode=True)
              if ln.startswith("data: ") and ln != "data: [DONE]"]
    assert events[0]["choices"][0]["text"] == "abc"                      # echoed prompt first
    assert events[-1]["choices"] == [] and events[-1]["usage"]["completion_tokens"] == 4
    r = requests.post(url + "/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                          "max_tokens": 3, "ignore_eos": True, "stream": True,
                                                          "stream_options": {"include_usage": True}},
                      stream=True, timeout=120)
    events = [json.loads(ln[6:]) for ln in r.iter_lines(decode_unicode=True)
              if ln.startswith("data: ") and ln != "data: [DONE]"]
    assert events[-1]["usage"]["completion_tokens"] == 3 and events[-1]["usage"]["prompt_tokens"] > 0


def test_server_with_prefix_cache_chunked_prefill_and_dspark():
    """The server over an engine with prefix caching, chunked prefill and (context-free)
    DSpark drafting:
    completions sharing a prefix are the target's greedy tokens; the metrics count hits."""
    import uvicorn
    from vllm_moet_b200.engine.llm import LLM
    from vllm_moet_b200.entrypoints.openai_server import EngineWorker, build_app
    from vllm_moet_b200.models import reference
    llm = LLM("tiny-moe", device="cpu", num_speculative_tokens=0, max_model_len=256, speculative_method="dspark",
              dspark={"block": 3, "tau": 0.0, "budget_frac": 1.0, "model": "simple"}, enable_prefix_caching=True,
              prefix_block_size=8,
              enable_chunked_prefill=True, max_num_batched_tokens=8)
    w = EngineWorker(llm, "tiny")
    port = _free_port()
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
        pre = list(range(3, 27))
        for tail in ([50, 51], [60]):
            p = pre + tail
            r = requests.post(url + "/v1/completions", json={"prompt": p, "max_tokens": 6, "ignore_eos": True},
                              timeout=120).json()
            assert r["choices"][0]["token_ids"] == reference.greedy_generate(llm.mw, p, 6)
        m = requests.get(url + "/metrics").text
        hits = [ln for ln in m.splitlines() if ln.startswith("moet_prefix_cache_hits_total")]
        assert hits and float(hits[0].split()[-1]) == 1      # the second prompt reused 24 cached tokens
    finally:
        srv.should_exit = True
        th.join(timeout=10)
        w.close()


def test_beam_search_over_http(server):
    """use_beam_search: the beams come back best first and equal LLM.beam_search."""
    url, llm = server
    from vllm_moet_b200 import BeamSearchParams
    r = requests.post(url + "/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 4, "n": 2,
                                                     "use_beam_search": True, "ignore_eos": True}, timeout=300)
    assert r.ok, r.text
    ch = r.json()["choices"]
    want = llm.beam_search([[5, 6, 7, 8]], BeamSearchParams(beam_width=2, max_tokens=4, ignore_eos=True))[0]
    assert [c["token_ids"] for c in ch] == [s.generated for s in want.sequences]
    assert ch[0]["cumulative_logprob"] >= ch[1]["cumulative_logprob"]
    bad = requests.post(url + "/v1/completions", json={"prompt": [5], "use_beam_search": True, "stream": True},
                        timeout=60)
    assert bad.status_code == 400


def test_constrained_decoding_requests_are_refused(server):
    url, _ = server
    for extra in ({"response_format": {"type": "json_object"}}, {"guided_json": {"type": "object"}}):
        r = requests.post(url + "/v1/completions", json={"prompt": [5, 6], "max_tokens": 2, **extra}, timeout=60)
        assert r.status_code == 400, (extra, r.text)
    ok = requests.post(url + "/v1/completions", json={"prompt": [5, 6], "max_tokens": 2,
                                                      "response_format": {"type": "text"}}, timeout=120)
    assert ok.ok


def test_chat_beam_search_over_http(server):
    url, _ = server
    r = requests.post(url + "/v1/chat/completions",
                      json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3, "n": 2,
                            "use_beam_search": True, "ignore_eos": True}, timeout=300)
    assert r.ok, r.text
    ch = r.json()["choices"]
    assert len(ch) == 2 and ch[0]["cumulative_logprob"] >= ch[1]["cumulative_logprob"]
    assert all(c["message"]["role"] == "assistant" for c in ch)
