"""DeepSeek-V4-style chat encoding: rendering OpenAI-format messages to a
prompt string and parsing a completion back into a message.

Semantics follow the reference's DS4 encoding changes (patch P:15130-15429):

* reasoning effort: ``none`` disables thinking; ``low`` (default) adds no
  prompt; ``high`` and ``max`` prepend their effort prompt at the start of the
  conversation; ``xhigh`` is an alias of ``max``; any other string rounds up to
  ``high``;
* a prior assistant turn's reasoning travels in the OpenAI-style
  ``reasoning_content`` key and is rendered inside the think block only for the
  turns after the last user message (earlier reasoning is dropped);
* tool calls are written in DSML (``<｜DSML｜function_calls>`` / ``invoke`` /
  ``parameter name=.. string="true|false"``); arguments may be a JSON string
  or a dict; an argument string that is not JSON is kept under the key
  ``arguments``; tool outputs are wrapped in ``<tool_result>``;
* parsing accepts ``reasoning</think>content`` (thinking mode) followed by an
  optional DSML tool-call block and the EOS token, and rejects special tokens
  inside content.
"""
from __future__ import annotations

import json
import re
from typing import Any, Dict, List, Optional, Tuple

BOS = "<｜begin▁of▁sentence｜>"
EOS = "<｜end▁of▁sentence｜>"
USER = "<｜User｜>"
ASSISTANT = "<｜Assistant｜>"
THINK_START, THINK_END = "<think>", "</think>"
DSML = "｜DSML｜"
CALLS_BLOCK = "function_calls"
SPECIAL = (BOS, EOS, THINK_START, THINK_END, DSML)

EFFORT_PROMPTS: Dict[str, str] = {
    "low": "",
    "high": ("Reasoning Effort: Absolute maximum with no shortcuts permitted.\n"
             "You MUST be very thorough in your thinking and comprehensively decompose the problem to resolve the "
             "root cause, rigorously stress-testing your logic against all potential paths, edge cases, and "
             "adversarial scenarios.\n"
             "Explicitly write out your entire deliberation process, documenting every intermediate step, considered "
             "alternative, and rejected hypothesis to ensure absolutely no assumption is left unchecked.\n\n"),
    "max": ("Reasoning Effort: Beyond maximum — exhaustive, relentless, and uncompromising.\n"
            "You MUST reason with the utmost depth and rigor, leaving absolutely nothing to chance: exhaustively "
            "decompose the problem into its most fundamental components, trace every causal chain to its root, and "
            "resolve the underlying cause rather than any surface symptom.\n"
            "Do not stop reasoning until you have independently verified the solution from multiple angles and are "
            "certain that no assumption remains unchecked and no error remains undiscovered.\n\n"),
}


def normalize_effort(effort: Optional[str]) -> Optional[str]:
    """-> None (thinking off), 'low', 'high' or 'max'."""
    if effort is None:
        return "low"
    if not isinstance(effort, str):
        return "low"
    e = effort.strip().lower()
    if e == "none":
        return None
    if e in ("max", "xhigh"):
        return "max"
    if e == "low":
        return "low"
    return "high"


def _to_json(v: Any) -> str:
    try:
        return json.dumps(v, ensure_ascii=False)
    except (TypeError, ValueError):
        return json.dumps(str(v))


def encode_tool_call(call: Dict[str, Any]) -> str:
    fn = call.get("function", call)
    args = fn.get("arguments", {})
    if isinstance(args, str):
        try:
            args = json.loads(args)
        except json.JSONDecodeError:
            args = {"arguments": args}
    if not isinstance(args, dict):
        args = {"arguments": args}
    params = []
    for k, v in args.items():
        is_str = isinstance(v, str)
        params.append(f'<{DSML}parameter name="{k}" string="{"true" if is_str else "false"}">'
                      f'{v if is_str else _to_json(v)}</{DSML}parameter>')
    return f'<{DSML}invoke name="{fn["name"]}">\n' + "\n".join(params) + f"\n</{DSML}invoke>"


def encode_tool_calls(calls: List[Dict[str, Any]]) -> str:
    return (f"\n\n<{DSML}{CALLS_BLOCK}>\n" + "\n".join(encode_tool_call(c) for c in calls)
            + f"\n</{DSML}{CALLS_BLOCK}>")


def _tools_section(tools: List[Dict[str, Any]]) -> str:
    lines = ["## Tools", "", "You may call the following functions by emitting a DSML function_calls block:"]
    for t in tools:
        fn = t.get("function", t)
        lines.append(_to_json({"name": fn.get("name"), "description": fn.get("description", ""),
                               "parameters": fn.get("parameters", {})}))
    return "\n".join(lines) + "\n\n"


def render(messages: List[Dict[str, Any]], tools: Optional[List[Dict[str, Any]]] = None,
           reasoning_effort: Optional[str] = "low", add_generation_prompt: bool = True, add_bos: bool = True) -> str:
    effort = normalize_effort(reasoning_effort)
    thinking = effort is not None
    last_user = max((i for i, m in enumerate(messages) if m.get("role") == "user"), default=-1)
    out = [BOS] if add_bos else []
    if thinking and EFFORT_PROMPTS[effort]:
        out.append(EFFORT_PROMPTS[effort])
    sys_parts = [m.get("content") or "" for m in messages if m.get("role") == "system"]
    if tools:
        sys_parts.append(_tools_section(tools))
    if sys_parts:
        out.append("".join(sys_parts))
    for i, m in enumerate(messages):
        role = m.get("role")
        if role == "system":
            continue
        if role == "user":
            out.append(USER + (m.get("content") or ""))
        elif role == "tool":
            out.append(USER + f"<tool_result>{m.get('content') or ''}</tool_result>")
        elif role == "assistant":
            out.append(ASSISTANT)
            rc = m.get("reasoning_content")
            if thinking and i > last_user:
                out.append(THINK_START + (rc or "") + THINK_END)
            elif thinking:
                out.append(THINK_END)
            out.append(m.get("content") or "")
            if m.get("tool_calls"):
                out.append(encode_tool_calls(m["tool_calls"]))
            out.append(EOS)
        else:
            raise ValueError(f"unknown role {role!r}")
    if add_generation_prompt:
        out.append(ASSISTANT + (THINK_START if thinking else THINK_END))
    return "".join(out)


_PARAM = re.compile(rf'<{DSML}parameter name="([^"]*)" string="(true|false)">(.*?)</{DSML}parameter>', re.S)
_INVOKE = re.compile(rf'<{DSML}invoke name="([^"]*)">(.*?)</{DSML}invoke>', re.S)


def parse_completion(text: str, thinking: bool = True) -> Dict[str, Any]:
    """Completion text (after the generation prompt) -> assistant message dict."""
    reasoning = ""
    rest = text
    if thinking:
        if THINK_END not in rest:
            raise ValueError("invalid thinking format: missing </think>")
        reasoning, rest = rest.split(THINK_END, 1)
    start = f"\n\n<{DSML}{CALLS_BLOCK}>"
    calls = []
    if start in rest:
        content, block = rest.split(start, 1)
        end = f"</{DSML}{CALLS_BLOCK}>"
        if end not in block:
            raise ValueError("invalid tool-call block: missing end tag")
        body, tail = block.split(end, 1)
        for n, (name, inner) in enumerate(_INVOKE.findall(body)):
            args = {}
            for k, is_str, v in _PARAM.findall(inner):
                args[k] = v if is_str == "true" else json.loads(v)
            calls.append({"id": f"call_{n}", "type": "function",
                          "function": {"name": name, "arguments": json.dumps(args, ensure_ascii=False)}})
        rest_after = tail
    else:
        content, rest_after = rest, ""
    content = content.replace(EOS, "") if not calls else content
    if rest_after.strip() not in ("", EOS):
        raise ValueError("unexpected content after the tool-call block")
    if content.endswith(EOS):
        content = content[: -len(EOS)]
    for tok in SPECIAL:
        if tok in content or tok in reasoning:
            raise ValueError(f"unexpected special token {tok!r} in content")
    msg: Dict[str, Any] = {"role": "assistant", "content": content}
    if thinking:
        msg["reasoning_content"] = reasoning
    if calls:
        msg["tool_calls"] = calls
    return msg
