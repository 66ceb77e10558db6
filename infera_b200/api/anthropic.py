"""Anthropic Messages API <-> OpenAI Chat Completions translation.

Request: ``system`` (string or text blocks) becomes the first system
message; user/assistant content blocks map to OpenAI messages (text
concatenated; ``tool_use`` -> assistant ``tool_calls``; ``tool_result`` ->
``tool`` role messages); ``tools`` -> function tools (``input_schema`` ->
``parameters``); ``tool_choice`` auto/any/tool/none -> auto/required/named/
none; ``stop_sequences`` -> ``stop``; sampling fields pass through.
Image / document / audio content is rejected with HTTP 400 (the text-only
block hashing cannot tell media apart).

Response: OpenAI JSON -> one ``message`` (text block, tool_use blocks with
parsed JSON input, ``stop_reason`` end_turn / max_tokens / tool_use /
stop_sequence, usage). Streaming: OpenAI SSE chunks -> ``message_start``,
``content_block_start`` / ``content_block_delta`` (text_delta,
input_json_delta) / ``content_block_stop``, ``message_delta`` with the stop
reason and output tokens, ``message_stop``. Behaviour of
``infera/api/anthropic.py:87-879``.
"""

from __future__ import annotations

import json
import time
import uuid
from typing import Any, AsyncIterator

MEDIA_TYPES = frozenset({"image", "document", "audio", "video", "file", "input_image", "input_audio"})


class TranslationError(ValueError):
    """A client error: the router answers it with HTTP 400."""


def _text_of(content: Any) -> str:
    if isinstance(content, str):
        return content
    if isinstance(content, list):
        return "".join(str(b.get("text", "")) for b in content if isinstance(b, dict) and b.get("type") == "text")
    return ""


def reject_if_multimodal(body: dict) -> None:
    def check(blocks, where):
        if isinstance(blocks, list):
            for b in blocks:
                if isinstance(b, dict) and b.get("type") in MEDIA_TYPES:
                    raise TranslationError(f"{b.get('type')} content in {where} is not supported")
                if isinstance(b, dict) and b.get("type") == "tool_result":
                    check(b.get("content"), "tool_result")

    check(body.get("system"), "system")
    for m in body.get("messages") or []:
        if isinstance(m, dict):
            check(m.get("content"), "messages")


def _tool_def(t: dict) -> dict:
    if t.get("type") not in (None, "custom") and "input_schema" not in t:
        raise TranslationError(f"unsupported tool type {t.get('type')!r}")
    fn = {"name": t["name"], "parameters": t.get("input_schema") or {"type": "object", "properties": {}}}
    if t.get("description"):
        fn["description"] = t["description"]
    return {"type": "function", "function": fn}


def _tool_choice(tc: Any) -> Any:
    if tc is None:
        return None
    if isinstance(tc, str):
        tc = {"type": tc}
    kind = tc.get("type")
    if kind == "auto":
        return "auto"
    if kind == "any":
        return "required"
    if kind == "none":
        return "none"
    if kind == "tool":
        if not tc.get("name"):
            raise TranslationError("tool_choice of type 'tool' needs a name")
        return {"type": "function", "function": {"name": tc["name"]}}
    raise TranslationError(f"unknown tool_choice {kind!r}")


def _messages(role: str, content: Any) -> list[dict]:
    if isinstance(content, str):
        return [{"role": role, "content": content}]
    if not isinstance(content, list):
        raise TranslationError("message content must be a string or a list of blocks")
    out: list[dict] = []
    text: list[str] = []
    calls: list[dict] = []
    for b in content:
        if not isinstance(b, dict):
            continue
        t = b.get("type")
        if t == "text":
            text.append(str(b.get("text", "")))
        elif t in ("thinking", "redacted_thinking"):
            continue
        elif t == "tool_use":
            if role != "assistant":
                raise TranslationError("tool_use blocks belong to assistant messages")
            calls.append({"id": b.get("id") or f"toolu_{uuid.uuid4().hex[:24]}", "type": "function",
                          "function": {"name": b.get("name", ""), "arguments": json.dumps(b.get("input", {}))}})
        elif t == "tool_result":
            if text:
                out.append({"role": role, "content": "".join(text)})
                text = []
            c = b.get("content")
            body = _text_of(c) if not isinstance(c, str) else c
            if b.get("is_error"):
                body = "[error] " + body
            out.append({"role": "tool", "tool_call_id": b.get("tool_use_id", ""), "content": body})
        else:
            raise TranslationError(f"unsupported content block {t!r}")
    if calls:
        out.append({"role": "assistant", "content": "".join(text) or None, "tool_calls": calls})
    elif text or not out:
        out.append({"role": role, "content": "".join(text)})
    return out


def anthropic_to_openai_request(body: dict) -> dict:
    if not isinstance(body, dict):
        raise TranslationError("body must be a JSON object")
    reject_if_multimodal(body)
    if "max_tokens" not in body:
        raise TranslationError("max_tokens is required")
    msgs: list[dict] = []
    sys_text = _text_of(body.get("system")) if body.get("system") is not None else ""
    if sys_text:
        msgs.append({"role": "system", "content": sys_text})
    for m in body.get("messages") or []:
        role = m.get("role")
        if role not in ("user", "assistant"):
            raise TranslationError(f"unsupported role {role!r}")
        msgs.extend(_messages(role, m.get("content")))
    out: dict[str, Any] = {"model": body.get("model"), "messages": msgs, "max_tokens": int(body["max_tokens"]),
                           "stream": bool(body.get("stream", False))}
    for k in ("temperature", "top_p", "top_k"):
        if body.get(k) is not None:
            out[k] = body[k]
    if body.get("stop_sequences"):
        out["stop"] = list(body["stop_sequences"])
    if body.get("tools"):
        out["tools"] = [_tool_def(t) for t in body["tools"]]
    tc = _tool_choice(body.get("tool_choice"))
    if tc is not None:
        out["tool_choice"] = tc
    if out["stream"]:
        out["stream_options"] = {"include_usage": True}
    md = body.get("metadata") or {}
    if isinstance(md, dict) and md.get("user_id"):
        out["user"] = str(md["user_id"])
    return out


def map_finish_reason(r: str | None) -> str | None:
    if r is None:
        return None
    return {"stop": "end_turn", "length": "max_tokens", "tool_calls": "tool_use", "function_call": "tool_use",
            "content_filter": "end_turn", "stop_sequence": "stop_sequence"}.get(r, "end_turn")


def _msg_id() -> str:
    return f"msg_{uuid.uuid4().hex[:24]}"


def openai_to_anthropic_response(resp: dict, model: str | None = None) -> dict:
    ch = (resp.get("choices") or [{}])[0]
    msg = ch.get("message") or {}
    content: list[dict] = []
    if msg.get("content"):
        content.append({"type": "text", "text": msg["content"]})
    for tc in msg.get("tool_calls") or []:
        fn = tc.get("function") or {}
        try:
            args = json.loads(fn.get("arguments") or "{}")
        except ValueError:
            args = {"_raw": fn.get("arguments")}
        content.append({"type": "tool_use", "id": tc.get("id") or f"toolu_{uuid.uuid4().hex[:24]}",
                        "name": fn.get("name", ""), "input": args})
    if not content:
        content.append({"type": "text", "text": ""})
    usage = resp.get("usage") or {}
    stop = map_finish_reason(ch.get("finish_reason"))
    if ch.get("stop_reason") is not None and ch.get("finish_reason") == "stop" and isinstance(ch["stop_reason"],
                                                                                             str):
        stop = "stop_sequence"
    return {"id": _msg_id(), "type": "message", "role": "assistant", "model": model or resp.get("model", ""),
            "content": content, "stop_reason": stop,
            "stop_sequence": ch.get("stop_reason") if stop == "stop_sequence" else None,
            "usage": {"input_tokens": int(usage.get("prompt_tokens", 0)),
                      "output_tokens": int(usage.get("completion_tokens", 0))}}


def _sse(event: str, payload: dict) -> bytes:
    return f"event: {event}\ndata: {json.dumps(payload, separators=(',', ':'))}\n\n".encode()


async def openai_to_anthropic_sse(chunks: AsyncIterator[bytes], model: str | None = None) -> AsyncIterator[bytes]:
    """Translate an OpenAI chat SSE byte stream into Anthropic events."""
    started = False
    block_open: str | None = None       # "text" or "tool:<index>"
    block_idx = -1
    tool_slots: dict[int, int] = {}
    finish = None
    out_tokens = 0
    in_tokens = 0
    buf = b""

    def start_msg():
        return _sse("message_start", {"type": "message_start", "message": {
            "id": _msg_id(), "type": "message", "role": "assistant", "model": model or "", "content": [],
            "stop_reason": None, "stop_sequence": None, "usage": {"input_tokens": in_tokens, "output_tokens": 0}}})

    async for raw in chunks:
        buf += raw
        while b"\n\n" in buf:
            ev, buf = buf.split(b"\n\n", 1)
            line = ev.strip()
            if not line.startswith(b"data:"):
                continue
            data = line[5:].strip()
            if data == b"[DONE]":
                continue
            try:
                obj = json.loads(data)
            except ValueError:
                continue
            if "error" in obj and not obj.get("choices"):
                yield _sse("error", {"type": "error", "error": {"type": "api_error", "message": str(obj["error"])}})
                return
            usage = obj.get("usage") or {}
            if usage:
                in_tokens = int(usage.get("prompt_tokens", in_tokens))
                out_tokens = int(usage.get("completion_tokens", out_tokens))
            if not started:
                started = True
                yield start_msg()
            for ch in obj.get("choices") or []:
                delta = ch.get("delta") or {}
                text = delta.get("content")
                if text:
                    if block_open != "text":
                        if block_open is not None:
                            yield _sse("content_block_stop", {"type": "content_block_stop", "index": block_idx})
                        block_idx += 1
                        block_open = "text"
                        yield _sse("content_block_start", {"type": "content_block_start", "index": block_idx,
                                                           "content_block": {"type": "text", "text": ""}})
                    yield _sse("content_block_delta", {"type": "content_block_delta", "index": block_idx,
                                                       "delta": {"type": "text_delta", "text": text}})
                for tc in delta.get("tool_calls") or []:
                    ti = int(tc.get("index", 0))
                    fn = tc.get("function") or {}
                    if ti not in tool_slots:
                        if block_open is not None:
                            yield _sse("content_block_stop", {"type": "content_block_stop", "index": block_idx})
                        block_idx += 1
                        tool_slots[ti] = block_idx
                        block_open = f"tool:{ti}"
                        yield _sse("content_block_start", {"type": "content_block_start", "index": block_idx,
                                                           "content_block": {"type": "tool_use",
                                                                             "id": tc.get("id") or f"toolu_{ti}",
                                                                             "name": fn.get("name", ""),
                                                                             "input": {}}})
                    if fn.get("arguments"):
                        yield _sse("content_block_delta", {"type": "content_block_delta", "index": tool_slots[ti],
                                                           "delta": {"type": "input_json_delta",
                                                                     "partial_json": fn["arguments"]}})
                if ch.get("finish_reason"):
                    finish = ch["finish_reason"]
    if not started:
        yield start_msg()
    if block_open is not None:
        yield _sse("content_block_stop", {"type": "content_block_stop", "index": block_idx})
    yield _sse("message_delta", {"type": "message_delta",
                                 "delta": {"stop_reason": map_finish_reason(finish or "stop"), "stop_sequence": None},
                                 "usage": {"output_tokens": out_tokens}})
    yield _sse("message_stop", {"type": "message_stop"})


def now_ts() -> int:
    return int(time.time())
