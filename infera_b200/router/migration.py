"""Mid-stream request migration.

While relaying a stream the router accumulates what the client has already
received (token ids when the worker returns them, else text). When the
stream breaks or the worker hands the request back while draining, the
generation continues on another worker: with exact ids the continuation is a
``/v1/completions`` call whose prompt is the original prompt ids plus the
generated ids; otherwise the generated text is appended to the prompt (or as
a partial assistant message). ``max_tokens`` shrinks by what was generated.
Continuation chunks from ``/v1/completions`` are reshaped into chat chunks
when the client asked for chat. Limited to ``limit`` hops per request; a
stream that cannot be re-tokenised faithfully is "poisoned" and not
migrated. Behaviour of ``infera/router/migration.py:64-375``.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass

from infera_b200.router.token_ids import (choice_text, choice_token_ids, finish_reason, parse_sse_json,
                                          strip_token_ids, to_sse)


def as_chat_chunk(ev: bytes) -> bytes:
    """Reshape a /v1/completions SSE chunk into a chat.completion.chunk."""
    obj = parse_sse_json(ev)
    if obj is None:
        return ev
    out = {"id": obj.get("id", ""), "object": "chat.completion.chunk", "created": obj.get("created", 0),
           "model": obj.get("model", ""), "choices": []}
    for ch in obj.get("choices") or []:
        out["choices"].append({"index": ch.get("index", 0), "delta": {"content": ch.get("text", "")},
                               "finish_reason": ch.get("finish_reason")})
    return to_sse(out)


@dataclass
class Continuation:
    body: dict
    path: str
    reshape_to_chat: bool


class MigrationState:
    def __init__(self, body: dict, limit: int, path: str, prompt_ids: list[int] | None = None):
        self.body = body
        self.limit = limit
        self.path = path
        self.hops = 0
        self.prompt_ids = prompt_ids
        self.gen_ids: list[int] = []
        self.gen_text = ""
        self.finished = False
        self.poisoned = False
        self.have_ids = True

    def observe(self, ev: bytes) -> bytes:
        """Record a relayed SSE event; return it with token ids stripped."""
        obj = parse_sse_json(ev)
        if obj is None:
            return ev
        if self.prompt_ids is None and isinstance(obj.get("prompt_token_ids"), list):
            self.prompt_ids = [int(x) for x in obj["prompt_token_ids"]]
        for ch in obj.get("choices") or []:
            if isinstance(ch.get("prompt_token_ids"), list) and self.prompt_ids is None:
                self.prompt_ids = [int(x) for x in ch["prompt_token_ids"]]
        ids = choice_token_ids(obj)
        text = choice_text(obj)
        if ids:
            self.gen_ids.extend(ids)
        elif text:
            self.have_ids = False
        self.gen_text += text
        if finish_reason(obj):
            self.finished = True
        return to_sse(strip_token_ids(obj))

    def can_migrate(self) -> bool:
        return not self.finished and not self.poisoned and self.hops < self.limit

    def remaining_tokens(self) -> int | None:
        mt = self.body.get("max_tokens") or self.body.get("max_completion_tokens")
        if mt is None:
            return None
        done = len(self.gen_ids) if self.have_ids else max(1, len(self.gen_text) // 4)
        return max(1, int(mt) - done)

    def next_continuation(self) -> Continuation:
        self.hops += 1
        body = copy.deepcopy({k: v for k, v in self.body.items() if not k.startswith("_infera")})
        rem = self.remaining_tokens()
        if rem is not None:
            body["max_tokens"] = rem
            body.pop("max_completion_tokens", None)
        chat = "messages" in body
        if self.have_ids and self.prompt_ids is not None:
            body.pop("messages", None)
            body["prompt"] = list(self.prompt_ids) + list(self.gen_ids)
            body["return_token_ids"] = True
            body["stream"] = True
            return Continuation(body, "/v1/completions", chat)
        if chat:
            msgs = list(body.get("messages") or [])
            msgs.append({"role": "assistant", "content": self.gen_text})
            body["messages"] = msgs
            body["continue_final_message"] = True
            body["add_generation_prompt"] = False
            return Continuation(body, self.path, False)
        prompt = body.get("prompt")
        if isinstance(prompt, str):
            body["prompt"] = prompt + self.gen_text
            return Continuation(body, self.path, False)
        self.poisoned = True
        return Continuation(body, self.path, False)
