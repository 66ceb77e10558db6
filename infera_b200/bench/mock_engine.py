"""A GPU-free stand-in engine worker for router plumbing tests and the
CPU fleet benchmark.

Service model (per request, no batching interference):
``prefill_ms_per_token`` (0.05 ms) for every prompt token whose 16-token
block is not in the worker's LRU prefix set (4096 blocks), then one output
token every ``decode_ms_per_token`` (10 ms). The prefix set is keyed by the
router's chained block hashes, and every insertion / eviction is published
as a vLLM-encoding KV event over ZMQ (``BlockStored`` with token ids,
``BlockRemoved``), so the router's view is built exactly as for a real
engine. The worker speaks the same OpenAI streaming API as the real one
(token ids in the prompt, ``return_token_ids``), reports in-flight counts on
/metrics, and drains: on ``shutdown()`` it deregisters first, then waits for
its in-flight requests to finish.
"""

from __future__ import annotations

import asyncio
import json
import random
import threading
import time
import uuid
from collections import OrderedDict

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, Response, StreamingResponse

from infera_b200.engine.kv_events import KvEventPublisher
from infera_b200.utils.hashing import chain_hashes
from infera_b200.utils.tokenizer import ByteTokenizer, request_token_ids


class MockEngine:
    def __init__(self, *, capacity_blocks: int = 4096, block_size: int = 16, prefill_ms_per_token: float = 0.05,
                 decode_ms_per_token: float = 10.0, vocab: int = 32000, publisher: KvEventPublisher | None = None,
                 seed: int = 0):
        self.cap = capacity_blocks
        self.bs = block_size
        self.prefill_s = prefill_ms_per_token / 1000.0
        self.decode_s = decode_ms_per_token / 1000.0
        self.vocab = vocab
        self.pub = publisher
        self.lru: OrderedDict[int, None] = OrderedDict()
        self.rng = random.Random(seed)
        self.inflight = 0
        self.draining = False
        self.fail_next = 0          # fault injection: next N requests fail before the first byte
        self.break_after = None     # fault injection: break streams after N tokens
        self.stats = {"requests": 0, "hit_tokens": 0, "prompt_tokens": 0}
        self.lock = threading.Lock()

    def _insert(self, tokens: list[int], hashes: list[int]) -> None:
        stored_h, stored_t, removed = [], [], []
        parent = None
        first_new = None
        for i, h in enumerate(hashes):
            if h in self.lru:
                self.lru.move_to_end(h)
                parent = h
                continue
            if first_new is None:
                first_new = i
            self.lru[h] = None
            stored_h.append(h)
            stored_t.extend(tokens[i * self.bs:(i + 1) * self.bs])
        while len(self.lru) > self.cap:
            h, _ = self.lru.popitem(last=False)
            removed.append(h)
        if self.pub is not None:
            if removed:
                self.pub("BlockRemoved", {"block_hashes": removed, "medium": "GPU"})
            if stored_h:
                par = hashes[first_new - 1] if first_new else None
                self.pub("BlockStored", {"block_hashes": stored_h, "parent_block_hash": par, "token_ids": stored_t,
                                         "block_size": self.bs, "lora_id": None, "medium": "GPU"})
            self.pub.flush()
        del parent

    def cached_prefix_tokens(self, hashes: list[int]) -> int:
        n = 0
        for h in hashes:
            if h not in self.lru:
                break
            n += 1
        return n * self.bs

    async def generate(self, prompt: list[int], max_tokens: int):
        """Yields token ids with the modelled timing."""
        hashes = chain_hashes(prompt, self.bs)
        with self.lock:
            hit = self.cached_prefix_tokens(hashes)
            self.stats["requests"] += 1
            self.stats["hit_tokens"] += hit
            self.stats["prompt_tokens"] += len(prompt)
        await asyncio.sleep(max(0, len(prompt) - hit) * self.prefill_s)
        with self.lock:
            self._insert(prompt, hashes)
        for i in range(max_tokens):
            if i > 0:
                await asyncio.sleep(self.decode_s)
            yield self.rng.randrange(self.vocab), hit


class WordIdTokenizer:
    """Text prompts written as ``t<id>`` words (one word per token id), the
    form in which the benchmark sends token-id traces through routers that
    accept text only (see ``infera_b200.bench.hf_model_dir``)."""

    name = "word-ids"

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        from infera_b200.bench.hf_model_dir import text_to_ids

        return text_to_ids(text)

    def apply_chat_template(self, messages: list[dict], add_generation_prompt: bool = True) -> list[int]:
        return self.encode(" ".join(str(m.get("content") or "") for m in messages))


def build_mock_app(eng: MockEngine, model: str, word_ids: bool = False) -> FastAPI:
    """``word_ids``: string prompts are ``t<id>`` words and generated text
    is written the same way (for text-only routers)."""
    app = FastAPI()
    tok = WordIdTokenizer() if word_ids else ByteTokenizer(vocab_size=eng.vocab)

    async def run(body: dict, chat: bool):
        if eng.draining:
            return JSONResponse({"error": {"message": "worker is draining"}}, status_code=503)
        if eng.fail_next > 0:
            eng.fail_next -= 1
            return JSONResponse({"error": {"message": "injected failure"}}, status_code=500)
        ids = request_token_ids(body, tok)
        mt = int(body.get("max_tokens") or 16)
        want_ids = bool(body.get("return_token_ids"))
        rid = uuid.uuid4().hex
        created = int(time.time())
        kind = "chat.completion.chunk" if chat else "text_completion"
        eng.inflight += 1

        def chunk(tok_id, finish):
            txt = f" t{tok_id}" if word_ids else "x"
            c = ({"index": 0, "delta": {"content": txt}, "finish_reason": finish} if chat
                 else {"index": 0, "text": txt, "finish_reason": finish})
            if want_ids:
                c["token_ids"] = [tok_id]
            return {"id": rid, "object": kind, "created": created, "model": model, "choices": [c]}

        if not body.get("stream"):
            out = []
            cached = 0
            try:
                async for t, hit in eng.generate(ids, mt):
                    out.append(t)
                    cached = hit
            finally:
                eng.inflight -= 1
            ch = {"index": 0, "text": "x" * len(out), "finish_reason": "length"}
            if chat:
                ch = {"index": 0, "message": {"role": "assistant", "content": "x" * len(out)},
                      "finish_reason": "length"}
            if want_ids:
                ch["token_ids"] = out
            return JSONResponse({"id": rid, "object": "chat.completion" if chat else "text_completion",
                                 "model": model, "choices": [ch],
                                 "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                                           "prompt_tokens_details": {"cached_tokens": cached}}})

        async def gen():
            n = 0
            try:
                first = True
                async for t, hit in eng.generate(ids, mt):
                    n += 1
                    c = chunk(t, "length" if n == mt else None)
                    if first and want_ids:
                        c["prompt_token_ids"] = ids
                    first = False
                    yield b"data: " + json.dumps(c).encode() + b"\n\n"
                    if eng.break_after is not None and n >= eng.break_after:
                        return  # injected mid-stream break: no [DONE]
                yield b"data: " + json.dumps({"id": rid, "object": kind, "model": model, "choices": [],
                                              "usage": {"prompt_tokens": len(ids), "completion_tokens": n,
                                                        "prompt_tokens_details": {"cached_tokens": hit}}}).encode() \
                    + b"\n\n"
                yield b"data: [DONE]\n\n"
            finally:
                eng.inflight -= 1

        return StreamingResponse(gen(), media_type="text/event-stream")

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await run(await request.json(), False)

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await run(await request.json(), True)

    @app.get("/health")
    async def health():
        return {"status": "ok"}

    @app.get("/metrics")
    async def metrics():
        return Response(f"infera_engine:num_requests_running{{model_name=\"{model}\"}} {eng.inflight}\n"
                        f"infera_engine:num_requests_waiting{{model_name=\"{model}\"}} 0\n",
                        media_type="text/plain")

    @app.post("/start_profile")
    async def start_profile():
        return {"status": "started"}

    @app.post("/stop_profile")
    async def stop_profile():
        return {"status": "stopped"}

    return app
