"""Open-loop HTTP load generator for the agentic trace.

Replays the same sessions / Poisson arrivals as the in-process replay, but
through an OpenAI-compatible ``/v1/completions`` endpoint with streaming:
each request's prompt is token ids, ``ignore_eos`` with the trace's output
length, and ``return_token_ids`` so the next turn can append exactly what
was generated. Time is the client's wall clock (``time.monotonic``).

Run as ``python -m infera_b200.bench.http_loadgen --url ... --sessions
A:B --rate R --duration S [--prewarm]``; prints one JSON object with the
per-request records on stdout. Arrivals are issued until ``duration``;
requests still in flight then are cancelled (``--drain-s``: wait that long
for them first). Running it as a separate process keeps the client's
parsing off the server's interpreter.
"""

from __future__ import annotations

import argparse
import asyncio
import json
import random
import sys
import time
from collections import deque

import httpx

from infera_b200.bench.trace import PRESETS, build_sessions


async def run(url: str, model: str, spec_name: str, sids: list[int], rate: float, duration: float, seed: int,
              stop_after_s: float | None = None, extra_body: dict | None = None, text_prompts: bool = False,
              start_at: float | None = None) -> dict:
    """``text_prompts``: send prompts as ``t<id>`` words and read generated
    ids back from the text (for servers whose tokenizer maps words to ids
    one to one; see :mod:`infera_b200.bench.hf_model_dir`)."""
    from infera_b200.bench.hf_model_dir import ids_to_text, text_to_ids

    spec = PRESETS[spec_name]
    sessions = build_sessions(spec, seed, sids)
    idle = deque(sessions)
    rng = random.Random(seed + 17)
    pending: deque[float] = deque()
    records: list[dict] = []
    t0 = time.monotonic() if start_at is None else start_at
    next_sid = max(sids) + 1 + 1_000_000 * (seed + 1)
    limits = httpx.Limits(max_connections=None, max_keepalive_connections=1024)
    tasks: set[asyncio.Task] = set()
    errors = [0]
    async with httpx.AsyncClient(base_url=url, timeout=httpx.Timeout(None, connect=30.0), limits=limits) as client:

        def now() -> float:
            return time.monotonic() - t0

        async def one(s, arrival):
            prompt = s.next_prompt()
            body = {"model": model, "prompt": ids_to_text(prompt) if text_prompts else prompt,
                    "max_tokens": s.out_lens[s.turn], "stream": True, "ignore_eos": True, "temperature": 0.0,
                    "stream_options": {"include_usage": True}}
            if not text_prompts:
                body["return_token_ids"] = True
            if extra_body:
                body.update(extra_body)
            rec = {"arrival": arrival, "token_times": [], "finish": None, "prompt_len": len(prompt),
                   "cached_len": 0, "out_len": 0}
            out_ids: list[int] = []
            try:
                async with client.stream("POST", "/v1/completions", json=body) as resp:
                    if resp.status_code >= 400:
                        await resp.aread()
                        errors[0] += 1
                    else:
                        buf = b""
                        async for chunk in resp.aiter_bytes():
                            buf += chunk
                            while b"\n\n" in buf:
                                ev, buf = buf.split(b"\n\n", 1)
                                line = ev.strip()
                                if not line.startswith(b"data:"):
                                    continue
                                data = line[5:].strip()
                                if data == b"[DONE]":
                                    rec["finish"] = now()
                                    continue
                                obj = json.loads(data)
                                t = now()
                                usage = obj.get("usage")
                                if usage:
                                    det = usage.get("prompt_tokens_details") or {}
                                    rec["cached_len"] = int(det.get("cached_tokens") or 0)
                                for ch in obj.get("choices") or []:
                                    ids = ch.get("token_ids")
                                    if ids is None and text_prompts:
                                        ids = text_to_ids(ch.get("text") or "")
                                    elif ids is None and ch.get("text") is not None:
                                        ids = [0]
                                    for tok in ids or []:
                                        out_ids.append(int(tok))
                                        rec["token_times"].append(t)
            except httpx.HTTPError:
                errors[0] += 1
            rec["out_len"] = len(out_ids)
            if rec["finish"] is None and rec["token_times"]:
                rec["finish"] = rec["token_times"][-1]
            records.append(rec)
            s.history = prompt + out_ids
            s.turn += 1
            s.busy = False
            s.idle_since = now()
            idle.append(s)

        t_next = rng.expovariate(rate)
        while now() < duration:
            t = now()
            while t_next <= t:
                pending.append(t_next)
                t_next += rng.expovariate(rate)
            while pending and idle:
                arr = pending.popleft()
                s = idle.popleft()
                since = s.idle_since
                if s.done(spec.context_cap):
                    fresh = build_sessions(spec, seed, [next_sid])[0]
                    fresh.group, fresh.prefix = s.group, s.prefix
                    next_sid += 1
                    s = fresh
                s.busy = True
                task = asyncio.create_task(one(s, max(arr, since)))
                tasks.add(task)
                task.add_done_callback(tasks.discard)
            await asyncio.sleep(min(0.002, max(0.0, t_next - now())))
        # let in-flight requests finish briefly so records near the window end resolve
        if tasks and stop_after_s:
            await asyncio.wait(list(tasks), timeout=stop_after_s)
        for task in list(tasks):
            task.cancel()
    return {"records": records, "errors": errors[0], "duration": duration}


async def prewarm(url: str, model: str, spec_name: str, sids: list[int], seed: int, text_prompts: bool = False,
                  extra: int = 8, extra_len: int = 1024, timeout: float = 600.0) -> dict:
    """Untimed warm-up given to every arm before its trace clock starts.

    Sends, concurrently, the system prefix of every prefix group among
    ``sids`` (16 output tokens each: the server caches the prefix and the
    router learns where it lives), and ``extra`` requests with fresh random
    prompts of ``extra_len`` tokens and 32 output tokens (first-use costs
    of batched prefill + decode shapes are paid here, not in the window).
    Returns counts of requests sent and failed."""
    from infera_b200.bench.hf_model_dir import ids_to_text

    spec = PRESETS[spec_name]
    sessions = build_sessions(spec, seed, sids)
    prompts, seen = [], set()
    for s in sessions:
        key = tuple(s.prefix[:8])
        if s.prefix and key not in seen:
            seen.add(key)
            prompts.append((s.prefix, 16))
    rng = random.Random(seed * 31 + 7)
    for _ in range(extra):
        prompts.append(([rng.randrange(spec.vocab) for _ in range(extra_len)], 32))
    failed = [0]
    t0 = time.monotonic()
    async with httpx.AsyncClient(base_url=url, timeout=httpx.Timeout(timeout, connect=30.0)) as client:

        async def one(p, n):
            body = {"model": model, "prompt": ids_to_text(p) if text_prompts else p, "max_tokens": n,
                    "ignore_eos": True, "temperature": 0.0}
            try:
                r = await client.post("/v1/completions", json=body)
                if r.status_code >= 400:
                    failed[0] += 1
            except httpx.HTTPError:
                failed[0] += 1

        await asyncio.gather(*(one(p, n) for p, n in prompts))
    return {"sent": len(prompts), "failed": failed[0], "wall_s": round(time.monotonic() - t0, 3)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", required=True)
    ap.add_argument("--model", default="llama-3.1-8b")
    ap.add_argument("--trace", default="agentic-8b")
    ap.add_argument("--sessions", required=True, help="A:B session id range")
    ap.add_argument("--rate", type=float, required=True)
    ap.add_argument("--duration", type=float, required=True)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--drain-s", type=float, default=0.0)
    ap.add_argument("--text-prompts", action="store_true")
    ap.add_argument("--prewarm", action="store_true", help="run prewarm() before the trace clock starts")
    a = ap.parse_args(argv)
    lo, hi = (int(x) for x in a.sessions.split(":"))
    warm = None
    if a.prewarm:
        warm = asyncio.run(prewarm(a.url, a.model, a.trace, list(range(lo, hi)), a.seed, text_prompts=a.text_prompts))
    res = asyncio.run(run(a.url, a.model, a.trace, list(range(lo, hi)), a.rate, a.duration, a.seed, a.drain_s,
                          text_prompts=a.text_prompts))
    res["prewarm"] = warm
    json.dump(res, sys.stdout)
    sys.stdout.flush()


if __name__ == "__main__":
    main()
