"""The worker's OpenAI-compatible HTTP server and the HTTP load generator,
end to end on CPU with the tiny model."""

import asyncio
import threading
import time

import httpx
import pytest

from infera_b200.bench.http_loadgen import run as loadgen_run
from infera_b200.engine.async_engine import AsyncEngine
from infera_b200.engine.llm_engine import EngineConfig, LLMEngine
from infera_b200.engine.server import build_worker_app
from infera_b200.utils.tokenizer import ByteTokenizer


@pytest.fixture(scope="module")
def worker():
    import uvicorn

    eng = LLMEngine(EngineConfig(model="tiny-dense", use_cuda_graphs=False, num_pages=256), device="cpu")
    aeng = AsyncEngine(eng)
    aeng.start()
    app = build_worker_app(aeng, ByteTokenizer(vocab_size=1024), "tiny")
    server = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=18931, log_level="warning"))
    th = threading.Thread(target=server.run, daemon=True)
    th.start()
    t0 = time.time()
    while not server.started and time.time() - t0 < 20:
        time.sleep(0.05)
    yield "http://127.0.0.1:18931", aeng
    server.should_exit = True
    th.join(timeout=5)
    aeng.stop()


def test_completions_json_and_stream(worker):
    url, _ = worker
    r = httpx.post(url + "/v1/completions", json={"model": "tiny", "prompt": [5, 6, 7, 8], "max_tokens": 3,
                                                   "ignore_eos": True, "return_token_ids": True}, timeout=30)
    assert r.status_code == 200
    body = r.json()
    assert len(body["choices"][0]["token_ids"]) == 3
    assert body["usage"]["completion_tokens"] == 3
    with httpx.stream("POST", url + "/v1/chat/completions",
                      json={"model": "tiny", "messages": [{"role": "user", "content": "hi"}], "max_tokens": 4,
                            "ignore_eos": True, "stream": True}, timeout=30) as resp:
        text = b"".join(resp.iter_bytes())
    assert text.count(b"data: ") >= 5 and text.rstrip().endswith(b"[DONE]")
    m = httpx.get(url + "/metrics").text
    assert "infera_engine:num_requests_running" in m


def test_loadgen_multiturn(worker):
    url, _ = worker
    res = asyncio.run(loadgen_run(url, "tiny", "tiny", list(range(4)), rate=20.0, duration=2.0, seed=0,
                                  stop_after_s=5.0))
    recs = res["records"]
    assert res["errors"] == 0
    assert len(recs) >= 4
    for r in recs:
        assert r["out_len"] == len(r["token_times"]) and r["out_len"] > 0
        assert r["token_times"][0] >= r["arrival"]


def test_worker_tp_core_command_launches_ranks():
    """--tp-size N: the worker launches its engine core ranks with
    torch.distributed.run (rank r on cuda:(first + r))."""
    from infera_b200.engine.worker import _core_cmd, parse_args

    a = parse_args(["--model", "llama-3.1-70b", "--tp-size", "4", "--first-device", "4", "--disagg-mode", "decode",
                    "--kv-push-endpoint", "ipc:///tmp/x"])
    cmd = _core_cmd(a, "ipc:///tmp/in", "ipc:///tmp/out")
    assert cmd[1:3] == ["-m", "torch.distributed.run"] and "--nproc-per-node=4" in cmd
    i = cmd.index("infera_b200.engine.core_ipc")
    assert cmd[i + 1:i + 5] == ["--tp-size", "4", "--first-device", "4"]
    assert "--kv-push-endpoint" in cmd and cmd[cmd.index("--disagg-mode") + 1] == "decode"
    single = _core_cmd(parse_args([]), "a", "b")
    assert single[1:3] == ["-m", "infera_b200.engine.core_ipc"]
