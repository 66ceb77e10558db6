"""Router unit tests: KV-aware policy behaviour, round-robin, targets, circuit
breaker, cache hints, KV-event client, protocols."""

import pytest

from infera_b200.common.worker_pool import DisaggMode, WorkerInfo, WorkerPool, WorkerStatus
from infera_b200.router.breaker import BreakerState, CircuitBreaker, is_worker_fault
from infera_b200.router.cache_control import Retention, extract_image_keys, parse_cache_hints
from infera_b200.router.disagg_protocols import ProtocolError, resolve_protocol
from infera_b200.router.kv_event.block_hasher import BlockHasher
from infera_b200.router.kv_event.client import KvEventClient
from infera_b200.router.kv_event.events import (AllBlocksCleared, BlockRemoved, BlockStored, KVEventBatch,
                                                decoder_for_engine, encode_batch)
from infera_b200.router.policy.kv_aware import KvAwarePolicy
from infera_b200.router.policy.round_robin import RoundRobinPolicy
from infera_b200.router.policy.target import RouteTarget, expand_targets
from infera_b200.utils.hashing import chain_hashes


def W(i, **kw):
    return WorkerInfo(worker_id=f"w{i}", url=f"http://w{i}", model_name="m", kv_block_size=16, **kw)


def _policy(workers, w=1.0):
    client = KvEventClient(use_zmq=False)
    for x in workers:
        client.on_worker_added(x)
    return KvAwarePolicy(client, BlockHasher(), overlap_weight=w), client


def _store(client, wid, tokens):
    client.feed(wid, [BlockStored(block_hashes=chain_hashes(tokens, 16), parent_block_hash=None, token_ids=tokens,
                                  block_size=16, lora_id=None)])


def test_only_holder_wins():
    ws = [W(0), W(1), W(2)]
    pol, client = _policy(ws)
    prompt = list(range(1000, 1000 + 640))
    _store(client, "w1", prompt)
    t, blocks = pol.pick(ws, {"prompt": prompt + [1, 2, 3]})
    assert t.worker.worker_id == "w1"
    assert len(blocks) == 40


def test_cold_fleet_spreads_with_recent_decay():
    ws = [W(0), W(1), W(2), W(3)]
    pol, _ = _policy(ws, w=20.0)
    picks = []
    for i in range(40):
        prompt = [(i * 7919 + j) % 30000 for j in range(320)]
        t, _ = pol.pick(ws, {"prompt": prompt})
        picks.append(t.worker.worker_id)
    counts = {w.worker_id: picks.count(w.worker_id) for w in ws}
    assert min(counts.values()) >= 5, counts


def test_unknown_cost_floor_rotates_short_prompts():
    ws = [W(0), W(1)]
    pol, _ = _policy(ws)
    picked = {pol.pick(ws, {"prompt": [1, 2, 3]})[0].worker.worker_id for _ in range(4)}
    assert picked == {"w0", "w1"}


def test_active_blocks_refcount_and_removal():
    ws = [W(0), W(1)]
    pol, _ = _policy(ws)
    pol.on_request_started("w0", [1, 2, 3])
    pol.on_request_started("w0", [2, 3, 4])
    assert pol.active_blocks("w0") == 4
    pol.on_request_finished("w0", [1, 2, 3])
    assert pol.active_blocks("w0") == 3
    pol.on_worker_removed("w0")
    assert pol.active_blocks("w0") == 0


def test_multimodal_ignores_locality():
    ws = [W(0), W(1)]
    pol, client = _policy(ws)
    _store(client, "w0", list(range(160)))
    body = {"messages": [{"role": "user", "content": [{"type": "image_url", "image_url": {"url": "http://x/a.png"}},
                                                      {"type": "text", "text": "hi"}]}]}
    h = parse_cache_hints(body)
    assert h.has_multimodal_content
    assert extract_image_keys(body)
    # first pick records affinity; the same image goes back to the same worker
    t1, _ = pol.pick(ws, dict(body))
    t2, _ = pol.pick(ws, dict(body))
    assert t1.worker.worker_id == t2.worker.worker_id


def test_round_robin_per_candidate_set():
    ws = [W(0), W(1), W(2)]
    rr = RoundRobinPolicy()
    a = [rr.pick(ws, {})[0].worker.worker_id for _ in range(3)]
    assert sorted(a) == ["w0", "w1", "w2"]
    b = [rr.pick(ws[:2], {}, role_hint="decode")[0].worker.worker_id for _ in range(2)]
    assert sorted(b) == ["w0", "w1"]


def test_dp_expansion_route_keys():
    w = W(0, dp_size=4)
    ts = expand_targets([w])
    assert [t.route_key for t in ts] == ["w0#dp0", "w0#dp1", "w0#dp2", "w0#dp3"]
    fixed = W(1, dp_size=4, dp_rank=2)
    assert [t.route_key for t in expand_targets([fixed])] == ["w1"]


def test_breaker_lifecycle():
    now = [0.0]
    br = CircuitBreaker(failure_threshold=3, cooldown=5.0, max_cooldown=60.0, now=lambda: now[0])
    for _ in range(2):
        br.record_failure("w", 500)
    assert br.state("w") == BreakerState.CLOSED
    br.record_failure("w", 503)
    assert br.state("w") == BreakerState.OPEN and not br.allows("w")
    br.record_failure("x", 404)  # client errors are neutral
    assert br.state("x") == BreakerState.CLOSED
    now[0] = 5.1
    assert br.allows("w")          # half-open probe
    assert not br.allows("w")      # only one probe at a time
    br.record_failure("w", 500)    # failed probe doubles the cooldown
    now[0] = 5.1 + 9.9
    assert not br.allows("w")
    now[0] = 5.1 + 10.1
    assert br.allows("w")
    br.record_success("w")
    assert br.state("w") == BreakerState.CLOSED
    assert is_worker_fault(0) and is_worker_fault(502) and not is_worker_fault(429)


def test_breaker_all_open_routes_anyway():
    br = CircuitBreaker(failure_threshold=1, now=lambda: 0.0)
    ws = [W(0), W(1)]
    for w in ws:
        br.record_failure(w.worker_id, 500)
    assert len(br.filter(ws)) == 2


def test_cache_hints():
    h = parse_cache_hints({"messages": [{"role": "user", "content": [
        {"type": "text", "text": "a", "cache_control": {"type": "ephemeral"}}]}]})
    assert h.retention == Retention.SHORT and h.explicit_hint_seen
    h = parse_cache_hints({"system": [{"type": "text", "text": "s",
                                       "cache_control": {"type": "ephemeral", "ttl": "1h"}}], "messages": []})
    assert h.retention == Retention.LONG
    h = parse_cache_hints({"prompt_cache_key": "sess-1"})
    assert h.retention == Retention.SHORT and h.session_id == "sess-1"
    h = parse_cache_hints({"prompt_cache_retention": "24h"})
    assert h.retention == Retention.LONG
    h = parse_cache_hints({"prompt": "x"})
    assert h.retention == Retention.NONE and not h.explicit_hint_seen
    h = parse_cache_hints({"messages": [{"role": "assistant", "content": [
        {"type": "thinking", "thinking": "...", "cache_control": {"type": "ephemeral"}}]}]})
    assert h.retention == Retention.NONE


def test_kv_event_wire_roundtrip_and_client_rehash():
    toks = list(range(48))
    hs = chain_hashes(toks, 16)
    engine_hashes = [111, 222, 333]  # an engine with its own hash function
    batch = KVEventBatch(ts=1.0, events=[BlockStored(block_hashes=engine_hashes, parent_block_hash=None,
                                                     token_ids=toks, block_size=16, lora_id=None, medium="GPU")])
    raw = encode_batch(batch)
    dec = decoder_for_engine("infera-b200").decode(raw)
    client = KvEventClient(use_zmq=False)
    client.on_worker_added(W(0))
    client.feed("w0", dec.events)
    assert client.cache_view("w0") == set(hs)
    # continuation chained on an engine parent hash
    more = list(range(48, 64))
    client.feed("w0", [BlockStored(block_hashes=[444], parent_block_hash=333, token_ids=more, block_size=16,
                                   lora_id=None)])
    assert chain_hashes(toks + more, 16)[-1] in client.cache_view("w0")
    # unknown parent: dropped
    client.feed("w0", [BlockStored(block_hashes=[555], parent_block_hash=999, token_ids=more, block_size=16,
                                   lora_id=None)])
    assert client.stats["dropped_parent"] == 1
    client.feed("w0", [BlockRemoved(block_hashes=[111])])
    assert hs[0] not in client.cache_view("w0")
    client.feed("w0", [AllBlocksCleared()])
    assert not client.cache_view("w0")


def test_non_attention_groups_not_indexed():
    client = KvEventClient(use_zmq=False)
    client.on_worker_added(W(0))
    client.feed("w0", [BlockStored(block_hashes=[1], parent_block_hash=None, token_ids=list(range(16)),
                                   block_size=16, lora_id=None, kv_cache_spec_kind="mamba")])
    assert not client.cache_view("w0")


def test_protocol_resolution_and_shaping():
    p = W(0, disagg_mode=DisaggMode.PREFILL, disagg_meta={"protocol": "b200-nvlink-push", "params": {}})
    d = W(1, disagg_mode=DisaggMode.DECODE, disagg_meta={"protocol": "b200-nvlink-push", "params": {}})
    proto = resolve_protocol(p, d)
    body = {"prompt": [1, 2], "max_tokens": 10, "stream": True}
    pb = proto.annotate_prefill(body, p, d, 77)
    db = proto.annotate_decode(body, p, d, 77, None)
    assert pb["max_tokens"] == 1 and pb["stream"] is False and pb["kv_transfer_params"]["room"] == 77
    assert db["max_tokens"] == 10 and db["kv_transfer_params"]["do_remote_prefill"]
    d2 = W(2, disagg_mode=DisaggMode.DECODE, disagg_meta={"protocol": "vllm-mooncake", "params": {}})
    with pytest.raises(ProtocolError):
        resolve_protocol(p, d2)


def test_worker_pool_filters():
    pool = WorkerPool()
    pool.add(W(0))
    pool.add(W(1, disagg_mode=DisaggMode.PREFILL))
    pool.add(W(2))
    pool.set_status("w2", WorkerStatus.DRAINING)
    assert [w.worker_id for w in pool.list_active(model="m", mode=DisaggMode.MIXED)] == ["w0"]
    assert pool.models() == ["m"]
