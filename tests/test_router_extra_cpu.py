"""More router / control-plane unit tests: routing extremes, KV-event client
bookkeeping (removal, clear, broken chains, DP-rank views), breaker
cooldown cap, registration records, KV chunk format, NATS framing."""

import pytest

from infera_b200.common.worker_pool import WorkerInfo, worker_info_from_json
from infera_b200.engine.packed_format import ChunkHeader, PackedFormatError, pack_chunk, unpack_chunk
from infera_b200.router.breaker import BreakerState, CircuitBreaker
from infera_b200.router.kv_event.block_hasher import BlockHasher
from infera_b200.router.kv_event.client import NATS_SUBJECT, KvEventClient, worker_token
from infera_b200.router.kv_event.events import AllBlocksCleared, BlockRemoved, BlockStored
from infera_b200.router.policy.kv_aware import KvAwarePolicy
from infera_b200.utils.hashing import chain_hashes


def W(i, **kw):
    return WorkerInfo(worker_id=f"w{i}", url=f"http://w{i}", model_name="m", kv_block_size=16, **kw)


def _policy(workers, w=1.0):
    client = KvEventClient(use_zmq=False)
    for x in workers:
        client.on_worker_added(x)
    return KvAwarePolicy(client, BlockHasher(), overlap_weight=w), client


def _stored(tokens, parent=None, hashes=None):
    return BlockStored(block_hashes=hashes or chain_hashes(tokens, 16), parent_block_hash=parent, token_ids=tokens,
                       block_size=16, lora_id=None)


def test_disjoint_prefixes_follow_their_holders():
    """Two prefix groups, each cached on one worker: every request goes to
    its group's holder, so the fleet splits by prefix."""
    ws = [W(0), W(1)]
    pol, client = _policy(ws)
    a, b = list(range(100, 100 + 512)), list(range(5000, 5000 + 512))
    client.feed("w0", [_stored(a)])
    client.feed("w1", [_stored(b)])
    picks = {"a": set(), "b": set()}
    for i in range(10):
        for name, pre in (("a", a), ("b", b)):
            t, _ = pol.pick(ws, {"prompt": pre + [i, i + 1]})
            picks[name].add(t.worker.worker_id)
    assert picks == {"a": {"w0"}, "b": {"w1"}}


def test_active_load_outweighs_a_small_prefix_hit():
    """A worker holding one block but carrying many active blocks loses to
    an idle worker: the cost is misses + load."""
    ws = [W(0), W(1)]
    pol, client = _policy(ws)
    p = list(range(64))
    client.feed("w0", [_stored(p[:16])])
    pol.on_request_started("w0", list(range(1000, 1100)))   # 100 active blocks
    t, _ = pol.pick(ws, {"prompt": p})
    assert t.worker.worker_id == "w1"
    pol.on_request_finished("w0", list(range(1000, 1100)))
    t, _ = pol.pick(ws, {"prompt": p})
    assert t.worker.worker_id == "w0"


def test_kv_client_remove_clear_and_broken_chain():
    client = KvEventClient(use_zmq=False)
    client.on_worker_added(W(0))
    toks = list(range(64))
    hs = chain_hashes(toks, 16)
    client.feed("w0", [_stored(toks[:32], hashes=hs[:2])])
    # continuation with the engine's parent hash
    client.feed("w0", [_stored(toks[32:], parent=hs[1], hashes=hs[2:])])
    assert len(client.cache_view("w0")) == 4
    client.feed("w0", [BlockRemoved(block_hashes=[hs[3]], medium=None)])
    assert len(client.cache_view("w0")) == 3
    # a continuation whose parent the client never saw is dropped
    client.feed("w0", [_stored(list(range(900, 916)), parent=123456789, hashes=[42])])
    assert client.stats["dropped_parent"] == 1 and len(client.cache_view("w0")) == 3
    client.feed("w0", [AllBlocksCleared()])
    assert client.cache_view("w0") == set()
    # unknown workers are ignored; removal forgets the view
    client.feed("nobody", [_stored(toks[:16])])
    client.on_worker_removed("w0")
    assert client.cache_view("w0") == set()


def test_kv_client_dp_rank_views_are_separate():
    client = KvEventClient(use_zmq=False)
    client.on_worker_added(W(0, dp_size=2))
    toks = list(range(32))
    client.feed("w0", [_stored(toks)], rank=1)
    assert len(client.cache_view("w0", 1)) == 2 and client.cache_view("w0", 0) == set()


def test_breaker_cooldown_doubles_up_to_its_cap():
    now = [0.0]
    br = CircuitBreaker(failure_threshold=1, cooldown=5.0, max_cooldown=20.0, now=lambda: now[0])
    br.record_failure("w", 500)
    t = 0.0
    for expect in (5.0, 10.0, 20.0, 20.0):   # each failed probe doubles, capped
        now[0] = t + expect - 0.05
        assert not br.allows("w")
        now[0] = t + expect + 0.05
        assert br.allows("w")
        t = now[0]
        br.record_failure("w", 502)
    br.forget("w")
    assert br.state("w") == BreakerState.CLOSED


def test_registration_record_roundtrip():
    w = W(3, dp_rank=1, dp_size=4, request_transport="bus", kv_events_endpoint="tcp://h:5557")
    back = worker_info_from_json(w.to_payload())
    for f in ("worker_id", "url", "model_name", "dp_rank", "dp_size", "request_transport", "kv_events_endpoint",
              "kv_block_size"):
        assert getattr(back, f) == getattr(w, f), f
    with pytest.raises(KeyError):
        worker_info_from_json({"url": "http://x"})


def test_worker_tokens_are_single_nats_tokens():
    assert worker_token("10.0.0.5:9000") == "10_0_0_5_9000"
    assert "." not in worker_token("a.b.c:1") and NATS_SUBJECT.endswith(".")


@pytest.mark.parametrize("channels", [1, 2])
def test_kv_chunk_roundtrip_and_corruption(channels):
    h = ChunkHeader(chunk_tokens=16, block_size=16, num_layers=3, hidden_dim=576 if channels == 1 else 256,
                    dtype="bf16", num_kv_channels=channels)
    payload = bytes(range(256)) * (h.payload_bytes // 256) + bytes(h.payload_bytes % 256)
    blob = pack_chunk(h, payload)
    h2, body = unpack_chunk(blob)
    assert h2.num_kv_channels == channels and bytes(body) == payload
    assert h2.payload_byte_offset % 4096 == 0
    with pytest.raises(PackedFormatError):
        unpack_chunk(blob[: len(blob) - 7])   # truncated payload


def test_nats_header_block_roundtrip():
    from infera_b200.common.nats_wire import encode_headers, parse_headers

    hb = encode_headers({"rs-type": "data", "rs-status": "200", "rid": "abc"})
    assert hb.startswith(b"NATS/1.0\r\n") and hb.endswith(b"\r\n\r\n")
    assert parse_headers(hb) == {"rs-type": "data", "rs-status": "200", "rid": "abc"}
    assert parse_headers(b"NATS/1.0 408 Request Timeout\r\n\r\n") == {"status": "408"}
