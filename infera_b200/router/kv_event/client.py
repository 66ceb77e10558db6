"""Router-side mirror of every worker's prefix cache, fed by KV events.

For each worker (and each DP rank of a rank-multiplexed worker) the client
keeps the set of ROUTER block hashes it holds. Engine events are re-hashed
from their ``token_ids`` with the router's chain, so any engine's own hash
function works: an engine-hash -> router-hash map resolves parents and
removals. A stored event whose parent is unknown is dropped (chain broken:
a later query can only miss by that block). Only attention KV groups are
indexed (``kv_cache_spec_kind`` absent, ``full_attention``,
``mla_attention`` or ``sink_full_attention``). Behaviour of
``infera/router/kv_event/client.py:104-350``.

Transports: ZMQ SUB per worker endpoint (per DP rank: port + rank), one
NATS subscription to ``infera.kv.events.>`` (:meth:`attach_nats`; workers'
relays republish their batches on ``infera.kv.events.<worker token>``), or
:meth:`feed` for in-process publishers.
"""

from __future__ import annotations

import asyncio
import logging
from dataclasses import dataclass, field

from infera_b200.router.kv_event.events import CLEARED, REMOVED, STORED, decoder_for_engine
from infera_b200.utils.hashing import ROUTER_SEED, chain_hashes

logger = logging.getLogger(__name__)

TOPIC = b"kv-events"
NATS_SUBJECT = "infera.kv.events."


def worker_token(worker_id: str) -> str:
    """A worker id as one NATS subject token (the bus transport's form)."""
    return str(worker_id).replace(".", "_").replace(":", "_")
INDEXABLE = frozenset({"full_attention", "mla_attention", "sink_full_attention"})
MAX_BACKOFF = 5.0


@dataclass
class WorkerView:
    worker_id: str
    block_size: int
    engine: str = "infera-b200"
    views: dict[int | None, set[int]] = field(default_factory=dict)
    maps: dict[int | None, dict] = field(default_factory=dict)
    tasks: list = field(default_factory=list)
    mismatch_logged: bool = False

    def view(self, rank: int | None) -> set[int]:
        return self.views.setdefault(rank, set())

    def hmap(self, rank: int | None) -> dict:
        return self.maps.setdefault(rank, {})


def rank_endpoints(endpoint: str, dp_size: int | None) -> list[tuple[int | None, str]]:
    """``tcp://h:p`` -> one endpoint per DP rank at port p + rank."""
    if not dp_size or dp_size <= 1:
        return [(None, endpoint)]
    head, _, port = endpoint.rpartition(":")
    return [(r, f"{head}:{int(port) + r}") for r in range(dp_size)]


class KvEventClient:
    def __init__(self, use_zmq: bool = True):
        self.workers: dict[str, WorkerView] = {}
        self.use_zmq = use_zmq
        self._ctx = None
        self.stats = {"stored": 0, "removed": 0, "dropped_parent": 0, "decode_errors": 0}

    # ------------------------------------------------------------------ fleet
    def on_worker_added(self, worker) -> None:
        bs = worker.kv_block_size or (worker.kv.index_block_size if worker.kv else None)
        if not bs:
            return
        wv = WorkerView(worker.worker_id, int(bs), getattr(worker.engine, "value", str(worker.engine)))
        old = self.workers.pop(worker.worker_id, None)
        if old is not None:
            self._cancel(old)
        self.workers[worker.worker_id] = wv
        if self.use_zmq and worker.kv_events_endpoint:
            try:
                loop = asyncio.get_running_loop()
            except RuntimeError:
                return
            for rank, ep in rank_endpoints(worker.kv_events_endpoint, worker.dp_size):
                wv.tasks.append(loop.create_task(self._subscribe(wv, rank, ep)))

    def on_worker_removed(self, worker_id: str) -> None:
        wv = self.workers.pop(worker_id, None)
        if wv is not None:
            self._cancel(wv)

    def _cancel(self, wv: WorkerView) -> None:
        for t in wv.tasks:
            t.cancel()
        wv.tasks.clear()

    def cache_view(self, worker_id: str, dp_rank: int | None = None) -> set[int]:
        wv = self.workers.get(worker_id)
        if wv is None:
            return set()
        return wv.views.get(dp_rank, set())

    # ------------------------------------------------------------------ events
    def feed(self, worker_id: str, events, rank: int | None = None) -> None:
        wv = self.workers.get(worker_id)
        if wv is None:
            return
        for ev in events:
            self._handle(wv, ev, rank)

    def _handle(self, wv: WorkerView, ev, rank) -> None:
        if isinstance(ev, STORED):
            self._stored(wv, ev, rank)
        elif isinstance(ev, REMOVED):
            view, m = wv.view(rank), wv.hmap(rank)
            for h in ev.block_hashes:
                rh = m.pop(h, None)
                if rh is not None:
                    view.discard(rh)
                    self.stats["removed"] += 1
        elif isinstance(ev, CLEARED):
            wv.view(rank).clear()
            wv.hmap(rank).clear()

    def _stored(self, wv: WorkerView, ev, rank) -> None:
        kind = getattr(ev, "kv_cache_spec_kind", None)
        if kind is not None and kind not in INDEXABLE:
            return
        view, m = wv.view(rank), wv.hmap(rank)
        if ev.parent_block_hash is None:
            parent = ROUTER_SEED
        else:
            parent = m.get(ev.parent_block_hash)
            if parent is None:
                self.stats["dropped_parent"] += 1
                return
        if ev.block_size and ev.block_size != wv.block_size and not wv.mismatch_logged:
            wv.mismatch_logged = True
            logger.error("kv events from %s use block_size=%d but it registered %d; its view cannot match",
                         wv.worker_id, ev.block_size, wv.block_size)
        tokens = list(ev.token_ids)
        rhs = chain_hashes(tokens, wv.block_size, parent)
        for rh in rhs:
            view.add(rh)
        self.stats["stored"] += len(rhs)
        if len(rhs) == len(ev.block_hashes):
            for eh, rh in zip(ev.block_hashes, rhs):
                m[eh] = rh

    # ------------------------------------------------------------------ ZMQ
    async def _subscribe(self, wv: WorkerView, rank, endpoint: str) -> None:
        import zmq
        import zmq.asyncio

        if self._ctx is None:
            self._ctx = zmq.asyncio.Context.instance()
        dec = decoder_for_engine(wv.engine)
        backoff = 0.25
        while True:
            sock = self._ctx.socket(zmq.SUB)
            try:
                sock.connect(endpoint)
                sock.subscribe(TOPIC)
                while True:
                    frames = await sock.recv_multipart()
                    try:
                        batch = dec.decode(frames[-1])
                    except Exception as e:
                        self.stats["decode_errors"] += 1
                        logger.warning("kv decode failed for %s: %s", wv.worker_id, e)
                        continue
                    r = batch.attn_dp_rank if batch.attn_dp_rank is not None else rank
                    for ev in batch.events:
                        self._handle(wv, ev, r)
            except asyncio.CancelledError:
                raise
            except Exception as e:
                logger.warning("kv subscriber %s failed (%s); retrying", wv.worker_id, e)
                await asyncio.sleep(backoff)
                backoff = min(backoff * 2, MAX_BACKOFF)
            finally:
                sock.close(linger=0)

    # ------------------------------------------------------------------ NATS
    async def attach_nats(self, bus, jetstream: bool = False) -> None:
        """Receive every worker's KV-event batches from the bus (subject
        ``infera.kv.events.<worker token>``). With ``jetstream``: first the
        workers' views from the ``INFERA_KV_VIEWS`` bucket (the latest value
        per worker, and every refresh after it: bootstrap and self-heal),
        then new batches from the ``INFERA_KV_EVENTS`` stream."""

        def by_token(token: str):
            return next((w for w in self.workers.values() if worker_token(w.worker_id) == token), None)

        async def on_batch(m) -> None:
            token = m.subject[len(NATS_SUBJECT):]
            wv = next((w for w in self.workers.values() if worker_token(w.worker_id) == token), None)
            if wv is None:
                return
            try:
                batch = decoder_for_engine(wv.engine).decode(m.data)
            except Exception as e:
                self.stats["decode_errors"] += 1
                logger.warning("kv decode failed for %s: %s", wv.worker_id, e)
                return
            for ev in batch.events:
                self._handle(wv, ev, batch.attn_dp_rank)

        if not jetstream:
            self._nats_unsub = await bus.subscribe(NATS_SUBJECT + ">", on_batch)
            return
        from infera_b200.common.jetstream import JetStream
        from infera_b200.kv.nats_relay import KV_STREAM, VIEW_BUCKET, decode_view

        js = JetStream(bus)
        await js.add_stream(KV_STREAM, [NATS_SUBJECT + ">"], max_age_s=600.0)
        kv = await js.key_value(VIEW_BUCKET)

        async def on_view(token: str, value: bytes | None) -> None:
            wv = by_token(token)
            if wv is None or value is None:
                return
            try:
                ranks = decode_view(value)
            except Exception:
                self.stats["decode_errors"] += 1
                return
            for r, (view, hmap) in ranks.items():
                wv.views[r] = view
                wv.maps[r] = hmap
            self.stats["bootstraps"] = self.stats.get("bootstraps", 0) + 1

        self._view_unsub = await kv.watch(on_view)
        self._nats_unsub = await js.subscribe_push(KV_STREAM, on_batch, filter_subject=NATS_SUBJECT + ">",
                                                   deliver_policy="new")

    async def aclose(self) -> None:
        for wv in self.workers.values():
            self._cancel(wv)
        if getattr(self, "_nats_unsub", None) is not None:
            self._nats_unsub()
        if getattr(self, "_view_unsub", None) is not None:
            self._view_unsub()
