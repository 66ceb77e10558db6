"""KV-aware routing: prefix-cache hits against load.

For each target t with the request's chained block hashes h_1..h_n::

    cost(t) = w * (n - hits(t)) + w_mm * mm_misses(t) + load(t)
    load(t) = |active blocks(t)| + recent(t)

* hits(t): length of the run h_1, h_2, ... present in t's cache view;
* active blocks: refcounted distinct hashes of t's in-flight requests;
* recent(t): a per-pick decayed (x0.97) sum of the blocks t MISSED on the
  requests it was handed (a request with no hashes is charged 1 block), so
  the load term survives traffic that never overlaps in time;
* w: the mixed / prefill / decode overlap weight, x2 for long-retention
  requests, x0.1 when the client explicitly opted out of caching, 0 for
  multimodal bodies (whose media token ids hash identically);
* image affinity: per-target LRU (256) of media keys, each miss weighted 48
  blocks;
* ties break on lower load.

Constants and semantics follow ``infera/router/policy/kv_event_aware.py:33-427``.
"""

from __future__ import annotations

import logging
from collections import OrderedDict

from infera_b200.router.cache_control import CacheHints, Retention, extract_image_keys, parse_cache_hints
from infera_b200.router.policy.base import Policy
from infera_b200.router.policy.target import RouteTarget, expand_targets

logger = logging.getLogger(__name__)

LONG_RETENTION_AMPLIFIER = 2.0
NONE_RETENTION_DAMPENER = 0.1
MM_AFFINITY_CAP = 256
MM_IMAGE_BLOCK_WEIGHT = 48.0
RECENT_DECAY = 0.97
UNKNOWN_COST_BLOCKS = 1.0


class KvAwarePolicy(Policy):
    name = "kv-aware"

    def __init__(self, kv_client, block_hasher, *, overlap_weight: float = 1.0,
                 prefill_overlap_weight: float | None = None, decode_overlap_weight: float | None = None,
                 metrics=None):
        self._kv = kv_client
        self._hasher = block_hasher
        self._w = overlap_weight
        self._wp = overlap_weight if prefill_overlap_weight is None else prefill_overlap_weight
        self._wd = overlap_weight if decode_overlap_weight is None else decode_overlap_weight
        self._active: dict[str, dict[int, int]] = {}
        self._recent: dict[str, float] = {}
        self._mm: dict[str, OrderedDict] = {}
        self.metrics = metrics

    @property
    def kv_client(self):
        return self._kv

    def _weight(self, role: str | None) -> float:
        return self._wp if role == "prefill" else self._wd if role == "decode" else self._w

    @staticmethod
    def _amplifier(h: CacheHints) -> float:
        if h.retention == Retention.LONG:
            return LONG_RETENTION_AMPLIFIER
        if h.retention == Retention.NONE and h.explicit_hint_seen:
            return NONE_RETENTION_DAMPENER
        return 1.0

    def active_blocks(self, key: str) -> int:
        return len(self._active.get(key, {}))

    def load(self, key: str) -> float:
        return self.active_blocks(key) + self._recent.get(key, 0.0)

    def _hits(self, t: RouteTarget, hashes: list[int]) -> int:
        if not hashes:
            return 0
        view = self._kv.cache_view(t.worker.worker_id, t.dp_rank)
        n = 0
        for h in hashes:
            if h not in view:
                break
            n += 1
        return n

    def _mm_hits(self, key: str, mm: list[int]) -> int:
        aff = self._mm.get(key)
        return sum(1 for k in mm if k in aff) if aff else 0

    def pick(self, candidates, request, *, role_hint=None):
        targets = expand_targets(candidates)
        if not targets:
            raise LookupError("no candidates")
        groups = {(t.worker.engine, t.worker.kv_block_size) for t in targets if t.worker.kv_block_size}
        hashes = {g: self._hasher.hash_for(request, block_size=g[1], engine=g[0]) for g in groups}
        hints = request.get("_infera_cache_hints")
        if not isinstance(hints, CacheHints):
            hints = parse_cache_hints(request)
        amp = self._weight(role_hint) * self._amplifier(hints)
        if hints.has_multimodal_content:
            w_overlap, mm = 0.0, extract_image_keys(request)
        else:
            w_overlap, mm = amp, []
        w_mm = amp * MM_IMAGE_BLOCK_WEIGHT

        def req_hashes(t):
            return hashes.get((t.worker.engine, t.worker.kv_block_size), []) if t.worker.kv_block_size else []

        scored = []
        for t in targets:
            hs = req_hashes(t)
            hits = self._hits(t, hs)
            ld = self.load(t.route_key)
            c = w_overlap * (len(hs) - hits) + w_mm * (len(mm) - self._mm_hits(t.route_key, mm)) + ld
            scored.append((c, ld, t, hits, hs))
        c, ld, picked, hits, hs = min(scored, key=lambda s: (s[0], s[1]))
        self._record_mm(picked.route_key, mm)
        self._record_dispatch(picked.route_key, len(hs) - hits, len(hs))
        if self.metrics is not None:
            self.metrics.record_pick(role_hint or "mixed", picked.route_key, hits, len(hs))
        logger.debug("pick kv-aware role=%s picked=%s hits=%d/%d load=%.1f", role_hint or "mixed",
                     picked.route_key, hits, len(hs), ld)
        return picked, list(hs)

    def _record_mm(self, key: str, mm: list[int]) -> None:
        if not mm:
            return
        aff = self._mm.setdefault(key, OrderedDict())
        for k in mm:
            aff[k] = None
            aff.move_to_end(k)
        while len(aff) > MM_AFFINITY_CAP:
            aff.popitem(last=False)

    def _record_dispatch(self, key: str, missed: int, total: int) -> None:
        for k in list(self._recent):
            v = self._recent[k] * RECENT_DECAY
            if v < 1e-3:
                del self._recent[k]
            else:
                self._recent[k] = v
        charge = UNKNOWN_COST_BLOCKS if total <= 0 else float(missed)
        if charge > 0:
            self._recent[key] = self._recent.get(key, 0.0) + charge

    def on_worker_added(self, worker) -> None:
        self._kv.on_worker_added(worker)

    def on_worker_removed(self, worker_id: str) -> None:
        self._kv.on_worker_removed(worker_id)
        pre = worker_id + "#dp"
        for d in (self._active, self._recent, self._mm):
            for k in [k for k in d if k == worker_id or k.startswith(pre)]:
                d.pop(k, None)

    def on_request_started(self, route_key, blocks=None) -> None:
        if not blocks:
            return
        refs = self._active.setdefault(route_key, {})
        for h in blocks:
            refs[h] = refs.get(h, 0) + 1
        if self.metrics is not None:
            self.metrics.set_active_blocks(route_key, len(refs))

    def on_request_finished(self, route_key, blocks=None) -> None:
        if not blocks:
            return
        refs = self._active.get(route_key)
        if refs is None:
            return
        for h in blocks:
            n = refs.get(h, 0) - 1
            if n <= 0:
                refs.pop(h, None)
            else:
                refs[h] = n
        if self.metrics is not None:
            self.metrics.set_active_blocks(route_key, len(refs))

    async def aclose(self) -> None:
        await self._kv.aclose()
