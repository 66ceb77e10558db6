"""Per-worker circuit breaker fed by dispatch outcomes.

States closed -> open -> half-open -> closed:

* ``failure_threshold`` (3) consecutive worker faults open the breaker for a
  cooldown (5 s), which doubles on every failed half-open probe up to
  ``max_cooldown`` (60 s) and resets on success;
* once the cooldown passes the worker is half-open: exactly one probe is let
  through; a probe slot unreported for ``probe_timeout`` (60 s) is reclaimed;
* only 5xx and transport errors (status 0) count as worker faults; 4xx and
  429 say nothing about the worker's health;
* if every candidate is open the filter returns them all: routing somewhere
  beats refusing everything;
* a threshold <= 0 disables the breaker.

Semantics of ``infera/router/breaker.py:69-304``. Single-threaded by design
(driven from one asyncio loop).
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from enum import Enum
from typing import Callable


def is_worker_fault(status: int) -> bool:
    return status >= 500 or status == 0


class BreakerState(str, Enum):
    CLOSED = "closed"
    OPEN = "open"
    HALF_OPEN = "half_open"


STATE_VALUE = {"closed": 0, "half_open": 1, "open": 2}


@dataclass
class _Entry:
    failures: int = 0
    state: BreakerState = BreakerState.CLOSED
    open_until: float = 0.0
    next_cooldown: float = 0.0
    probe_at: float | None = None
    trips: int = 0


@dataclass
class CircuitBreaker:
    failure_threshold: int = 3
    cooldown: float = 5.0
    max_cooldown: float = 60.0
    probe_timeout: float = 60.0
    now: Callable[[], float] = time.monotonic
    on_change: Callable[[str, BreakerState, bool], None] | None = None
    _e: dict[str, _Entry] = field(default_factory=dict, init=False)

    @property
    def enabled(self) -> bool:
        return self.failure_threshold > 0

    def _entry(self, wid: str) -> _Entry:
        e = self._e.get(wid)
        if e is None:
            e = _Entry(next_cooldown=self.cooldown)
            self._e[wid] = e
        return e

    def _set(self, wid: str, e: _Entry, st: BreakerState, tripped: bool = False) -> None:
        if e.state != st or tripped:
            e.state = st
            if self.on_change is not None:
                try:
                    self.on_change(wid, st, tripped)
                except Exception:
                    pass

    def state(self, wid: str) -> BreakerState:
        e = self._e.get(wid)
        if e is None:
            return BreakerState.CLOSED
        if e.state == BreakerState.OPEN and self.now() >= e.open_until:
            return BreakerState.HALF_OPEN
        return e.state

    def allows(self, wid: str) -> bool:
        """May a request go to ``wid`` now? Claims the half-open probe slot."""
        if not self.enabled:
            return True
        e = self._e.get(wid)
        if e is None or e.state == BreakerState.CLOSED:
            return True
        t = self.now()
        if e.state == BreakerState.OPEN:
            if t < e.open_until:
                return False
            self._set(wid, e, BreakerState.HALF_OPEN)
        if e.probe_at is not None and t - e.probe_at < self.probe_timeout:
            return False
        e.probe_at = t
        return True

    def filter(self, workers: list) -> list:
        if not self.enabled or not workers:
            return list(workers)
        ok = [w for w in workers if self.allows(w.worker_id)]
        return ok if ok else list(workers)

    def record_success(self, wid: str) -> None:
        if not self.enabled:
            return
        e = self._entry(wid)
        e.failures = 0
        e.probe_at = None
        e.next_cooldown = self.cooldown
        self._set(wid, e, BreakerState.CLOSED)

    def record_failure(self, wid: str, status: int = 0) -> None:
        if not self.enabled or not is_worker_fault(status):
            if self.enabled:
                # neutral outcome: frees a probe slot without judging
                e = self._e.get(wid)
                if e is not None:
                    e.probe_at = None
            return
        e = self._entry(wid)
        t = self.now()
        if e.state in (BreakerState.HALF_OPEN, BreakerState.OPEN) and (e.state == BreakerState.HALF_OPEN
                                                                     or t >= e.open_until):
            # failed probe: reopen with a doubled cooldown
            e.next_cooldown = min(self.max_cooldown, e.next_cooldown * 2)
            e.open_until = t + e.next_cooldown
            e.probe_at = None
            e.trips += 1
            self._set(wid, e, BreakerState.OPEN, tripped=True)
            return
        e.failures += 1
        if e.state == BreakerState.CLOSED and e.failures >= self.failure_threshold:
            e.open_until = t + e.next_cooldown
            e.trips += 1
            self._set(wid, e, BreakerState.OPEN, tripped=True)

    def record_outcome(self, wid: str, status: int) -> None:
        if 200 <= status < 400:
            self.record_success(wid)
        else:
            self.record_failure(wid, status)

    def forget(self, wid: str) -> None:
        self._e.pop(wid, None)

    def snapshot(self) -> dict[str, dict]:
        return {w: {"state": self.state(w).value, "failures": e.failures, "trips": e.trips}
                for w, e in self._e.items()}
