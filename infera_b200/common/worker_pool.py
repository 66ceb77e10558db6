"""Worker records and the pool the router selects from.

The registration record is a wire contract shared with every discovery
backend (etcd lease, Kubernetes Pod annotation, in-process registry), so its
field names and enum values follow the reference
(``infera/common/worker_pool.py:13-232``,
``infera/common/registration.py:22-52``). ``EngineType.INFERA_B200`` is this
framework's own engine.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Any


class WorkerStatus(str, Enum):
    ACTIVE = "active"
    DRAINING = "draining"
    DEAD = "dead"


class DisaggMode(str, Enum):
    MIXED = "mixed"
    PREFILL = "prefill"
    DECODE = "decode"


class EngineType(str, Enum):
    INFERA_B200 = "infera-b200"
    SGLANG = "sglang"
    VLLM = "vllm"
    ATOM = "atom"


@dataclass
class KvRegistrationMetadata:
    """The ``kv`` block of a registration: how the worker's cache is indexed."""

    engine_block_size: int
    index_block_size: int
    tokenizer: str
    tokenizer_digest: str
    tokenizer_canary: list[int]
    supports_events: bool = True
    event_version: int = 1
    events_endpoint: str | None = None
    snapshot_endpoint: str | None = None
    tiers: list[str] = field(default_factory=lambda: ["device"])

    _FIELDS = ("engine_block_size", "index_block_size", "tokenizer", "tokenizer_digest", "tokenizer_canary",
               "supports_events", "event_version", "events_endpoint", "snapshot_endpoint", "tiers")

    def to_dict(self) -> dict:
        d = {k: getattr(self, k) for k in self._FIELDS}
        d["tokenizer_canary"] = list(self.tokenizer_canary)
        d["tiers"] = list(self.tiers)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "KvRegistrationMetadata":
        return cls(
            engine_block_size=int(d["engine_block_size"]),
            index_block_size=int(d["index_block_size"]),
            tokenizer=str(d["tokenizer"]),
            tokenizer_digest=str(d["tokenizer_digest"]),
            tokenizer_canary=[int(x) for x in d["tokenizer_canary"]],
            supports_events=bool(d.get("supports_events", True)),
            event_version=int(d.get("event_version", 1)),
            events_endpoint=d.get("events_endpoint"),
            snapshot_endpoint=d.get("snapshot_endpoint"),
            tiers=list(d.get("tiers") or ["device"]),
        )


@dataclass
class WorkerInfo:
    worker_id: str
    url: str
    model_name: str
    engine: EngineType = EngineType.INFERA_B200
    status: WorkerStatus = WorkerStatus.ACTIVE
    disagg_mode: DisaggMode = DisaggMode.MIXED
    disagg_meta: dict[str, Any] = field(default_factory=dict)
    kv_events_endpoint: str | None = None
    kv_block_size: int | None = None
    dp_rank: int | None = None
    dp_size: int | None = None
    request_transport: str = "http"
    kv: KvRegistrationMetadata | None = None

    def to_payload(self) -> dict:
        """The registration record (no status: presence means available)."""
        out = {
            "worker_id": self.worker_id,
            "url": self.url,
            "model_name": self.model_name,
            "engine": self.engine.value,
            "disagg_mode": self.disagg_mode.value,
            "disagg_meta": dict(self.disagg_meta),
            "kv_events_endpoint": self.kv_events_endpoint,
            "kv_block_size": self.kv_block_size,
            "dp_rank": self.dp_rank,
            "dp_size": self.dp_size,
            "request_transport": self.request_transport,
        }
        if self.kv is not None:
            out["kv"] = self.kv.to_dict()
        return out

    def to_public(self) -> dict:
        """The /v1/workers view (record + status)."""
        d = self.to_payload()
        d["status"] = self.status.value
        return d


def worker_info_from_json(data: dict) -> WorkerInfo:
    """Parse a registration record; raises on malformed input."""
    kv = data.get("kv")
    return WorkerInfo(
        worker_id=str(data["worker_id"]),
        url=str(data["url"]),
        model_name=str(data["model_name"]),
        engine=EngineType(data.get("engine", EngineType.INFERA_B200.value)),
        status=WorkerStatus(data.get("status", WorkerStatus.ACTIVE.value)),
        disagg_mode=DisaggMode(data.get("disagg_mode", DisaggMode.MIXED.value)),
        disagg_meta=dict(data.get("disagg_meta") or {}),
        kv_events_endpoint=data.get("kv_events_endpoint"),
        kv_block_size=data.get("kv_block_size"),
        dp_rank=data.get("dp_rank"),
        dp_size=data.get("dp_size"),
        request_transport=data.get("request_transport", "http"),
        kv=KvRegistrationMetadata.from_dict(kv) if kv else None,
    )


class CanaryMismatch(Exception):
    def __init__(self, model_name: str, first_worker: str, new_worker: str, expected, got):
        self.model_name = model_name
        self.first_worker_id = first_worker
        self.new_worker_id = new_worker
        self.expected = tuple(expected)
        self.got = tuple(got)
        super().__init__(f"tokenizer canary mismatch for model {model_name!r}: worker {new_worker!r} produced "
                         f"{list(got)[:6]} vs first-registered worker {first_worker!r} {list(expected)[:6]}")


class CanaryVerifier:
    """First registration per model sets the tokenizer canary; later ones
    must match it, or the router's block hashes would silently miss."""

    def __init__(self) -> None:
        self._ref: dict[str, tuple[tuple[int, ...], str]] = {}

    def verify(self, *, model_name: str, worker_id: str, canary: list[int]) -> None:
        got = tuple(canary)
        have = self._ref.get(model_name)
        if have is None:
            self._ref[model_name] = (got, worker_id)
        elif have[0] != got:
            raise CanaryMismatch(model_name, have[1], worker_id, have[0], got)

    def forget(self, model_name: str) -> None:
        self._ref.pop(model_name, None)

    def reference(self, model_name: str) -> tuple[int, ...] | None:
        v = self._ref.get(model_name)
        return None if v is None else v[0]


class WorkerPool:
    """Current view of the fleet. Mutated by a registry; read by routers."""

    def __init__(self) -> None:
        self._workers: dict[str, WorkerInfo] = {}
        self.version = 0

    def add(self, worker: WorkerInfo) -> None:
        self._workers[worker.worker_id] = worker
        self.version += 1

    def remove(self, worker_id: str) -> WorkerInfo | None:
        w = self._workers.pop(worker_id, None)
        self.version += 1
        return w

    def get(self, worker_id: str) -> WorkerInfo | None:
        return self._workers.get(worker_id)

    def set_status(self, worker_id: str, status: WorkerStatus) -> bool:
        w = self._workers.get(worker_id)
        if w is None:
            return False
        w.status = status
        self.version += 1
        return True

    def all(self) -> list[WorkerInfo]:
        return list(self._workers.values())

    def list_active(self, model: str | None = None, mode: DisaggMode | None = None) -> list[WorkerInfo]:
        out = []
        for w in self._workers.values():
            if w.status != WorkerStatus.ACTIVE:
                continue
            if model and w.model_name != model:
                continue
            if mode is not None and w.disagg_mode != mode:
                continue
            out.append(w)
        return out

    def models(self) -> list[str]:
        return sorted({w.model_name for w in self._workers.values() if w.status == WorkerStatus.ACTIVE})

    def __len__(self) -> int:
        return len(self._workers)
