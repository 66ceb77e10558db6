"""Request state inside the engine."""

from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field

from infera_b200.engine.block_manager import SeqBlocks


@dataclass
class SamplingParams:
    max_tokens: int = 256
    temperature: float = 0.0
    seed: int | None = None
    stop_token_ids: list[int] = field(default_factory=list)
    ignore_eos: bool = False
    min_tokens: int = 0
    # retention hint from the router (none / ephemeral / short / long); the
    # engine uses it to order prefix-cache eviction and tier spills
    retention: str | None = None
    # prefill/decode disaggregation parameters from the router
    # (kv_transfer_params of the b200-nvlink-push protocol)
    kv_transfer: dict | None = None


class Status(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED_STOPPED = "stop"
    FINISHED_LENGTH = "length"
    FINISHED_ABORTED = "abort"

    @property
    def finished(self) -> bool:
        return self in (Status.FINISHED_STOPPED, Status.FINISHED_LENGTH, Status.FINISHED_ABORTED)


@dataclass
class Request:
    request_id: str
    prompt_token_ids: list[int]
    sampling: SamplingParams
    arrival_time: float = field(default_factory=time.monotonic)
    eos_token_id: int | None = None
    output_token_ids: list[int] = field(default_factory=list)
    status: Status = Status.WAITING
    blocks: SeqBlocks | None = None
    num_computed: int = 0          # tokens whose K/V is in the cache
    table_row: int = -1            # row of the device block table owned while running
    pages_synced: int = 0          # pages already written to the device block table
    prompt_hashes: list[int] | None = None
    num_preemptions: int = 0
    # timing (engine clock)
    first_token_time: float | None = None
    token_times: list[float] = field(default_factory=list)
    finish_time: float | None = None
    num_cached_prompt_tokens: int = 0
    # PD: decode side waits for room ``remote_room``'s pushed KV; prefill side
    # pushes to (room, decode endpoint) once its prompt is computed
    remote_room: int | None = None
    remote_decode: tuple | None = None
    # KV tiers: first page of the prefix an asynchronous promote fills
    tier_start: int = 0

    @property
    def num_tokens(self) -> int:
        return len(self.prompt_token_ids) + len(self.output_token_ids)

    def all_token_ids(self) -> list[int]:
        if not self.output_token_ids:
            return self.prompt_token_ids
        return self.prompt_token_ids + self.output_token_ids

    def token_at(self, i: int) -> int:
        n = len(self.prompt_token_ids)
        return self.prompt_token_ids[i] if i < n else self.output_token_ids[i - n]

    def tokens_range(self, a: int, b: int) -> list[int]:
        n = len(self.prompt_token_ids)
        if b <= n:
            return self.prompt_token_ids[a:b]
        if a >= n:
            return self.output_token_ids[a - n:b - n]
        return self.prompt_token_ids[a:] + self.output_token_ids[: b - n]

    def check_stop(self) -> Status | None:
        if not self.output_token_ids:
            return None
        n = len(self.output_token_ids)
        last = self.output_token_ids[-1]
        if n >= self.sampling.min_tokens:
            if not self.sampling.ignore_eos and self.eos_token_id is not None and last == self.eos_token_id:
                return Status.FINISHED_STOPPED
            if last in self.sampling.stop_token_ids:
                return Status.FINISHED_STOPPED
        if n >= self.sampling.max_tokens:
            return Status.FINISHED_LENGTH
        return None


@dataclass
class RequestOutput:
    request_id: str
    new_token_ids: list[int]
    finished: bool
    finish_reason: str | None = None
    num_prompt_tokens: int = 0
    num_cached_tokens: int = 0
    num_output_tokens: int = 0
