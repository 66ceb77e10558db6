"""Types of the tier-aware KV index (the ``infera_b200.kv`` package).

A cached block is identified by two hashes: ``block_hash`` (its token
content, position-independent) and ``sequence_hash`` (the chain of every
block up to and including it: what makes two prefixes equal). Tiers say
where a publisher holds the block: GPU memory, pinned host memory, local
disk (NVMe), or a shared fabric store. Role of ``infera/kv/types.py:12-160``.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass, field


class Tier(str, enum.Enum):
    DEVICE = "device"
    HOST = "host"
    DISK = "disk"
    FABRIC = "fabric"

    @property
    def rank(self) -> int:  # lower is faster
        return _TIER_RANK[self]


_TIER_RANK = {Tier.DEVICE: 0, Tier.HOST: 1, Tier.DISK: 2, Tier.FABRIC: 3}


class AttentionRole(str, enum.Enum):
    MIXED = "mixed"
    PREFILL = "prefill"
    DECODE = "decode"


@dataclass(frozen=True)
class BlockKey:
    block_hash: int
    sequence_hash: int


@dataclass
class OverlapBlocks:
    """How much of a query prefix one publisher holds, per tier: the length
    of the leading run of query blocks present in that tier or a faster one."""

    publisher: str
    by_tier: dict[Tier, int] = field(default_factory=dict)

    def best(self) -> int:
        return max(self.by_tier.values(), default=0)

    def device(self) -> int:
        return self.by_tier.get(Tier.DEVICE, 0)


@dataclass(frozen=True)
class MmRun:
    """A multimodal span of the prompt: token positions [start, start+length)
    stand for one media item whose content hash is ``media_hash``."""

    start: int
    length: int
    media_hash: int
