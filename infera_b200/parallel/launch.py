"""Process-group setup for one tensor-parallel group on one node.

Ranks come from the standard launcher environment (``RANK``,
``LOCAL_RANK``, ``WORLD_SIZE``, ``MASTER_ADDR``, ``MASTER_PORT``): NCCL for
the model's collectives, a gloo group for host-side control (command
broadcast, handle exchange), and the NVLink symmetric region of
:class:`~infera_b200.parallel.comm.TPComm`.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist

from infera_b200.parallel.comm import TPComm


def init_tp(tp_size: int, hidden: int | None = None, model: str | None = None, max_rows: int = 256,
            timeout_s: float = 600.0, max_rows_rs: int = 2048 + 256, first_device: int = 0):
    """Returns (TPComm, rank, device). ``hidden`` defaults from ``model``;
    steps of up to ``max_rows`` tokens use the one-shot fused all-reduce, up
    to ``max_rows_rs`` the two-shot one (at 4 or more ranks). Rank r runs on
    ``cuda:(first_device + LOCAL_RANK)``: two instances on one box (a PD
    pair on GPUs 0-3 and 4-7) both see every GPU, so that CUDA-IPC mappings
    of the other instance's caches work."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(tp_size)))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world != tp_size:
        raise ValueError(f"WORLD_SIZE={world} but tensor-parallel size {tp_size}")
    dev = torch.device("cuda", first_device + local)
    torch.cuda.set_device(dev)
    if not dist.is_initialized():
        dist.init_process_group("nccl", timeout=timedelta(seconds=timeout_s), device_id=dev)
    # followers block on the leader's broadcasts while it idles; heartbeats
    # arrive every half second, so a long timeout only bounds a dead leader
    gloo = dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))
    if hidden is None:
        from infera_b200.models.config import get_config

        hidden = get_config(model or "llama-3.1-8b").hidden
    tp = TPComm(rank, world, dev, hidden, max_rows=max_rows, nccl_group=dist.group.WORLD, gloo_group=gloo,
                max_rows_rs=max_rows_rs)
    return tp, rank, dev
