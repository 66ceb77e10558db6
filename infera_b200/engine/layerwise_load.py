"""Layer-by-layer loading of tiered KV into the paged cache.

A chunk promoted from host or NVMe must reach the device before attention
reads it, but only layer by layer: layer ``l``'s pages can be copied while
layers ``< l`` compute. The loader owns a side copy stream and a pool of
pinned host staging buffers; ``load(chunk)`` issues one host->device copy
per layer on the side stream and records an event per (chunk, layer);
``wait_layer(l)`` makes the compute stream wait for every pending chunk's
layer ``l`` only. Buffers return to the pool once their last copy is done.
Role of ``infera/engine/vllm/layerwise_load_helper.py:45-253`` (which is a
draft there too; this one is exercised by its test but the engine's
forward does not call ``wait_layer`` yet).
"""

from __future__ import annotations

from collections import deque

import torch


class LayerwiseLoader:
    def __init__(self, num_layers: int, buf_bytes: int, pool_size: int = 4, device: str | torch.device = "cuda"):
        self.num_layers = num_layers
        self.device = torch.device(device)
        self.on_gpu = self.device.type == "cuda"
        pin = self.on_gpu
        self.free = deque(torch.empty(buf_bytes, dtype=torch.uint8, pin_memory=pin) for _ in range(pool_size))
        self.stream = torch.cuda.Stream(self.device) if self.on_gpu else None
        self.pending: list[tuple[list, torch.Tensor]] = []   # (per-layer events, staging buffer)

    def staging(self) -> torch.Tensor:
        self._recycle()
        if not self.free:
            raise RuntimeError("no free staging buffer (raise pool_size)")
        return self.free.popleft()

    def load(self, staging: torch.Tensor, layer_dsts: list[torch.Tensor], layer_bytes: int) -> None:
        """``staging`` holds ``num_layers`` consecutive slices of
        ``layer_bytes``; slice l goes to ``layer_dsts[l]`` (uint8 views)."""
        evs = []
        for li, dst in enumerate(layer_dsts):
            src = staging[li * layer_bytes:(li + 1) * layer_bytes]
            if self.on_gpu:
                with torch.cuda.stream(self.stream):
                    dst.copy_(src, non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
                evs.append(ev)
            else:
                dst.copy_(src)
                evs.append(None)
        self.pending.append((evs, staging))

    def wait_layer(self, layer: int, stream=None) -> None:
        if not self.on_gpu:
            return
        s = stream or torch.cuda.current_stream(self.device)
        for evs, _ in self.pending:
            if layer < len(evs):
                s.wait_event(evs[layer])

    def _recycle(self) -> None:
        keep = []
        for evs, buf in self.pending:
            if all(e is None or e.query() for e in evs):
                self.free.append(buf)
            else:
                keep.append((evs, buf))
        self.pending = keep

    def synchronize(self) -> None:
        if self.on_gpu:
            self.stream.synchronize()
        self._recycle()
