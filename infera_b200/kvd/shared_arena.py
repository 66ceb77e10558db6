"""Shared-memory arena: the pinned host-DRAM tier shared between the kvd
daemon and engine processes.

A ``memfd`` is split into fixed-size slots. Each slot starts with a 16-byte
header ``[u64 version][u32 size][u32 reserved]`` followed by the payload.
Writers use a seqlock: bump the version to odd, write the payload and size,
bump it to even. Readers copy the payload between two version reads and
retry when the version was odd or changed, so a reader never returns a torn
value (``infera/kvd/shared_arena.py:193-1201`` uses the same slot protocol).

The fd is handed to clients over the daemon's Unix socket (SCM_RIGHTS); an
engine on a GPU registers its mapping with ``cudaHostRegister``
(:meth:`ArenaView.register_cuda`), so the tier's promotes copy a page
straight from the arena into device memory (a DMA transfer, no host-side
copy) and validate the slot's version after the copy landed.
"""

from __future__ import annotations

import mmap
import os
import struct
import threading

HEADER = 16
_HDR = struct.Struct("<QII")


class SharedArena:
    def __init__(self, num_slots: int, slot_size: int, *, fd: int | None = None, name: str = "infera-kvd-arena"):
        if slot_size <= HEADER:
            raise ValueError("slot too small")
        self.num_slots = num_slots
        self.slot_size = slot_size
        self.size = num_slots * slot_size
        self.owner = fd is None
        if fd is None:
            fd = os.memfd_create(name, 0)
            os.ftruncate(fd, self.size)
        self.fd = fd
        self.mm = mmap.mmap(fd, self.size, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)
        self.view = memoryview(self.mm)
        self._free = list(range(num_slots - 1, -1, -1))
        self._lock = threading.Lock()

    # ------------------------------------------------------------------ slots
    def alloc(self) -> int | None:
        with self._lock:
            return self._free.pop() if self._free else None

    def free(self, slot: int) -> None:
        with self._lock:
            self._free.append(slot)

    def free_slots(self) -> int:
        return len(self._free)

    def payload_offset(self, slot: int) -> int:
        return slot * self.slot_size + HEADER

    @property
    def payload_max(self) -> int:
        return self.slot_size - HEADER

    # ------------------------------------------------------------------ seqlock
    def write(self, slot: int, data) -> int:
        """Write ``data`` into ``slot``; returns the new (even) version."""
        n = len(data)
        if n > self.payload_max:
            raise ValueError(f"value of {n} bytes exceeds slot payload {self.payload_max}")
        base = slot * self.slot_size
        ver, _, _ = _HDR.unpack_from(self.mm, base)
        odd = ver + 1 if ver % 2 == 0 else ver + 2
        _HDR.pack_into(self.mm, base, odd, 0, 0)
        self.view[base + HEADER: base + HEADER + n] = data
        _HDR.pack_into(self.mm, base, odd + 1, n, 0)
        return odd + 1

    def begin_write(self, slot: int) -> int:
        """Mark a slot as being written in place (zero-copy save lease)."""
        base = slot * self.slot_size
        ver, _, _ = _HDR.unpack_from(self.mm, base)
        odd = ver + 1 if ver % 2 == 0 else ver
        _HDR.pack_into(self.mm, base, odd, 0, 0)
        return odd

    def end_write(self, slot: int, size: int) -> int:
        base = slot * self.slot_size
        ver, _, _ = _HDR.unpack_from(self.mm, base)
        _HDR.pack_into(self.mm, base, ver + 1, size, 0)
        return ver + 1

    def version(self, slot: int) -> int:
        return _HDR.unpack_from(self.mm, slot * self.slot_size)[0]

    def close(self) -> None:
        try:
            self.view.release()
            self.mm.close()
        finally:
            if self.owner:
                os.close(self.fd)


class ArenaView:
    """Client-side read-only view of an arena received over SCM_RIGHTS."""

    def __init__(self, fd: int, size: int, slot_size: int):
        self.fd = fd
        self.size = size
        self.slot_size = slot_size
        self.mm = mmap.mmap(fd, size, mmap.MAP_SHARED, mmap.PROT_READ | mmap.PROT_WRITE)

    def read(self, payload_offset: int, expect_version: int | None = None, retries: int = 64) -> bytes | None:
        """Seqlock read of the slot whose payload starts at ``payload_offset``.
        Returns None when the slot was rewritten (version moved on)."""
        base = payload_offset - HEADER
        for _ in range(retries):
            v1, n, _ = _HDR.unpack_from(self.mm, base)
            if v1 % 2:
                continue
            if expect_version is not None and v1 != expect_version:
                return None
            data = self.mm[payload_offset: payload_offset + n]
            v2 = _HDR.unpack_from(self.mm, base)[0]
            if v1 == v2:
                return data
        return None

    def version_at(self, payload_offset: int) -> int:
        return _HDR.unpack_from(self.mm, payload_offset - HEADER)[0]

    def register_cuda(self):
        """Page-lock the mapping for the CUDA device copies (cudaHostRegister)
        and return a uint8 CPU tensor over it (torch reports it pinned, so
        ``copy_(..., non_blocking=True)`` from its slices is a DMA transfer).
        Returns None when no GPU is usable."""
        try:
            import ctypes

            import torch

            if not torch.cuda.is_available():
                return None
            addr = ctypes.addressof(ctypes.c_char.from_buffer(self.mm))
            rc = torch.cuda.cudart().cudaHostRegister(addr, self.size, 0)
            if int(rc) != 0:
                return None
            self._registered = addr
            return torch.frombuffer(self.mm, dtype=torch.uint8)
        except Exception:
            return None

    def write_payload(self, payload_offset: int, data) -> None:
        """Fill a slot leased by SET_RESERVE (the daemon owns the seqlock)."""
        self.mm[payload_offset: payload_offset + len(data)] = data

    def close(self) -> None:
        if getattr(self, "_registered", None) is not None:
            try:
                import torch

                torch.cuda.cudart().cudaHostUnregister(self._registered)
            except Exception:
                pass
            self._registered = None
        self.mm.close()
        os.close(self.fd)
