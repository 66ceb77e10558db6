"""File-descriptor passing over Unix sockets (SCM_RIGHTS), sync and asyncio
(``infera/kvd/fd_passing.py:63-287`` offers the same primitives)."""

from __future__ import annotations

import asyncio
import socket


def send_fd(sock: socket.socket, fd: int, tag: bytes = b"F") -> None:
    socket.send_fds(sock, [tag], [fd])


def recv_fd(sock: socket.socket) -> int:
    _msg, fds, _flags, _addr = socket.recv_fds(sock, 16, 1)
    if not fds:
        raise ConnectionError("peer sent no file descriptor")
    return fds[0]


async def async_send_fd(writer: asyncio.StreamWriter, fd: int) -> None:
    await writer.drain()
    sock = writer.get_extra_info("socket")
    loop = asyncio.get_running_loop()
    raw = socket.socket(fileno=sock.fileno(), family=socket.AF_UNIX, type=socket.SOCK_STREAM)
    try:
        await loop.run_in_executor(None, lambda: socket.send_fds(raw, [b"F"], [fd]))
    finally:
        raw.detach()
