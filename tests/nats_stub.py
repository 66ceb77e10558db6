"""A minimal NATS-protocol broker for tests (core NATS: INFO / CONNECT /
PING / SUB / UNSUB / PUB / HPUB, token wildcards ``*`` and ``>``, and the
no-responders 503 status for requests nobody subscribes to)."""

from __future__ import annotations

import asyncio
import json


def matches(pattern: str, subject: str) -> bool:
    p, s = pattern.split("."), subject.split(".")
    for i, tok in enumerate(p):
        if tok == ">":
            return len(s) > i
        if i >= len(s) or (tok != "*" and tok != s[i]):
            return False
    return len(p) == len(s)


class Broker:
    def __init__(self):
        self.subs: list[tuple[object, str, int]] = []   # (connection writer, subject, sid)
        self.server = None
        self.port = 0
        self.published = 0
        self.writers: set = set()

    async def start(self) -> "Broker":
        self.server = await asyncio.start_server(self._conn, "127.0.0.1", 0)
        self.port = self.server.sockets[0].getsockname()[1]
        return self

    def kick(self) -> None:
        """Close every client connection (a broker that went away)."""
        for w in list(self.writers):
            w.close()

    async def stop(self) -> None:
        self.server.close()
        await self.server.wait_closed()

    async def _conn(self, r: asyncio.StreamReader, w: asyncio.StreamWriter) -> None:
        self.writers.add(w)
        w.write(b'INFO {"server_id":"stub","version":"2.10.0","headers":true,"max_payload":1048576}\r\n')
        opts = {}
        try:
            while True:
                line = await r.readline()
                if not line:
                    break
                op, _, rest = line.rstrip(b"\r\n").partition(b" ")
                op = op.upper()
                if op == b"CONNECT":
                    opts = json.loads(rest)
                elif op == b"PING":
                    w.write(b"PONG\r\n")
                elif op == b"SUB":
                    parts = rest.decode().split()
                    self.subs.append((w, parts[0], int(parts[-1])))
                elif op == b"UNSUB":
                    sid = int(rest.decode().split()[0])
                    self.subs = [x for x in self.subs if not (x[0] is w and x[2] == sid)]
                elif op in (b"PUB", b"HPUB"):
                    parts = rest.decode().split()
                    subject = parts[0]
                    if op == b"PUB":
                        n = int(parts[-1])
                        reply = parts[1] if len(parts) == 3 else None
                        body = (await r.readexactly(n + 2))[:n]
                        hl = None
                    else:
                        hl, n = int(parts[-2]), int(parts[-1])
                        reply = parts[1] if len(parts) == 4 else None
                        body = (await r.readexactly(n + 2))[:n]
                    self.published += 1
                    targets = [x for x in self.subs if matches(x[1], subject)]
                    rp = f" {reply}" if reply else ""
                    for tw, _, sid in targets:
                        if hl is None:
                            tw.write(f"MSG {subject} {sid}{rp} {n}\r\n".encode() + body + b"\r\n")
                        else:
                            tw.write(f"HMSG {subject} {sid}{rp} {hl} {n}\r\n".encode() + body + b"\r\n")
                    if not targets and reply and opts.get("no_responders") and opts.get("headers"):
                        hb = b"NATS/1.0 503\r\n\r\n"
                        for tw, pat, sid in [x for x in self.subs if matches(x[1], reply)]:
                            tw.write(f"HMSG {reply} {sid} {len(hb)} {len(hb)}\r\n".encode() + hb + b"\r\n")
                await w.drain()
        except (asyncio.IncompleteReadError, ConnectionError):
            pass
        finally:
            self.subs = [x for x in self.subs if x[0] is not w]
            self.writers.discard(w)
            w.close()
