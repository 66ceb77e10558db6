"""A minimal NATS-protocol broker for tests (core NATS: INFO / CONNECT /
PING / SUB / UNSUB / PUB / HPUB, token wildcards ``*`` and ``>``, and the
no-responders 503 status for requests nobody subscribes to), with an
in-memory JetStream subset: streams (limits / workqueue retention, a
per-subject message limit), PubAcks, durable pull consumers (MSG.NEXT,
+ACK, pending counts), ephemeral push consumers (deliver policy all / new /
last_per_subject) and STREAM.MSG.GET by last subject - what the framework's
JetStream client uses."""

from __future__ import annotations

import asyncio
import base64
import json
import time


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
        self.streams: dict[str, dict] = {}
        self.pulls: list[dict] = []     # waiting CONSUMER.MSG.NEXT requests

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
                    if subject.startswith("$JS.API."):
                        self._js_api(subject, body[hl:] if hl else body, reply)
                        await w.drain()
                        continue
                    if subject.startswith("$JS.ACK."):
                        self._js_ack(subject)
                        continue
                    stored = self._js_store(subject, body, hl, reply)
                    targets = [x for x in self.subs if matches(x[1], subject)]
                    rp = f" {reply}" if reply else ""
                    for tw, _, sid in targets:
                        if hl is None:
                            tw.write(f"MSG {subject} {sid}{rp} {n}\r\n".encode() + body + b"\r\n")
                        else:
                            tw.write(f"HMSG {subject} {sid}{rp} {hl} {n}\r\n".encode() + body + b"\r\n")
                    if not targets and not stored and reply and opts.get("no_responders") and opts.get("headers"):
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


    # ------------------------------------------------------------------ JetStream
    def _send(self, route: str, data: bytes, headers: bytes | None = None, reply: str | None = None,
              subject: str | None = None) -> None:
        """Deliver to every subscription matching ``route``, as a message on
        ``subject`` (JetStream deliveries keep the stored message's subject)."""
        rp = f" {reply}" if reply else ""
        subject = subject or route
        for tw, _, sid in [x for x in self.subs if matches(x[1], route)]:
            if headers is None:
                tw.write(f"MSG {subject} {sid}{rp} {len(data)}\r\n".encode() + data + b"\r\n")
            else:
                tw.write(f"HMSG {subject} {sid}{rp} {len(headers)} {len(headers) + len(data)}\r\n".encode()
                         + headers + data + b"\r\n")

    def _reply(self, reply: str | None, obj: dict) -> None:
        if reply:
            self._send(reply, json.dumps(obj).encode())

    @staticmethod
    def _err(code: int, err_code: int, desc: str) -> dict:
        return {"error": {"code": code, "err_code": err_code, "description": desc}}

    def _stream_of(self, subject: str) -> dict | None:
        for st in self.streams.values():
            if any(matches(p, subject) for p in st["config"]["subjects"]):
                return st
        return None

    def _js_store(self, subject: str, body: bytes, hl: int | None, reply: str | None) -> bool:
        st = self._stream_of(subject)
        if st is None:
            return False
        hdrs = body[:hl] if hl else None
        data = body[hl:] if hl else body
        st["last_seq"] += 1
        msg = {"seq": st["last_seq"], "subject": subject, "data": data, "hdrs": hdrs, "t": time.time()}
        if st["config"].get("max_msgs_per_subject", -1) == 1:
            st["msgs"] = [m for m in st["msgs"] if m["subject"] != subject]
        st["msgs"].append(msg)
        self._reply(reply, {"stream": st["config"]["name"], "seq": msg["seq"]})
        for c in st["consumers"].values():
            if c.get("deliver_subject") and self._wants(c, msg):
                self._deliver_push(st, c, msg)
        self._serve_pulls()
        return True

    @staticmethod
    def _wants(c: dict, msg: dict) -> bool:
        f = c["config"].get("filter_subject")
        return f is None or matches(f, msg["subject"])

    def _ack_subject(self, st: dict, c: dict, msg: dict) -> str:
        c["cseq"] += 1
        return f"$JS.ACK.{st['config']['name']}.{c['name']}.1.{msg['seq']}.{c['cseq']}.{int(time.time() * 1e9)}.0"

    def _deliver_push(self, st: dict, c: dict, msg: dict) -> None:
        self._send(c["deliver_subject"], msg["data"], msg["hdrs"], self._ack_subject(st, c, msg), msg["subject"])

    def _pending(self, st: dict, c: dict) -> list[dict]:
        return [m for m in st["msgs"] if m["seq"] > c["delivered"] and self._wants(c, m)]

    def _serve_pulls(self) -> None:
        now = time.time()
        keep = []
        for pr in self.pulls:
            st = self.streams.get(pr["stream"])
            c = st["consumers"].get(pr["consumer"]) if st else None
            if c is None:
                continue
            for m in self._pending(st, c)[: pr["left"]]:
                c["delivered"] = m["seq"]
                c["ack_pending"].add(m["seq"])
                self._send(pr["reply"], m["data"], m["hdrs"], self._ack_subject(st, c, m), m["subject"])
                pr["left"] -= 1
            if pr["left"] > 0 and now < pr["deadline"]:
                keep.append(pr)
            elif pr["left"] > 0:
                self._send(pr["reply"], b"", b"NATS/1.0 408 Request Timeout\r\n\r\n")
        self.pulls = keep

    async def _expire_pulls(self) -> None:
        while self.pulls:
            await asyncio.sleep(0.02)
            self._serve_pulls()

    def _js_ack(self, subject: str) -> None:
        parts = subject.split(".")
        st = self.streams.get(parts[2])
        if st is None:
            return
        c = st["consumers"].get(parts[3])
        seq = int(parts[5])
        if c is not None:
            c["ack_pending"].discard(seq)
        if st["config"].get("retention") == "workqueue":
            st["msgs"] = [m for m in st["msgs"] if m["seq"] != seq]

    def _js_api(self, subject: str, body: bytes, reply: str | None) -> None:
        api = subject[len("$JS.API."):].split(".")
        req = json.loads(body or b"{}")
        if api[0] == "STREAM" and api[1] in ("CREATE", "UPDATE"):
            name = api[2]
            if api[1] == "CREATE" and name in self.streams:
                return self._reply(reply, self._err(400, 10058, "stream name already in use"))
            if api[1] == "UPDATE" and name not in self.streams:
                return self._reply(reply, self._err(404, 10059, "stream not found"))
            st = self.streams.setdefault(name, {"msgs": [], "last_seq": 0, "consumers": {}})
            st["config"] = req
            return self._reply(reply, {"config": req, "state": {"messages": len(st["msgs"])}})
        if api[0] == "STREAM" and api[1] == "INFO":
            st = self.streams.get(api[2])
            if st is None:
                return self._reply(reply, self._err(404, 10059, "stream not found"))
            return self._reply(reply, {"config": st["config"], "state": {"messages": len(st["msgs"]),
                                                                         "last_seq": st["last_seq"]}})
        if api[0] == "STREAM" and api[1] == "MSG" and api[2] == "GET":
            st = self.streams.get(api[3])
            subj = req.get("last_by_subj")
            found = [m for m in (st["msgs"] if st else []) if m["subject"] == subj]
            if not found:
                return self._reply(reply, self._err(404, 10037, "no message found"))
            m = found[-1]
            out = {"subject": m["subject"], "seq": m["seq"], "data": base64.b64encode(m["data"]).decode()}
            if m["hdrs"]:
                out["hdrs"] = base64.b64encode(m["hdrs"]).decode()
            return self._reply(reply, {"message": out})
        if api[0] == "CONSUMER" and api[1] == "CREATE":
            st = self.streams.get(api[2])
            if st is None:
                return self._reply(reply, self._err(404, 10059, "stream not found"))
            cfg = req.get("config", {})
            name = cfg.get("durable_name") or f"eph{len(st['consumers'])}_{int(time.time() * 1e6)}"
            c = st["consumers"].get(name)
            if c is None:
                c = {"name": name, "config": cfg, "delivered": 0, "ack_pending": set(), "cseq": 0,
                     "deliver_subject": cfg.get("deliver_subject")}
                st["consumers"][name] = c
                pol = cfg.get("deliver_policy", "all")
                if pol == "new":
                    c["delivered"] = st["last_seq"]
                if c["deliver_subject"]:
                    msgs = [m for m in st["msgs"] if self._wants(c, m)]
                    if pol == "last_per_subject":
                        last = {}
                        for m in msgs:
                            last[m["subject"]] = m
                        msgs = sorted(last.values(), key=lambda m: m["seq"])
                    elif pol == "new":
                        msgs = []
                    for m in msgs:
                        self._deliver_push(st, c, m)
            return self._reply(reply, {"name": name, "config": c["config"], "num_pending": len(self._pending(st, c))})
        if api[0] == "CONSUMER" and api[1] == "INFO":
            st = self.streams.get(api[2])
            c = st["consumers"].get(api[3]) if st else None
            if c is None:
                return self._reply(reply, self._err(404, 10014, "consumer not found"))
            return self._reply(reply, {"name": c["name"], "num_pending": len(self._pending(st, c)),
                                       "num_ack_pending": len(c["ack_pending"]),
                                       "delivered": {"stream_seq": c["delivered"]}})
        if api[0] == "CONSUMER" and api[1] == "MSG" and api[2] == "NEXT":
            expires = req.get("expires", 0) / 1e9 or 1.0
            self.pulls.append({"stream": api[3], "consumer": api[4], "reply": reply, "left": int(req.get("batch", 1)),
                               "deadline": time.time() + expires})
            self._serve_pulls()
            if self.pulls:
                asyncio.get_running_loop().create_task(self._expire_pulls())
            return None
        return self._reply(reply, self._err(400, 10003, f"unsupported API {subject}"))
