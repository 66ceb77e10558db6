"""Prefill/decode disaggregation between two engine instances: the
``b200-nvlink-push`` protocol, engine side.

The router sends the same request to a prefill instance (one output token,
``kv_transfer_params = {do_remote_decode, room, decode_kv_endpoint}``) and
to a decode instance (the remaining tokens, ``{do_remote_prefill, room}``).

Decode instance (:class:`PDRendezvous`): on admission of a remote-prefill
request it allocates KV pages for the prompt minus its last token (reusing
any prefix it already caches), parks the request, and publishes
``room -> (page ids beyond the cached prefix, number of cached tokens)``.
It serves, on its KV endpoint (ZMQ REP, msgpack):

    {"op": "describe"} -> CUDA-IPC handles (+ offsets) of its K / V caches,
                          slots per layer, layers, pid, device
    {"op": "pages", "room"} -> {"ready", "pages", "skip_tokens", "n_tokens"}
    {"op": "done", "room", "ok"} -> ack; the parked request resumes with the
                          pushed tokens counted as computed (or, if not ok,
                          computes its prompt itself)

Prefill instance (:class:`PDPushAgent`): when a remote-decode request has
computed its prompt, its pages are held (not freed) until the push ends;
between engine steps the agent gets the room's page list, maps the decode
caches once per endpoint (CUDA IPC; plain pointers when both instances
live in one process), and the engine launches ``ib_kv_push_pages`` on its
stream (peer stores over NVLink); when the copy's event completes it sends
``done`` and releases the pages. A room that never becomes ready within
``timeout_s`` is dropped (the decode side times out too and recomputes).

Layer by layer: the agent starts resolving a room's page list when the
request is admitted (``prefetch``). If the list is known when the step that
completes the prompt is scheduled, that step's forward pushes each layer's
pages right after the layer's KV write, on a side stream that waits only
for that layer (:class:`LayerPush`): the transfer overlaps the remaining
layers' compute instead of following the whole prefill. Otherwise the push
runs after the prompt as above.

Protocol role of ``infera/router/disagg_protocols`` + the engines' KV
connectors (Mooncake / MoRI / NIXL in the reference); the transport here is
this framework's own NVLink page push.
"""

from __future__ import annotations

import logging
import os
import threading
import time
from dataclasses import dataclass, field

import msgpack
import torch

logger = logging.getLogger(__name__)

# endpoint -> decode engine, for instances sharing one process (tests, 1-GPU demos)
_LOCAL: dict[str, object] = {}


def _pack(o) -> bytes:
    return msgpack.packb(o, use_bin_type=True)


def _unpack(b: bytes):
    return msgpack.unpackb(b, raw=False)


def _ipc_handle(t: torch.Tensor) -> tuple[bytes, int]:
    """(cudaIpcMemHandle of the allocation holding ``t``, byte offset of ``t`` in it)."""
    st = t.untyped_storage()
    info = st._share_cuda_()
    handle, offset = info[1], info[3]
    return bytes(handle), int(offset) + t.storage_offset() * t.element_size()


# --------------------------------------------------------------------------- decode side


@dataclass
class Room:
    room: int
    rid: str
    pages: list[int]
    skip_tokens: int
    n_tokens: int
    created: float = field(default_factory=time.monotonic)
    done: bool = False
    ok: bool = False


class PDRendezvous:
    """Decode side. With a tensor-parallel group (``tp``), every rank parks
    the same requests on the same pages (lockstep scheduling); only the
    leader serves the endpoint, its ``describe`` lists every rank's cache
    handles (``ranks``), and it decides when a parked request resumes
    (:meth:`tp_decisions`, replayed on the followers as commands)."""

    def __init__(self, engine, endpoint: str, timeout_s: float = 30.0, tp=None):
        self.engine = engine
        self.endpoint = endpoint
        self.timeout_s = timeout_s
        self.rooms: dict[int, Room] = {}
        self.lock = threading.Lock()
        self._stop = False
        self.stats = {"rooms": 0, "done": 0, "failed": 0, "timeouts": 0}
        self.tp = tp
        rank = tp.rank if tp is not None else 0
        self.leader = rank == 0
        d = self._make_describe()
        self._local_key = None
        if tp is not None:
            import torch.distributed as dist

            d["local"] = self._local_key = f"{endpoint}#{rank}"
            _LOCAL[d["local"]] = engine
            alld = [None] * tp.world
            dist.all_gather_object(alld, d, group=tp.gloo)
            d = dict(alld[0], ranks=alld)
        self._describe = d
        self._th = None
        if self.leader:
            _LOCAL[endpoint] = engine
            self._th = threading.Thread(target=self._serve, name="pd-rendezvous", daemon=True)
            self._th.start()

    def tp_decisions(self) -> list:
        """Leader, before a tensor-parallel step: parked requests whose room
        ended (pushed, failed or timed out), as ``("pd_resume", rid, ok)``."""
        out = []
        for r in list(self.engine.scheduler.parked.values()):
            st = self.poll(r.remote_room)
            if st != "pending":
                out.append(("pd_resume", r.request_id, st == "ok"))
        return out

    # called by the engine thread
    def publish(self, room: int, rid: str, pages: list[int], skip_tokens: int, n_tokens: int) -> None:
        with self.lock:
            self.rooms[room] = Room(room, rid, pages, skip_tokens, n_tokens)
            self.stats["rooms"] += 1

    def poll(self, room: int) -> str:
        """pending / ok / failed / timeout"""
        with self.lock:
            r = self.rooms.get(room)
            if r is None:
                return "failed"
            if r.done:
                self.rooms.pop(room, None)
                return "ok" if r.ok else "failed"
            if time.monotonic() - r.created > self.timeout_s:
                self.rooms.pop(room, None)
                self.stats["timeouts"] += 1
                return "timeout"
            return "pending"

    def forget(self, room: int) -> None:
        with self.lock:
            self.rooms.pop(room, None)

    def _make_describe(self) -> dict:
        run = self.engine.runner
        from infera_b200.ops import kernels as K

        d = {"pid": os.getpid(), "layers": int(run.k_cache.shape[0]), "slots": int(run.k_cache.shape[1]),
             "H": int(run.k_cache.shape[2]), "channels": K.kv_channels(run.k_cache, run.v_cache),
             "device": run.k_cache.device.index if run.k_cache.is_cuda else -1}
        kb = getattr(run, "_k_buf", None)
        if run.k_cache.is_cuda:
            if kb is not None:  # own allocations: whole-buffer handles at offset 0
                d["k"], d["k_off"] = kb.ipc_handle(), 0
                d["v"], d["v_off"] = run._v_buf.ipc_handle(), 0
            else:
                d["k"], d["k_off"] = _ipc_handle(run.k_cache)
                d["v"], d["v_off"] = _ipc_handle(run.v_cache)
        return d

    def describe(self) -> dict:
        return self._describe

    def handle(self, msg: dict) -> dict:
        op = msg.get("op")
        if op == "describe":
            return self.describe()
        if op == "pages":
            with self.lock:
                r = self.rooms.get(int(msg["room"]))
                if r is None:
                    return {"ready": False}
                return {"ready": True, "pages": r.pages, "skip_tokens": r.skip_tokens, "n_tokens": r.n_tokens}
        if op == "done":
            with self.lock:
                r = self.rooms.get(int(msg["room"]))
                if r is not None:
                    r.done, r.ok = True, bool(msg.get("ok"))
                    self.stats["done" if r.ok else "failed"] += 1
            return {"ack": True}
        return {"error": f"unknown op {op!r}"}

    def _serve(self) -> None:
        if not self.endpoint.startswith(("ipc://", "tcp://")):
            return  # in-process only
        import zmq

        sock = zmq.Context.instance().socket(zmq.REP)
        sock.bind(self.endpoint)
        poller = zmq.Poller()
        poller.register(sock, zmq.POLLIN)
        while not self._stop:
            if not poller.poll(200):
                continue
            try:
                req = _unpack(sock.recv())
                sock.send(_pack(self.handle(req)))
            except Exception as e:  # keep serving
                logger.warning("pd rendezvous: %s", e)
                try:
                    sock.send(_pack({"error": str(e)}))
                except Exception:
                    pass
        sock.close(linger=0)

    def close(self) -> None:
        self._stop = True
        if self.leader:
            _LOCAL.pop(self.endpoint, None)
        if self._local_key is not None:
            _LOCAL.pop(self._local_key, None)


# --------------------------------------------------------------------------- prefill side


def _record_done(eng):
    """Completion marker of the work queued so far on the engine's stream
    (True on CPU, where everything ran synchronously)."""
    if not eng.runner.k_cache.is_cuda:
        return True
    ev = torch.cuda.Event(enable_timing=True)
    ev.record()
    return ev


@dataclass
class PushJob:
    rid: str
    room: int
    endpoint: str
    blocks: object              # SeqBlocks held until the push ends
    created: float = field(default_factory=time.monotonic)
    plan: dict | None = None    # page list from the decode side
    event: object = None        # CUDA event of the launched copy
    launched_at: float = 0.0
    layerwise: bool = False     # pushed layer by layer inside the prompt's last forward
    resolved: tuple | None = None   # tensor-parallel leader: (plan, describe) to adopt at the next step
    fail_seen: bool = False         # tensor-parallel leader: failure to announce at the next step


class LayerPush:
    """Per-layer page pushes of one forward (see the module docstring).
    ``items``: (job, source pages, destination pages, peer) per request."""

    def __init__(self, engine, items: list):
        self.eng = engine
        self.items = items
        self.on_gpu = engine.runner.k_cache.is_cuda
        if self.on_gpu:
            agent = engine.pd_agent
            if agent.side is None:
                agent.side = torch.cuda.Stream(engine.device)
            self.side = agent.side
            self.start = torch.cuda.Event(enable_timing=True)
            self.start.record()

    def __call__(self, layer: int) -> None:
        from infera_b200.ops import kernels as K

        r = self.eng.runner
        if not self.on_gpu:
            for _, sp, dp, peer in self.items:
                K.kv_push_pages(r.k_cache, r.v_cache, peer.k, peer.v, sp, dp, layers=(layer, layer + 1),
                                dst_slots=peer.slots)
            return
        ev = torch.cuda.Event()
        ev.record()  # this layer's KV pages are written
        self.side.wait_event(ev)
        with torch.cuda.stream(self.side):
            for _, sp, dp, peer in self.items:
                K.kv_push_pages(r.k_cache, r.v_cache, peer.k, peer.v, sp, dp, layers=(layer, layer + 1),
                                dst_slots=peer.slots)

    def finish(self) -> None:
        """After the forward: every job's completion event (the side stream's
        last push); the main stream also waits for it before the pages can be
        reused."""
        from infera_b200.ops import kernels as K

        end = True
        if self.on_gpu:
            end = torch.cuda.Event(enable_timing=True)
            end.record(self.side)
            torch.cuda.current_stream().wait_event(end)
        if self.eng.pd_agent.tp is not None:
            self.eng.pd_fence()   # see PDPushAgent.progress
            end = _record_done(self.eng)
        L, _, H = self.eng.runner.k_cache.shape
        ps = self.eng.bm.page_size
        for job, sp, dp, _ in self.items:
            job.event = end
            job.start_event = self.start if self.on_gpu else None
            job.launched_at = time.monotonic()
            job._tensors = (sp, dp)
            job.layerwise = True
            st = self.eng.pd_agent.stats
            st["pages"] += int(dp.shape[0])
            st["bytes"] += (K.kv_channels(self.eng.runner.k_cache, self.eng.runner.v_cache) * int(dp.shape[0]) * ps
                            * L * H * self.eng.runner.k_cache.element_size())
            st["layerwise"] += 1


class _Peer:
    """Where a decode instance's caches are, seen from this process."""

    def __init__(self, endpoint: str, engine_device: torch.device, want: tuple | None = None,
                 tp_rank: int | None = None, tp_world: int = 1):
        self.endpoint = endpoint
        self.want = want              # this side's (layers, H, channels): the peer's cache must match
        self.device = engine_device
        self.tp_rank, self.tp_world = tp_rank, tp_world   # set: map that rank of a TP decode group
        self.local = _LOCAL.get(endpoint)
        self.sock = None
        self.k = self.v = None
        self.slots = 0
        self.described = None
        if self.local is not None and tp_rank is None:
            self.k, self.v = self.local.runner.k_cache, self.local.runner.v_cache
            self.slots = self.k.shape[1]
            if want is not None:
                from infera_b200.ops import kernels as K

                got = (int(self.k.shape[0]), int(self.k.shape[2]), K.kv_channels(self.k, self.v))
                if got != want:
                    raise RuntimeError(f"decode instance at {endpoint} has a (layers, H, channels) = {got} "
                                       f"cache, this instance {want}")
            if self.k.is_cuda and self.k.device != engine_device:
                # one process driving both GPUs: map the peer directly
                from infera_b200.ops import _native

                _native.check(_native.kernels().ib_enable_peer_access(self.k.device.index),
                              f"enable peer access to {self.k.device}")
                self.k, self.v = self.k.data_ptr(), self.v.data_ptr()

    def call(self, msg: dict, timeout_ms: int = 2000) -> dict:
        if self.local is not None:
            return self.local.pd_rendezvous.handle(msg)
        import zmq

        if self.sock is None:
            self.sock = zmq.Context.instance().socket(zmq.REQ)
            self.sock.setsockopt(zmq.RCVTIMEO, timeout_ms)
            self.sock.setsockopt(zmq.SNDTIMEO, timeout_ms)
            self.sock.setsockopt(zmq.LINGER, 0)
            self.sock.connect(self.endpoint)
        try:
            self.sock.send(_pack(msg))
            return _unpack(self.sock.recv())
        except zmq.Again:
            self.sock.close(linger=0)  # a REQ socket is stuck after a timeout
            self.sock = None
            raise TimeoutError(f"pd endpoint {self.endpoint} did not answer")

    def describe(self) -> dict:
        if self.described is None:
            self.described = self.call({"op": "describe"})
        return self.described

    def map(self) -> None:
        if self.k is not None:
            return
        self.map_from(self.describe())

    def map_from(self, d: dict) -> None:
        """Map the decode caches that ``d`` (the decode leader's describe)
        names for this rank."""
        if self.k is not None:
            return
        if self.tp_rank is not None:
            ranks = d.get("ranks", [d])
            if len(ranks) != self.tp_world:
                raise RuntimeError(f"decode instance at {self.endpoint} has {len(ranks)} tensor-parallel ranks, "
                                   f"this instance {self.tp_world}")
            d = ranks[self.tp_rank]
        if self.want is not None:
            got = (d["layers"], d["H"], d.get("channels", 2))
            if got != self.want:
                raise RuntimeError(f"decode instance at {self.endpoint} has a (layers, H, channels) = {got} "
                                   f"cache, this instance {self.want}")
        self.slots = d["slots"]
        loc = _LOCAL.get(d.get("local", ""))
        if loc is not None:   # the decode rank lives in this process
            k, v = loc.runner.k_cache, loc.runner.v_cache
            if k.is_cuda and k.device != self.device:
                from infera_b200.ops import _native

                _native.check(_native.kernels().ib_enable_peer_access(k.device.index),
                              f"enable peer access to {k.device}")
                k, v = k.data_ptr(), v.data_ptr()
            self.k, self.v = k, v
            return
        if d["pid"] == os.getpid():
            raise RuntimeError("same-process decode engine not registered locally")
        from infera_b200.ops import _native
        import ctypes

        lib = _native.kernels()
        ptrs = []
        for key in ("k", "v"):
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(d[key])
            _native.check(lib.ib_ipc_open(buf, ctypes.byref(p)), "ib_ipc_open(decode KV cache)")
            ptrs.append(p.value + d[key + "_off"])
        self.k, self.v = ptrs


class PDPushAgent:
    """Network I/O (page lists, cache mapping, done notices) runs on the
    agent's thread; the engine thread only launches copies and polls their
    events, so a slow decode instance never stalls prefill steps."""

    def __init__(self, engine, timeout_s: float = 30.0, tp=None):
        self.engine = engine
        self.timeout_s = timeout_s
        # tensor-parallel prefill group: only the leader talks to the decode
        # side; plans, failures and completions reach every rank as commands
        # (:meth:`tp_decisions` / :meth:`apply`) so the ranks' block managers
        # stay identical, and each rank pushes its own KV-head shard into the
        # same rank of the decode group
        self.tp = tp
        self.leader = tp is None or tp.rank == 0
        self.jobs: list[PushJob] = []
        self.peers: dict[str, _Peer] = {}
        self.lock = threading.Lock()
        self._peer_lock = threading.Lock()
        self._notices: list[tuple[str, int, bool]] = []
        self._wake = threading.Event()
        self._stop = False
        self.stats = {"pushes": 0, "pages": 0, "bytes": 0, "timeouts": 0, "failures": 0, "push_s": 0.0,
                      "push_device_s": 0.0, "layerwise": 0}
        self.early: dict[str, PushJob] = {}   # admitted, plan being resolved, prompt not done yet
        self.side = None                       # stream of the layer-by-layer pushes
        self._th = None
        if self.leader:
            self._th = threading.Thread(target=self._run, name="pd-push-agent", daemon=True)
            self._th.start()

    def submit(self, job: PushJob) -> None:
        with self.lock:
            self.early.pop(job.rid, None)
            self.jobs.append(job)
        self._wake.set()

    def prefetch(self, rid: str, room: int, endpoint: str) -> None:
        """Start resolving the room's page list at admission."""
        with self.lock:
            self.early[rid] = PushJob(rid, room, endpoint, None)
        self._wake.set()

    def take_early(self, rid: str) -> PushJob | None:
        with self.lock:
            return self.early.pop(rid, None)

    def layer_item(self, req):
        """(job, source pages, destination pages, peer) for a request whose
        prompt completes in the next forward, if its page list is known."""
        with self.lock:
            j = self.early.get(req.request_id)
        if j is None or j.plan is None or req.blocks is None:
            return None
        peer = self.peers.get(j.endpoint)
        if peer is None or peer.k is None:
            return None
        ps = self.engine.bm.page_size
        skip = j.plan["skip_tokens"] // ps
        n_pages = (j.plan["n_tokens"] + ps - 1) // ps - skip
        dst = j.plan["pages"][:n_pages]
        src = req.blocks.pages[skip:skip + len(dst)]
        if len(src) != len(dst):
            return None
        dev = self.engine.runner.k_cache.device
        return (j, torch.tensor(src, dtype=torch.int32, device=dev), torch.tensor(dst, dtype=torch.int32, device=dev),
                peer)

    def pending(self) -> int:
        return len(self.jobs)

    def _peer(self, ep: str) -> _Peer:
        with self._peer_lock:   # the agent thread and the engine thread both look peers up
            return self._peer_locked(ep)

    def _peer_locked(self, ep: str) -> _Peer:
        p = self.peers.get(ep)
        if p is None:
            r = self.engine.runner
            from infera_b200.ops import kernels as K

            want = (int(r.k_cache.shape[0]), int(r.k_cache.shape[2]), K.kv_channels(r.k_cache, r.v_cache))
            if self.tp is not None:
                p = _Peer(ep, self.engine.device, want, tp_rank=self.tp.rank, tp_world=self.tp.world)
            else:
                p = _Peer(ep, self.engine.device, want)
            self.peers[ep] = p
        return p

    # ------------------------------------------------------------------ tensor-parallel commands
    def _find(self, rid: str):
        with self.lock:
            j = self.early.get(rid)
            if j is None:
                j = next((x for x in self.jobs if x.rid == rid), None)
        return j

    def tp_decisions(self) -> list:
        """Leader, before a tensor-parallel step: what the agent thread and
        the leader's copy events decided since the last step, as commands
        that every rank (this one included) then applies in the same order."""
        out = []
        with self.lock:
            cands = list(self.early.values()) + list(self.jobs)
            queued = {id(j) for j in self.jobs}
        now = time.monotonic()
        for j in cands:
            if getattr(j, "failed", False):
                continue
            if j.fail_seen:
                out.append(("pd_fail", j.rid))
            elif j.plan is None and j.resolved is not None:
                out.append(("pd_plan", j.rid, j.resolved[0], j.endpoint, j.resolved[1]))
            elif id(j) in queued and j.event is not None and (j.event is True or j.event.query()):
                out.append(("pd_done", j.rid))
            elif id(j) in queued and j.event is None and now - j.created > self.timeout_s:
                out.append(("pd_timeout", j.rid))
        return out

    def apply(self, cmd: tuple) -> None:
        """Apply one ``pd_*`` command (every rank of a tensor-parallel group)."""
        j = self._find(cmd[1])
        if j is None:
            return
        kind = cmd[0]
        if kind == "pd_plan":
            _, _, plan, ep, desc = cmd
            try:
                self._peer(ep).map_from(desc)
                j.plan = plan
            except Exception as e:   # every rank sees the same describe: the same outcome
                logger.warning("kv push for room %s failed: %s", j.room, e)
                j.failed = True
                if self.leader:
                    with self.lock:
                        self._notices.append((j.endpoint, j.room, False))
                    self._wake.set()
        elif kind == "pd_fail":
            j.failed = True
        elif kind == "pd_timeout":
            self.stats["timeouts"] += 1
            self._drop(j)
        elif kind == "pd_done":
            self._complete(j)

    def _drop(self, j) -> None:
        self.engine._release_pushed(j)
        with self.lock:
            self.jobs = [x for x in self.jobs if x is not j]

    def _complete(self, j) -> None:
        self.stats["pushes"] += 1
        self.stats["push_s"] += time.monotonic() - j.launched_at
        if j.event is not True and getattr(j, "start_event", None) is not None:
            # the copy kernels' own device time (CUDA events around them;
            # layer by layer: from the forward's start to the last push)
            self.stats["push_device_s"] += j.start_event.elapsed_time(j.event) / 1000.0
        if self.leader:
            with self.lock:
                self._notices.append((j.endpoint, j.room, True))
            self._wake.set()
        self._drop(j)

    # ------------------------------------------------------------------ agent thread
    def _run(self) -> None:
        dev = self.engine.device
        if dev.type == "cuda":
            torch.cuda.set_device(dev)  # IPC mappings are made in this thread
        while not self._stop:
            self._wake.wait(0.002)
            self._wake.clear()
            with self.lock:
                todo = [j for j in self.jobs if j.plan is None and not getattr(j, "failed", False)]
                todo += [j for j in self.early.values() if j.plan is None and not getattr(j, "failed", False)]
                notices, self._notices = self._notices, []
            for ep, room, ok in notices:
                try:
                    self._peer(ep).call({"op": "done", "room": room, "ok": ok})
                except Exception as e:
                    logger.warning("kv push: done notice for room %s failed: %s", room, e)
            for j in todo:
                if j.resolved is not None or j.fail_seen:
                    continue   # waiting for the next tensor-parallel step to adopt it
                peer = self._peer(j.endpoint)
                try:
                    r = peer.call({"op": "pages", "room": j.room}, timeout_ms=500)
                    if r.get("ready"):
                        if self.tp is not None:
                            j.resolved = (r, peer.describe())
                        else:
                            peer.map()
                            j.plan = r
                except TimeoutError:
                    pass
                except Exception as e:
                    logger.warning("kv push for room %s failed: %s", j.room, e)
                    if self.tp is not None:
                        j.fail_seen = True
                    else:
                        j.failed = True
                    if j.blocks is not None or j in self.jobs:
                        with self.lock:
                            self._notices.append((j.endpoint, j.room, False))

    # ------------------------------------------------------------------ engine thread
    def progress(self) -> None:
        from infera_b200.ops import kernels as K

        eng = self.engine
        keep = []
        launched = []
        with self.lock:
            jobs = list(self.jobs)
        for j in jobs:
            if getattr(j, "failed", False):
                self.stats["failures"] += 1
                eng._release_pushed(j)
                continue
            if j.event is None and j.plan is not None:
                launched.append(j)
                peer = self.peers[j.endpoint]
                ps = eng.bm.page_size
                skip = j.plan["skip_tokens"] // ps
                n_pages = (j.plan["n_tokens"] + ps - 1) // ps - skip
                dst = j.plan["pages"][:n_pages]
                src = j.blocks.pages[skip:skip + len(dst)]
                dev = eng.runner.k_cache.device
                sp = torch.tensor(src, dtype=torch.int32, device=dev)
                dp = torch.tensor(dst, dtype=torch.int32, device=dev)
                if eng.runner.k_cache.is_cuda:
                    j.start_event = torch.cuda.Event(enable_timing=True)
                    j.start_event.record()
                K.kv_push_pages(eng.runner.k_cache, eng.runner.v_cache, peer.k, peer.v, sp, dp, dst_slots=peer.slots)
                j.launched_at = time.monotonic()
                if self.tp is None:
                    j.event = _record_done(eng)
                j._tensors = (sp, dp)
                L, _, H = eng.runner.k_cache.shape
                self.stats["pages"] += len(dst)
                C = K.kv_channels(eng.runner.k_cache, eng.runner.v_cache)
                self.stats["bytes"] += C * len(dst) * ps * L * H * eng.runner.k_cache.element_size()
            if self.tp is not None:
                keep.append(j)   # completion and timeouts arrive as commands
                continue
            if j.event is not None and (j.event is True or j.event.query()):
                self.stats["pushes"] += 1
                self.stats["push_s"] += time.monotonic() - j.launched_at
                if j.event is not True and getattr(j, "start_event", None) is not None:
                    # the copy kernels' own device time (CUDA events around them;
                    # layer by layer: from the forward's start to the last push)
                    self.stats["push_device_s"] += j.start_event.elapsed_time(j.event) / 1000.0
                with self.lock:
                    self._notices.append((j.endpoint, j.room, True))
                self._wake.set()
                eng._release_pushed(j)
                continue
            if j.event is None and time.monotonic() - j.created > self.timeout_s:
                self.stats["timeouts"] += 1
                eng._release_pushed(j)
                continue
            keep.append(j)
        with self.lock:
            done_ids = {id(j) for j in jobs} - {id(j) for j in keep}
            self.jobs = [j for j in self.jobs if id(j) not in done_ids]
        if self.tp is not None and launched:
            # every rank launched the same pushes: a collective after them
            # means, once the leader sees it complete, that every rank's
            # copies have completed (each rank's collective waits for its
            # own stream's pushes)
            eng.pd_fence()
            ev = _record_done(eng)
            for j in launched:
                j.event = ev

    def close(self) -> None:
        self._stop = True
