"""The serving engine: scheduler + block manager + model runner.

``LLMEngine.step()`` runs one iteration (schedule -> one forward -> sample
-> bookkeeping) and returns the new tokens of every request that produced
one. It is single-threaded by design; :mod:`infera_b200.engine.async_engine`
runs it on a dedicated thread for the HTTP server.
"""

from __future__ import annotations

import contextlib

import time
from dataclasses import dataclass, field
from typing import Callable

import torch

from infera_b200.engine.block_manager import BlockManager
from infera_b200.engine.model_runner import ModelRunner
from infera_b200.engine.request import Request, RequestOutput, SamplingParams, Status
from infera_b200.engine.scheduler import Scheduler
from infera_b200.models.config import DenseConfig, get_config
from infera_b200.models.dense import DenseModel


def _tier_store(spec: str):
    """Build the store behind a ``kv_tier`` spec (see EngineConfig)."""
    kind, _, rest = spec.partition(":")
    if kind == "kvd":
        from infera_b200.kvd.client import SyncKvdStore

        return SyncKvdStore(rest)
    if kind == "pinned":
        # one page-locked arena of page slots, copied to and from by DMA
        from infera_b200.engine.pinned_store import PinnedPageStore

        return PinnedPageStore(int(float(rest or 4) * (1 << 30)))
    if kind == "host":
        from infera_b200.kvd.store import HostStore
        from infera_b200.kvd.tablespace import Tablespace

        gib, _, nvme = rest.partition(":")
        if nvme.startswith("files:"):
            # one file per chunk, kept under INFERA_KVD_L3_BUDGET_BYTES by the reaper
            from infera_b200.engine.l3_reaper import FileChunkStore

            l3 = FileChunkStore(nvme[len("files:"):])
        else:
            l3 = Tablespace(nvme, fsync=False) if nvme else None
        return HostStore(int(float(gib or 4) * (1 << 30)), l3=l3)
    raise ValueError(f"unknown kv_tier spec {spec!r}")


@dataclass
class EngineConfig:
    model: str = "llama-3.1-8b"
    page_size: int = 16
    max_num_seqs: int = 256
    max_batched_tokens: int = 2048
    gpu_memory_utilization: float = 0.90
    num_pages: int | None = None          # override the memory-derived page count
    use_cuda_graphs: bool = True
    enable_prefix_cache: bool = True
    seed: int = 0
    long_prefill_threshold: int = 0
    # prompt tokens per step while sequences are decoding: bounds the step
    # time that decoding sequences see as their inter-token latency (0: the
    # whole max_batched_tokens budget). On the 8B agentic trace at 8 req/s,
    # 256 gave ITL p99 19.1 ms / TTFT p50 48 ms against 22.0 ms / 37 ms for
    # 512, both far inside the SLO
    mixed_prefill_tokens: int = 256
    max_model_len: int | None = None
    model_overrides: dict = field(default_factory=dict)
    # KV tiering: None (off), "pinned:<GiB>" (in-process page-locked arena of
    # page slots, DMA both ways), "host:<GiB>[:<nvme dir>]" (in-process host store,
    # optional NVMe tablespace), "host:<GiB>:files:<dir>" (NVMe tier of one
    # file per chunk under the reaper's budget) or "kvd:<socket path>"
    # (shared daemon)
    kv_tier: str | None = None
    # promote tier hits on a loader thread while the engine keeps stepping
    # (tensor-parallel ranks always promote inline)
    kv_tier_async: bool = True
    # prefill/decode disaggregation: "mixed", "prefill" or "decode"; a decode
    # instance serves its KV rendezvous on kv_push_endpoint
    disagg_mode: str = "mixed"
    kv_push_endpoint: str | None = None
    # PD prefill: push each layer's KV pages inside the prompt's last forward
    pd_layerwise: bool = True


class _PhaseRange:
    """One named range in the torch profiler's trace and in NVTX."""

    def __init__(self, name: str, cuda: bool):
        self.name, self.cuda = name, cuda
        self.rf = None

    def __enter__(self):
        self.rf = torch.profiler.record_function(self.name)
        self.rf.__enter__()
        if self.cuda:
            torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        if self.cuda:
            torch.cuda.nvtx.range_pop()
        self.rf.__exit__(*exc)
        return False


class LLMEngine:
    def __init__(self, cfg: EngineConfig, device: str | torch.device = "cuda:0",
                 event_sink: Callable[[str, dict], None] | None = None, model_cfg: DenseConfig | None = None,
                 tp=None, ep=None):
        self.cfg = cfg
        self.device = torch.device(device)
        if self.device.type == "cuda":
            torch.cuda.set_device(self.device)
        mcfg = model_cfg or get_config(cfg.model)
        for k, v in cfg.model_overrides.items():
            setattr(mcfg, k, v)
        if cfg.max_model_len:
            mcfg.max_model_len = cfg.max_model_len
        self.model_cfg = mcfg
        self.tp = tp
        if getattr(mcfg, "kv_channels", 2) == 1:  # MLA: one latent cache row per token
            from infera_b200.models.mla import MLAModel

            self.model = MLAModel(mcfg, self.device, seed=cfg.seed, tp=tp, ep=ep)
        else:
            self.model = DenseModel(mcfg, self.device, seed=cfg.seed, tp=tp)
        num_pages = cfg.num_pages or self._derive_num_pages()
        if tp is not None and tp.world > 1:
            # every rank runs the same scheduler: agree on the page count
            import torch.distributed as dist

            t = torch.tensor([num_pages], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MIN, group=tp.gloo)
            num_pages = int(t.item())
        self._event_sink = event_sink
        self.kv_index = None
        self.bm = BlockManager(num_pages, cfg.page_size, cfg.enable_prefix_cache, event_sink=self._on_kv_event)
        self.scheduler = Scheduler(self.bm, cfg.max_num_seqs, cfg.max_batched_tokens, mcfg.max_model_len,
                                   watermark_pages=max(1, num_pages // 100),
                                   long_prefill_threshold=cfg.long_prefill_threshold,
                                   mixed_prefill_tokens=cfg.mixed_prefill_tokens)
        self.runner = ModelRunner(self.model, num_pages, cfg.page_size, cfg.max_num_seqs, cfg.max_batched_tokens,
                                  use_graphs=cfg.use_cuda_graphs, exportable=cfg.disagg_mode == "decode")
        self.tier = None
        if cfg.kv_tier:
            from infera_b200.engine.tiering import TierManager

            tp_world = tp.world if tp is not None else 1
            # tensor-parallel ranks hold different KV-head shards under the same
            # block hashes (their keys carry the rank), and promote inline so
            # that every rank makes the same scheduling decisions
            self.tier = TierManager(self.runner.k_cache, self.runner.v_cache, _tier_store(cfg.kv_tier),
                                    cfg.page_size, async_load=cfg.kv_tier_async and tp_world == 1,
                                    key_tag=f"/tp{tp.rank}of{tp_world}".encode() if tp_world > 1 else b"")
            self.bm.tier = self.tier
            self.scheduler.on_tier_load = self._begin_tier_load
        self.pd_rendezvous = None
        self.pd_agent = None
        if cfg.disagg_mode == "decode":
            from infera_b200.engine.pd import PDRendezvous

            ep = cfg.kv_push_endpoint or f"local://{id(self)}"
            self.pd_rendezvous = PDRendezvous(self, ep, tp=self._pd_tp())
            self.scheduler.on_park = lambda r, pages, skip, n: self.pd_rendezvous.publish(
                r.remote_room, r.request_id, [int(x) for x in pages], skip, n)
        self.requests: dict[str, Request] = {}
        # commands applied since the last step, when a tensor-parallel leader
        # replays them on its followers (None: not recorded)
        self.cmd_log: list | None = None
        self.num_steps = 0
        self.last_step_shape = (0, 0)
        self.last_step_kv = 0
        self.clock: Callable[[], float] = time.monotonic
        # forward_s: host time inside the model forward (each step ends by
        # reading its sampled tokens back, so this is the engine's busy time)
        self.counters = {"prompt_tokens": 0, "generation_tokens": 0, "finished": 0, "preemptions": 0,
                         "forward_s": 0.0}
        # named phase ranges (torch.profiler record_function + NVTX) while a
        # profile is being taken: schedule / forward (prefill+decode counts) / kv push
        self.trace_phases = False

    # ------------------------------------------------------------------ sizing
    def _derive_num_pages(self) -> int:
        mcfg = self.model.cfg  # this rank's shard of the model
        per_page = getattr(mcfg, "kv_channels", 2) * mcfg.num_layers * self.cfg.page_size * mcfg.kv_size * 2
        if self.device.type != "cuda":
            return 512
        torch.cuda.synchronize()
        free, total = torch.cuda.mem_get_info(self.device)
        # leave room for activations, graphs, workspaces
        max_tok = self.cfg.max_batched_tokens + self.cfg.max_num_seqs
        act = max_tok * (mcfg.hidden * 3 + mcfg.qkv_size + mcfg.q_size + mcfg.ffn) * 2
        act += self.cfg.max_num_seqs * mcfg.vocab * 2 * 2
        reserve = act + 2 * 1024 ** 3 + int(total * (1.0 - self.cfg.gpu_memory_utilization))
        budget = max(0, free - reserve)
        return max(64, budget // per_page)

    # ------------------------------------------------------------------ events
    def _on_kv_event(self, kind: str, payload: dict) -> None:
        if self._event_sink is not None:
            self._event_sink(kind, payload)
        if self.kv_index is not None:
            self.kv_index.on_engine_event(kind, payload)

    def attach_kv_index(self, feed) -> None:
        """Announce this engine's device / host / disk blocks to the router's
        tier-aware KV index through ``feed`` (a
        :class:`~infera_b200.engine.kv_index_feed.KvIndexFeed`)."""
        self.kv_index = feed
        if self.tier is not None:
            self.tier.index_sink = feed.on_tier_event

    def set_event_sink(self, sink: Callable[[str, dict], None] | None) -> None:
        self._event_sink = sink

    # ------------------------------------------------------------------ API
    def add_request(self, request_id: str, prompt_token_ids: list[int], sampling: SamplingParams | None = None,
                    arrival_time: float | None = None) -> Request:
        if request_id in self.requests:
            raise ValueError(f"duplicate request id {request_id}")
        if not prompt_token_ids:
            raise ValueError("empty prompt")
        req = Request(request_id=request_id, prompt_token_ids=list(prompt_token_ids),
                      sampling=sampling or SamplingParams(), eos_token_id=self.model_cfg.eos_token_id)
        req.arrival_time = self.clock() if arrival_time is None else arrival_time
        ktp = req.sampling.kv_transfer or {}
        if ktp.get("do_remote_prefill") and self.pd_rendezvous is not None and "room" in ktp:
            req.remote_room = int(ktp["room"])
        if ktp.get("do_remote_decode") and ktp.get("decode_kv_endpoint") and "room" in ktp:
            req.remote_decode = (int(ktp["room"]), str(ktp["decode_kv_endpoint"]))
            if self.cfg.pd_layerwise and ktp.get("layerwise", True):   # per request: {"layerwise": false}
                from infera_b200.engine.pd import PDPushAgent

                if self.pd_agent is None:
                    self.pd_agent = PDPushAgent(self, tp=self._pd_tp())
                self.pd_agent.prefetch(request_id, *req.remote_decode)
        self.requests[request_id] = req
        self.scheduler.add(req)
        if self.cmd_log is not None:
            self.cmd_log.append(("add", request_id, list(prompt_token_ids), req.sampling))
        return req

    def abort_request(self, request_id: str) -> bool:
        if self.cmd_log is not None:
            self.cmd_log.append(("abort", request_id))
        r = self.scheduler.abort(request_id)
        if r is not None:
            self.requests.pop(request_id, None)
            return True
        return False

    def has_unfinished(self) -> bool:
        return self.scheduler.num_unfinished() > 0 or (self.pd_agent is not None and self.pd_agent.pending() > 0)

    # ------------------------------------------------------------------ PD
    def _pd_tp(self):
        """The tensor-parallel group when PD runs over one (world > 1)."""
        return self.tp if self.tp is not None and self.tp.world > 1 else None

    def pd_tp_decisions(self) -> list:
        """Tensor-parallel leader, before broadcasting a step: PD events that
        change scheduling state (plans adopted, pushes completed or failed,
        parked requests resumed), applied here and returned for the
        followers to apply at the same point."""
        cmds = []
        if self.pd_agent is not None:
            cmds += self.pd_agent.tp_decisions()
        if self.pd_rendezvous is not None:
            cmds += self.pd_rendezvous.tp_decisions()
        for c in cmds:
            self.pd_apply(c)
        return cmds

    def pd_apply(self, c: tuple) -> None:
        if c[0] == "pd_resume":
            r = self.scheduler.parked.get(c[1])
            if r is not None:
                self.pd_rendezvous.forget(r.remote_room)
                self.scheduler.resume_parked(r, bool(c[2]))
        elif self.pd_agent is not None:
            self.pd_agent.apply(c)

    def pd_fence(self) -> None:
        """A collective over the tensor-parallel group, queued after this
        rank's KV pushes (see ``PDPushAgent.progress``)."""
        import torch.distributed as dist

        if getattr(self, "_fence_buf", None) is None:
            self._fence_buf = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.all_reduce(self._fence_buf, group=self.tp.nccl)

    def _pd_progress(self) -> None:
        if self.pd_agent is not None and self.pd_agent.pending():
            self.pd_agent.progress()
        if self.pd_rendezvous is not None and self.scheduler.parked and self._pd_tp() is None:
            for r in list(self.scheduler.parked.values()):
                st = self.pd_rendezvous.poll(r.remote_room)
                if st != "pending":
                    self.scheduler.resume_parked(r, st == "ok")

    # ------------------------------------------------------------------ KV tiers
    def _begin_tier_load(self, r: Request, pages: list[int], hashes: list[int]) -> None:
        self.tier.begin_load(r, pages, hashes)

    def _tier_progress(self) -> None:
        """Requests whose tier promote landed: register the promoted pages in
        the prefix cache and let them run."""
        ps = self.bm.page_size
        for r, got in self.tier.poll_loads():
            if r.request_id in self.scheduler.loading and r.status != Status.FINISHED_ABORTED and got > 0:
                done = (r.tier_start + got) * ps
                self.bm.commit_full_pages(r.blocks, r.all_token_ids(), done)
                r.num_computed = max(r.num_computed, done)
                if r.num_preemptions == 0:
                    r.num_cached_prompt_tokens = r.num_computed
                self.bm.stats["tier_hit_tokens"] += got * ps
                self.bm.stats["hit_tokens"] += got * ps
            self.scheduler.resume_loaded(r)

    def _release_pushed(self, job) -> None:
        if job.blocks is not None:
            self.bm.free(job.blocks)
            job.blocks = None

    def num_running(self) -> int:
        return len(self.scheduler.running)

    def num_waiting(self) -> int:
        return len(self.scheduler.waiting)

    def _block_table_updates(self, chunks) -> tuple[list[int], list[int]]:
        idx, val = [], []
        mp = self.runner.max_pages
        for c in chunks:
            r = c.req
            pages = r.blocks.pages
            if r.pages_synced < len(pages):
                base = r.table_row * mp
                for j in range(r.pages_synced, len(pages)):
                    idx.append(base + j)
                    val.append(pages[j])
                r.pages_synced = len(pages)
        return idx, val

    def _phase(self, name: str):
        if not self.trace_phases:
            return contextlib.nullcontext()
        return _PhaseRange(name, self.device.type == "cuda")

    def step(self) -> list[RequestOutput]:
        # the CUDA current device is per host thread: a step driven from a
        # thread that never selected this engine's GPU would launch the
        # kernels on the wrong device with this device's pointers
        if self.device.type == "cuda" and torch.cuda.current_device() != self.device.index:
            torch.cuda.set_device(self.device)
        if self.pd_agent is not None or self.pd_rendezvous is not None:
            with self._phase("kv_push"):
                self._pd_progress()
        if self.tier is not None and self.scheduler.loading:
            self._tier_progress()
        with self._phase("schedule"):
            sched = self.scheduler.schedule()
        if self.tier is not None:
            # evicted prefix pages are copied out before this step's forward
            # can overwrite them; promotes start after that
            self.tier.flush_saves()
            self.tier.submit_loads()
        outputs: list[RequestOutput] = []
        for r in sched.preempted:
            if r.status == Status.FINISHED_LENGTH:  # prompt longer than the model allows
                outputs.append(self._finish(r, Status.FINISHED_LENGTH))
            else:
                self.counters["preemptions"] += 1
        if sched.empty:
            if (self.scheduler.parked or self.scheduler.loading
                    or (self.pd_agent is not None and self.pd_agent.pending())):
                time.sleep(0.0005)  # only waiting on a KV push or a tier promote
            return outputs
        upd = self._block_table_updates(sched.prefills + sched.decodes)
        layer_push = None
        if self.pd_agent is not None and self.pd_agent.early:
            items = []
            for c in sched.prefills:
                r = c.req
                if r.remote_decode is not None and c.start + c.num_tokens >= len(r.prompt_token_ids):
                    it = self.pd_agent.layer_item(r)
                    if it is not None:
                        items.append(it)
            if items:
                from infera_b200.engine.pd import LayerPush

                layer_push = LayerPush(self, items)
        t_fwd = time.perf_counter()
        with self._phase(f"forward prefill={len(sched.prefills)} decode={len(sched.decodes)}"):
            res = self.runner.execute(sched, upd, layer_hook=layer_push)
        self.counters["forward_s"] += time.perf_counter() - t_fwd
        if layer_push is not None:
            layer_push.finish()
        now = self.clock()
        self.num_steps += 1
        # (prompt tokens, decoding sequences) of this step, for step-time profiles
        self.last_step_shape = (sum(c.num_tokens for c in sched.prefills), len(sched.decodes))
        # cached tokens the step's decode attention read (the step's KV bytes)
        self.last_step_kv = sum(c.req.num_computed for c in sched.decodes)
        for c in sched.prefills:
            c.req.num_computed = c.start + c.num_tokens
            self.counters["prompt_tokens"] += c.num_tokens
        for c in sched.decodes:
            c.req.num_computed = c.start + 1
        # register newly completed pages in the prefix cache
        for c in sched.prefills + sched.decodes:
            r = c.req
            if r.blocks is not None and r.num_computed // self.bm.page_size > len(r.blocks.hashes):
                self.bm.commit_full_pages(r.blocks, r.all_token_ids(), r.num_computed)
        for c, tok in zip(res.rows, res.token_ids):
            r = c.req
            if r.status != Status.RUNNING:
                continue
            r.output_token_ids.append(int(tok))
            self.counters["generation_tokens"] += 1
            if r.first_token_time is None:
                r.first_token_time = now
            r.token_times.append(now)
            st = r.check_stop()
            if st is not None:
                outputs.append(self._finish(r, st, new=[int(tok)]))
            else:
                outputs.append(RequestOutput(r.request_id, [int(tok)], False, None, len(r.prompt_token_ids),
                                             r.num_cached_prompt_tokens, len(r.output_token_ids)))
        return outputs

    def _finish(self, r: Request, st: Status, new: list[int] | None = None) -> RequestOutput:
        if r.remote_decode is not None and r.num_computed >= len(r.prompt_token_ids) - 1:
            # PD prefill: hold the prompt's pages until they are pushed
            from infera_b200.engine.pd import PDPushAgent, PushJob

            held = self.scheduler.finish(r, st, hold_blocks=True)
            if self.pd_agent is None:
                self.pd_agent = PDPushAgent(self, tp=self._pd_tp())
            room, ep = r.remote_decode
            job = self.pd_agent.take_early(r.request_id)
            if job is None:
                job = PushJob(r.request_id, room, ep, held)
            else:
                job.blocks = held  # pushed layer by layer already, or still waiting for its plan
            self.pd_agent.submit(job)
        else:
            self.scheduler.finish(r, st)
        r.finish_time = self.clock()
        self.requests.pop(r.request_id, None)
        self.counters["finished"] += 1
        return RequestOutput(r.request_id, new or [], True, st.value, len(r.prompt_token_ids),
                             r.num_cached_prompt_tokens, len(r.output_token_ids))

    def close(self) -> None:
        """Release device resources that outlive a process group (graphs)."""
        self.runner.release_graphs()

    # ------------------------------------------------------------------ helpers
    def generate(self, prompts: list[list[int]], sampling: SamplingParams | None = None) -> list[list[int]]:
        """Offline batch generation: returns the output ids of each prompt."""
        ids = []
        for i, p in enumerate(prompts):
            rid = f"gen-{self.num_steps}-{i}"
            self.add_request(rid, p, sampling)
            ids.append(rid)
        outs: dict[str, list[int]] = {rid: [] for rid in ids}
        while self.has_unfinished():
            for o in self.step():
                if o.request_id in outs:
                    outs[o.request_id].extend(o.new_token_ids)
        return [outs[r] for r in ids]

    def stats(self) -> dict:
        bm = self.bm
        q = max(1, bm.stats["query_tokens"])
        return {
            "running": self.num_running(),
            "waiting": self.num_waiting(),
            "kv_usage": bm.usage(),
            "num_pages": bm.num_pages,
            "prefix_hit_rate": bm.stats["hit_tokens"] / q,
            "steps": self.num_steps,
            "h2d_bytes": self.runner.h2d_bytes,
            "d2h_bytes": self.runner.d2h_bytes,
            "pd_push_queue": self.pd_agent.pending() if self.pd_agent is not None else 0,
            "pd_pushes": self.pd_agent.stats["pushes"] if self.pd_agent is not None else 0,
            "pd_push_bytes": self.pd_agent.stats["bytes"] if self.pd_agent is not None else 0,
            "pd_push_seconds": self.pd_agent.stats["push_s"] if self.pd_agent is not None else 0.0,
            "pd_push_device_seconds": self.pd_agent.stats["push_device_s"] if self.pd_agent is not None else 0.0,
            "pd_parked": len(self.scheduler.parked),
            **self.counters,
        }
