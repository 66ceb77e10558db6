"""Open-loop replay of an agentic trace through an in-process engine.

Arrivals are Poisson at ``rate`` requests/s; each arrival becomes the next
turn of the next idle session (a session never has two turns in flight).
Time is measured on the device: a CUDA event is recorded at the end of
every engine step's kernels, and token timestamps are those events'
offsets from the window's start event. Arrival times are host offsets from
the same origin (taken right after a synchronize, so both clocks start
together).

The replay advances in slices of ``slice_s`` seconds; one slice is one
benchmark step.
"""

from __future__ import annotations

import random
import time
from collections import deque

import torch

from infera_b200.bench.slo import ReqRecord
from infera_b200.bench.trace import Session, TraceSpec, build_sessions
from infera_b200.engine.request import SamplingParams


class EngineReplay:
    def __init__(self, engine, spec: TraceSpec, session_ids: list[int], rate: float, seed: int = 0,
                 device_timing: bool = True):
        self.eng = engine
        self.spec = spec
        self.rate = rate
        self.rng = random.Random(seed + 17)
        self.seed = seed
        self.sessions: list[Session] = build_sessions(spec, seed, session_ids)
        self.next_sid = max(session_ids) + 1 + 1_000_000 * (seed + 1)
        self.idle: deque[Session] = deque(self.sessions)
        self.pending_arrivals: deque[float] = deque()
        self.records: dict[str, ReqRecord] = {}
        self.inflight: dict[str, tuple[Session, list[int]]] = {}
        self.device_timing = device_timing and torch.cuda.is_available() and engine.device.type == "cuda"
        self.t0_host = None
        self.ev0 = None
        self.step_events: list = []         # (event, host_time)
        self.step_shapes: list = []         # (prompt tokens, decoding sequences) per step
        self.step_kv: list = []             # cached tokens read by decode attention per step
        self.step_host: list = []           # (host issue s, host wait-for-device s) per step
        self.token_steps: dict[str, list[int]] = {}
        self.collected: dict[str, list[int]] = {}
        self.next_arrival = None
        self.req_counter = 0

    # ------------------------------------------------------------------ clocks
    def start_clock(self) -> None:
        if self.device_timing:
            torch.cuda.synchronize()
            self.ev0 = torch.cuda.Event(enable_timing=True)
            self.ev0.record()
        self.t0_host = time.monotonic()
        self.next_arrival = self._draw_gap()

    def now(self) -> float:
        return time.monotonic() - self.t0_host

    def _draw_gap(self) -> float:
        return self.rng.expovariate(self.rate)

    # ------------------------------------------------------------------ sessions
    def _recycle(self, s: Session) -> Session:
        fresh = build_sessions(self.spec, self.seed, [self.next_sid])[0]
        fresh.group = s.group
        fresh.prefix = s.prefix
        self.next_sid += 1
        return fresh

    def _issue(self, s: Session, arrival: float) -> None:
        prompt = s.next_prompt()
        rid = f"s{s.sid}-t{s.turn}-{self.req_counter}"
        self.req_counter += 1
        out_len = s.out_lens[s.turn]
        self.eng.add_request(rid, prompt, SamplingParams(max_tokens=out_len, ignore_eos=True))
        self.records[rid] = ReqRecord(rid, arrival, prompt_len=len(prompt))
        self.inflight[rid] = (s, prompt)
        self.token_steps[rid] = []
        self.collected[rid] = []
        s.busy = True

    def _admit_arrivals(self) -> None:
        now = self.now()
        while self.next_arrival is not None and self.next_arrival <= now:
            self.pending_arrivals.append(self.next_arrival)
            self.next_arrival += self._draw_gap()
        while self.pending_arrivals and self.idle:
            arr = self.pending_arrivals.popleft()
            s = self.idle.popleft()
            idle_since = s.idle_since
            if s.done(self.spec.context_cap):
                s = self._recycle(s)
            # a turn cannot exist before its session's previous turn ended
            self._issue(s, max(arr, idle_since, 0.0))

    # ------------------------------------------------------------------ main loop
    def prime_prefixes(self) -> None:
        """Compute every group's system prefix once (a long-running server
        has them cached); not part of any measured window."""
        seen = set()
        prompts = []
        for s in self.sessions:
            key = tuple(s.prefix[:8])
            if s.prefix and key not in seen:
                seen.add(key)
                prompts.append(s.prefix)
        if prompts:
            self.eng.generate(prompts, SamplingParams(max_tokens=1, ignore_eos=True))

    def run_until(self, t_end: float) -> None:
        while True:
            now = self.now()
            if now >= t_end:
                return
            self._admit_arrivals()
            if self.eng.has_unfinished():
                self.step_once()
            else:
                wait = (self.next_arrival or now) - now
                if wait > 0:
                    time.sleep(min(wait, t_end - now, 0.002))

    def step_once(self) -> None:
        """One engine step and its bookkeeping (token steps, finished turns
        returning their session to the idle pool)."""
        outs = self.eng.step()
        step_idx = len(self.step_events)
        self.step_shapes.append(getattr(self.eng, "last_step_shape", (0, 0)))
        self.step_kv.append(getattr(self.eng, "last_step_kv", 0))
        runner = getattr(self.eng, "runner", None)
        self.step_host.append(getattr(runner, "last_timing", (0.0, 0.0)))
        if self.device_timing:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self.step_events.append((ev, self.now()))
        else:
            self.step_events.append((None, self.now()))
        for o in outs:
            rid = o.request_id
            rec = self.records.get(rid)
            if rec is None:
                continue
            self.token_steps[rid].extend([step_idx] * len(o.new_token_ids))
            self.collected[rid].extend(o.new_token_ids)
            if o.finished:
                s, prompt = self.inflight.pop(rid)
                rec.cached_len = o.num_cached_tokens
                rec.out_len = o.num_output_tokens
                rec.finish = step_idx  # resolved to a time later
                s.history = prompt + self.collected.pop(rid)
                s.turn += 1
                s.busy = False
                s.idle_since = self.now()
                self.idle.append(s)

    # ------------------------------------------------------------------ results
    def step_profile(self, window: tuple[float, float]) -> dict:
        """Durations of the engine steps that ended inside ``window`` (device
        time between consecutive step-end events), by kind: decode-only,
        mixed (prompt chunks joining decodes, by prompt tokens) and
        prompt-only. Call after :meth:`resolve`."""
        from infera_b200.bench.slo import percentile

        times = self._times
        kinds: dict[str, list[float]] = {}
        toks: dict[str, list[int]] = {}
        issue: dict[str, list[float]] = {}
        wait: dict[str, list[float]] = {}
        for i in range(1, len(times)):
            if not (window[0] <= times[i] <= window[1]):
                continue
            pt, nd = self.step_shapes[i]
            if nd and not pt:
                k = "decode"
            elif nd:
                k = "mixed<=256" if pt <= 256 else ("mixed<=512" if pt <= 512 else "mixed>512")
            else:
                k = "prefill"
            kinds.setdefault(k, []).append(1000 * (times[i] - times[i - 1]))
            toks.setdefault(k, []).append(pt)
            hi, hw = self.step_host[i] if i < len(self.step_host) else (0.0, 0.0)
            issue.setdefault(k, []).append(1000 * hi)
            wait.setdefault(k, []).append(1000 * hw)
        # host_issue: host time from the start of the forward to its last
        # launch; host_wait: time the host then waited for the device (near
        # zero means the step was bound by the host's launch rate)
        out = {k: {"n": len(v), "p50_ms": round(percentile(v, 50), 3), "p99_ms": round(percentile(v, 99), 3),
                   "mean_prompt_tokens": round(sum(toks[k]) / len(v), 1),
                   "host_issue_p50_ms": round(percentile(issue[k], 50), 3),
                   "host_wait_p50_ms": round(percentile(wait[k], 50), 3)} for k, v in sorted(kinds.items())}
        # decode steps against their byte roofline: every weight byte plus
        # the K/V bytes of the cached tokens read, at the measured copy rate
        wb, kvb = self.roofline_bytes()
        if "decode" in out and wb:
            kv = [self.step_kv[i] for i in range(1, len(times)) if window[0] <= times[i] <= window[1]
                  and i < len(self.step_kv) and self.step_shapes[i][1] and not self.step_shapes[i][0]]
            if kv:
                roof = [(wb + kvb * n) / self.PEAK_HBM * 1e3 for n in kv]
                r50 = percentile(roof, 50)
                out["decode"].update(mean_kv_tokens=round(sum(kv) / len(kv)), weight_gb=round(wb / 1e9, 2),
                                     roofline_p50_ms=round(r50, 3),
                                     frac_of_roofline_p50=round(r50 / out["decode"]["p50_ms"], 3)
                                     if out["decode"]["p50_ms"] else None)
        return out

    PEAK_HBM = 6418.2e9   # measured B200 copy rate (bytes/s)

    def roofline_bytes(self) -> tuple[int, int]:
        """(weight bytes, K/V bytes per cached token) of this GPU's model."""
        m = getattr(self.eng, "model", None)
        w = getattr(m, "w", None)
        cfg = getattr(m, "cfg", None)
        if w is None or cfg is None or not hasattr(w, "nbytes"):
            return 0, 0
        hd = getattr(cfg, "head_dim", 0)
        kvh = getattr(cfg, "num_kv_heads", 0)
        if hd and kvh:
            per_tok = cfg.num_layers * kvh * hd * 2 * 2
        else:  # latent cache: one 576-element row per token and layer
            per_tok = cfg.num_layers * 576 * 2
        return w.nbytes(), per_tok

    def resolve(self) -> list[ReqRecord]:
        """Convert step indices into timestamps (device when available)."""
        if self.device_timing:
            torch.cuda.synchronize()
            times = [self.ev0.elapsed_time(ev) / 1000.0 for ev, _ in self.step_events]
        else:
            times = [t for _, t in self.step_events]
        self._times = times
        out = []
        for rid, rec in self.records.items():
            steps = self.token_steps.get(rid, [])
            rec.token_times = [times[i] for i in steps]
            rec.first_token = rec.token_times[0] if rec.token_times else None
            if isinstance(rec.finish, int):
                rec.finish = times[rec.finish]
            out.append(rec)
        return out
