"""Latency records and SLO goodput.

A request meets its SLO when its time to first token is within the TTFT
bound and the 99th percentile of its inter-token latencies is within the
ITL bound. Goodput = SLO-meeting requests of the window's cohort (by
default: the requests that arrived in it) per second of window. The fleet-level p99 TTFT / p99 ITL over all requests and tokens and
the p50 TTFT are reported beside it.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field


@dataclass
class ReqRecord:
    rid: str
    arrival: float
    first_token: float | None = None
    token_times: list[float] = field(default_factory=list)
    finish: float | None = None
    prompt_len: int = 0
    cached_len: int = 0
    out_len: int = 0

    @property
    def ttft(self) -> float | None:
        return None if self.first_token is None else self.first_token - self.arrival

    def itls(self) -> list[float]:
        t = self.token_times
        return [b - a for a, b in zip(t, t[1:])]


def percentile(xs: list[float], q: float) -> float:
    if not xs:
        return float("nan")
    s = sorted(xs)
    k = (len(s) - 1) * q / 100.0
    f, c = math.floor(k), math.ceil(k)
    if f == c:
        return s[int(k)]
    return s[f] + (s[c] - s[f]) * (k - f)


@dataclass
class SLO:
    ttft_s: float = 2.0
    itl_s: float = 0.050


def summarize(records: list[ReqRecord], window: tuple[float, float], slo: SLO, by: str = "arrival") -> dict:
    """``by="arrival"``: the cohort is every request that ARRIVED in the
    window; it counts toward goodput once it has finished within the SLO
    (a request still unfinished when the run stops has missed it). The run
    must continue past the window (same arrival process) long enough for
    the cohort to finish. Counting by arrival makes the figure independent
    of where the window's edges fall relative to each server's latency: two
    servers that both meet the SLO on the same trace get the same goodput.

    ``by="finish"``: the cohort is every request that FINISHED in the window
    (a server whose backlog drains into the window is credited with it)."""
    t0, t1 = window
    dur = max(1e-9, t1 - t0)
    if by == "arrival":
        cohort = [r for r in records if t0 <= r.arrival < t1]
        done = [r for r in cohort if r.finish is not None]
    elif by == "finish":
        done = [r for r in records if r.finish is not None and t0 <= r.finish <= t1]
        cohort = done
    else:
        raise ValueError(f"unknown cohort {by!r}")
    good = 0
    ttfts, itls = [], []
    for r in done:
        tt = r.ttft
        it = r.itls()
        ttfts.append(tt)
        itls.extend(it)
        p99 = percentile(it, 99) if it else 0.0
        if tt is not None and tt <= slo.ttft_s and p99 <= slo.itl_s:
            good += 1
    out_tokens = sum(1 for r in records for t in r.token_times if t0 <= t <= t1)
    prompt_tokens = sum(r.prompt_len for r in done)
    cached_tokens = sum(r.cached_len for r in done)
    return {
        "window_s": dur,
        "cohort": len(cohort),
        "completed": len(done),
        "slo_met": good,
        "goodput_rps": good / dur,
        "throughput_rps": len(done) / dur,
        "output_tok_s": out_tokens / dur,
        "ttft_p50_s": percentile(ttfts, 50),
        "ttft_p99_s": percentile(ttfts, 99),
        "itl_p50_s": percentile(itls, 50),
        "itl_p99_s": percentile(itls, 99),
        "slo_attainment": good / max(1, len(cohort)),
        "prefix_hit_rate": cached_tokens / max(1, prompt_tokens),
    }


def cohort(records: list[ReqRecord], window: tuple[float, float], by: str = "arrival") -> list[ReqRecord]:
    """The finished requests that :func:`summarize` counts for ``window``."""
    t0, t1 = window
    if by == "arrival":
        return [r for r in records if t0 <= r.arrival < t1 and r.finish is not None]
    return [r for r in records if r.finish is not None and t0 <= r.finish <= t1]
