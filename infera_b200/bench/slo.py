"""Latency records and SLO goodput.

A request meets its SLO when its time to first token is within the TTFT
bound and the 99th percentile of its inter-token latencies is within the
ITL bound. Goodput = SLO-meeting requests completed in the window per
second. The fleet-level p99 TTFT / p99 ITL over all requests and tokens and
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


def summarize(records: list[ReqRecord], window: tuple[float, float], slo: SLO) -> dict:
    t0, t1 = window
    dur = max(1e-9, t1 - t0)
    done = [r for r in records if r.finish is not None and t0 <= r.finish <= t1]
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
        "completed": len(done),
        "slo_met": good,
        "goodput_rps": good / dur,
        "throughput_rps": len(done) / dur,
        "output_tok_s": out_tokens / dur,
        "ttft_p50_s": percentile(ttfts, 50),
        "ttft_p99_s": percentile(ttfts, 99),
        "itl_p50_s": percentile(itls, 50),
        "itl_p99_s": percentile(itls, 99),
        "slo_attainment": good / max(1, len(done)),
        "prefix_hit_rate": cached_tokens / max(1, prompt_tokens),
    }
