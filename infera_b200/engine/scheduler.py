"""Continuous-batching scheduler with chunked prefill.

Each step packs, within ``max_batched_tokens``:
  1. one token for every running sequence that is decoding;
  2. the next chunk of every running sequence still in prefill;
  3. new sequences from the waiting queue (FCFS), each with as large a
     first chunk as the budget allows, while pages and sequence slots last.

A decoding sequence that cannot get a page preempts the most recently
admitted running sequence (its pages are freed and it re-enters the waiting
queue at the front; its prompt plus generated tokens are recomputed, with
any surviving prefix pages reused through the prefix cache).

Reference parity: the reference relies on vLLM's / SGLang's schedulers; the
router-visible behaviour it depends on (prefix-cache hits announced through
KV events, in-flight counts for drain) is reproduced here.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field

from infera_b200.engine.block_manager import BlockManager
from infera_b200.engine.request import Request, Status


@dataclass
class ScheduledChunk:
    req: Request
    start: int          # first position computed this step
    num_tokens: int
    is_decode: bool
    needs_logits: bool  # the chunk ends at the last known token -> sample


@dataclass
class SchedulerOutput:
    prefills: list[ScheduledChunk] = field(default_factory=list)
    decodes: list[ScheduledChunk] = field(default_factory=list)
    preempted: list[Request] = field(default_factory=list)

    @property
    def num_tokens(self) -> int:
        return sum(c.num_tokens for c in self.prefills) + len(self.decodes)

    @property
    def empty(self) -> bool:
        return not self.prefills and not self.decodes


class Scheduler:
    def __init__(self, block_manager: BlockManager, max_num_seqs: int = 256, max_batched_tokens: int = 4096,
                 max_model_len: int = 32768, watermark_pages: int = 0, long_prefill_threshold: int = 0,
                 mixed_prefill_tokens: int = 0):
        self.bm = block_manager
        self.max_num_seqs = max_num_seqs
        self.max_batched_tokens = max_batched_tokens
        self.max_model_len = max_model_len
        self.watermark = watermark_pages
        # a single sequence's chunk is capped so that one long prompt cannot
        # occupy the whole budget while decode latency suffers (0: no cap)
        self.long_prefill_threshold = long_prefill_threshold
        # prompt tokens per step while sequences are decoding (0: no cap)
        self.mixed_prefill_tokens = mixed_prefill_tokens
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        # PD decode side: admitted requests waiting for their pushed KV
        self.parked: dict[str, Request] = {}
        self.on_park = None  # fn(request, pages to receive, skip_tokens, n_tokens)
        # KV-tier promotes in flight: admitted requests whose prefix pages a
        # tier is copying in (asynchronously); on_tier_load(request, pages,
        # chained hashes) starts one
        self.loading: dict[str, Request] = {}
        self.on_tier_load = None
        self.free_rows: list[int] = list(range(max_num_seqs - 1, -1, -1))

    # ------------------------------------------------------------------
    def add(self, req: Request) -> None:
        self.waiting.append(req)

    def num_unfinished(self) -> int:
        return len(self.waiting) + len(self.running) + len(self.parked) + len(self.loading)

    def resume_loaded(self, r: Request) -> None:
        """A tier promote for ``r`` completed (the caller registered what
        landed): the request runs, or - aborted meanwhile - its pages, which
        the copies were writing, are released only now."""
        if self.loading.pop(r.request_id, None) is None:
            return
        if r.status == Status.FINISHED_ABORTED:
            self._release(r)
            return
        r.status = Status.RUNNING
        self.running.append(r)

    def resume_parked(self, r: Request, pushed_ok: bool) -> None:
        """The pushed KV arrived (prompt minus its last token now cached) or
        the push failed (the request computes its prompt itself)."""
        if self.parked.pop(r.request_id, None) is None:
            return
        if pushed_ok:
            r.num_computed = max(r.num_computed, len(r.prompt_token_ids) - 1)
        r.status = Status.RUNNING
        self.running.append(r)

    def abort(self, request_id: str) -> Request | None:
        r = self.loading.get(request_id)
        if r is not None:
            # the promote is still writing its pages: released when it lands
            r.status = Status.FINISHED_ABORTED
            return r
        r = self.parked.pop(request_id, None)
        if r is not None:
            self._release(r)
            r.status = Status.FINISHED_ABORTED
            return r
        for i, r in enumerate(self.running):
            if r.request_id == request_id:
                self.running.pop(i)
                self._release(r)
                r.status = Status.FINISHED_ABORTED
                return r
        for r in list(self.waiting):
            if r.request_id == request_id:
                self.waiting.remove(r)
                r.status = Status.FINISHED_ABORTED
                return r
        return None

    def _release(self, r: Request) -> None:
        if r.blocks is not None:
            self.bm.free(r.blocks)
            r.blocks = None
        if r.table_row >= 0:
            self.free_rows.append(r.table_row)
            r.table_row = -1
        r.pages_synced = 0

    def finish(self, r: Request, status: Status, hold_blocks: bool = False):
        """``hold_blocks``: keep the pages referenced (returned) for a KV push."""
        r.status = status
        if r in self.running:
            self.running.remove(r)
        if r.blocks is not None:
            # make everything computed so far reusable by later turns
            self.bm.commit_full_pages(r.blocks, r.all_token_ids(), r.num_computed)
        held = None
        if hold_blocks:
            held, r.blocks = r.blocks, None
        self._release(r)
        return held

    def _preempt(self, victim: Request, out: SchedulerOutput) -> None:
        self.running.remove(victim)
        if victim.blocks is not None:
            self.bm.commit_full_pages(victim.blocks, victim.all_token_ids(), victim.num_computed)
        self._release(victim)
        victim.status = Status.WAITING
        victim.num_computed = 0
        victim.num_preemptions += 1
        victim.prompt_hashes = None
        self.waiting.appendleft(victim)
        out.preempted.append(victim)

    # ------------------------------------------------------------------
    def schedule(self) -> SchedulerOutput:
        out = SchedulerOutput()
        budget = self.max_batched_tokens
        ps = self.bm.page_size
        # While sequences are decoding, every step is one of their inter-token
        # gaps: prefill chunks joining it are capped so that the step stays
        # near the decode-step time (the cap does not apply to steps with no
        # decodes, which run prompts at the full budget).
        n_dec = sum(1 for r in self.running
                    if r.num_tokens - r.num_computed == 1 and len(r.output_token_ids) > 0)
        pbudget = budget
        if n_dec and self.mixed_prefill_tokens:
            pbudget = min(budget, n_dec + self.mixed_prefill_tokens)

        # 1 + 2: running sequences (oldest first)
        i = 0
        while i < len(self.running):
            r = self.running[i]
            pending = r.num_tokens - r.num_computed
            if pending <= 0:
                i += 1
                continue
            is_decode = pending == 1 and len(r.output_token_ids) > 0
            if is_decode:
                n = 1
            else:
                # decodes still to come in this pass keep their token
                n = min(pending, pbudget - n_dec)
            if self.long_prefill_threshold and not is_decode:
                n = min(n, self.long_prefill_threshold)
            if n <= 0:
                i += 1
                continue
            while not self.bm.ensure_capacity(r.blocks, r.num_computed + n):
                victim = self.running[-1]
                if victim is r:
                    # nothing else to take pages from: this one waits
                    self._preempt(r, out)
                    r = None
                    break
                if victim.num_tokens - victim.num_computed == 1 and len(victim.output_token_ids) > 0:
                    n_dec -= 1
                self._preempt(victim, out)
            if r is None:
                if is_decode:
                    n_dec -= 1
                continue
            chunk = ScheduledChunk(r, r.num_computed, n, is_decode, r.num_computed + n == r.num_tokens)
            (out.decodes if is_decode else out.prefills).append(chunk)
            budget -= n
            pbudget -= n
            if is_decode:
                n_dec -= 1
            i += 1
            if budget <= 0:
                break
        budget = min(budget, pbudget)

        # 3: admit waiting sequences
        while self.waiting and budget > 0 and self.free_rows and len(self.running) < self.max_num_seqs:
            r = self.waiting[0]
            toks = r.all_token_ids()
            total = len(toks)
            if total >= self.max_model_len:
                self.waiting.popleft()
                r.status = Status.FINISHED_LENGTH
                r.finish_time = None
                out.preempted.append(r)  # reported as finished by the engine
                continue
            if r.prompt_hashes is None:
                from infera_b200.utils.hashing import chain_hashes

                r.prompt_hashes = chain_hashes(toks, ps)
            sb = self.bm.allocate_prompt(toks, total, r.prompt_hashes)
            if sb is None or not self.bm.can_allocate(0, self.watermark):
                if sb is not None:
                    self.bm.free(sb)
                break
            self.waiting.popleft()
            r.blocks = sb
            r.num_computed = sb.num_cached_tokens
            if r.num_preemptions == 0:
                r.num_cached_prompt_tokens = sb.num_cached_tokens
            r.table_row = self.free_rows.pop()
            r.pages_synced = 0
            tl, sb.tier_load = sb.tier_load, None
            if tl is not None and self.on_tier_load is not None and r.remote_room is None:
                # a tier holds the next blocks of the prompt: park the request
                # until the asynchronous promote has copied them in
                r.status = Status.WAITING
                r.tier_start = tl[0]
                self.loading[r.request_id] = r
                self.on_tier_load(r, sb.pages[tl[0]:tl[0] + tl[1]], r.prompt_hashes[tl[0]:tl[0] + tl[1]])
                continue
            if r.remote_room is not None and self.on_park is not None and r.num_preemptions == 0:
                # PD decode: the prefill instance pushes the prompt's KV
                # (all but the last token) into the pages beyond the prefix
                # this instance already caches; wait for it
                n_tok = len(r.prompt_token_ids) - 1
                skip = min(sb.num_cached_tokens, n_tok) // ps
                n_pages = (n_tok + ps - 1) // ps
                r.status = Status.WAITING
                self.parked[r.request_id] = r
                self.on_park(r, sb.pages[skip:n_pages], skip * ps, n_tok)
                continue
            r.status = Status.RUNNING
            self.running.append(r)
            pending = total - r.num_computed
            n = min(pending, budget)
            if self.long_prefill_threshold:
                n = min(n, self.long_prefill_threshold)
            out.prefills.append(ScheduledChunk(r, r.num_computed, n, False, r.num_computed + n == total))
            budget -= n
        return out
