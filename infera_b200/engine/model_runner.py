"""Turns a scheduler step into one forward pass on the GPU.

Per step the host packs every int32 input (token ids, positions, cache
slots, logits rows, attention metadata, block-table updates, sampling
parameters) into ONE pinned buffer and issues ONE host-to-device copy; the
sampled token ids come back with ONE device-to-host copy. Block tables live
on the device ([max_num_seqs + 1, max_pages], one row per running sequence,
plus a dummy row for graph padding) and only new page ids are scattered in.

Decode-only steps replay a CUDA graph captured for the next larger batch
bucket and the length class of the step's longest sequence (the decode
attention's split count is fixed inside a graph); steps with prefill chunks
run eagerly.
"""

from __future__ import annotations

import bisect
import time
import zlib
from dataclasses import dataclass

import numpy as np
import torch

from infera_b200.engine.scheduler import SchedulerOutput
from infera_b200.models.dense import DenseModel, ForwardBatch
from infera_b200.ops import kernels as K

DEFAULT_GRAPH_SIZES = [1, 2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256]


@dataclass
class StepResult:
    rows: list                  # ScheduledChunk per sampled row
    token_ids: list[int]


class ModelRunner:
    def __init__(self, model: DenseModel, num_pages: int, page_size: int, max_num_seqs: int,
                 max_batched_tokens: int, use_graphs: bool = True, graph_sizes: list[int] | None = None,
                 exportable: bool = False):
        self.model = model
        cfg = model.cfg
        self.cfg = cfg
        self.dev = model.device
        self.page_size = page_size
        self.num_pages = num_pages
        self.max_num_seqs = max_num_seqs
        self.max_tokens = max_batched_tokens + max_num_seqs
        self.max_pages = (cfg.max_model_len + page_size - 1) // page_size
        self.on_gpu = self.dev.type == "cuda"
        # KV cache: [layers, slots, kv_size] for K and for V, zero-initialised so
        # that padding pages always hold finite values
        slots = num_pages * page_size
        shape = (cfg.num_layers, slots, cfg.kv_size)
        # latent (MLA) caches have one channel: v_cache is a placeholder
        v_shape = shape if getattr(cfg, "kv_channels", 2) == 2 else (cfg.num_layers, 1, 1)
        if exportable and self.on_gpu:
            # own cudaMalloc allocations: exportable whole with CUDA IPC
            # (the decode side of a PD pair maps them into prefill processes)
            from infera_b200.parallel.symmem import device_tensor

            self.k_cache, self._k_buf = device_tensor(shape, torch.bfloat16, self.dev)
            self.v_cache, self._v_buf = device_tensor(v_shape, torch.bfloat16, self.dev)
        else:
            self.k_cache = torch.zeros(shape, dtype=torch.bfloat16, device=self.dev)
            self.v_cache = torch.zeros(v_shape, dtype=torch.bfloat16, device=self.dev)
        self.block_table = torch.zeros(max_num_seqs + 1, self.max_pages, dtype=torch.int32, device=self.dev)
        self.dummy_row = max_num_seqs
        self.bufs = model.alloc_buffers(self.max_tokens, max(max_num_seqs, 1))
        # one packed int32 input buffer (host pinned + device)
        self.in_cap = 16 * self.max_tokens + 8 * max_num_seqs + 4 * self.max_pages + 4096
        pin = self.on_gpu
        self.h_in = torch.empty(self.in_cap, dtype=torch.int32, pin_memory=pin)
        self.d_in = torch.empty(self.in_cap, dtype=torch.int32, device=self.dev)
        self.h_out = torch.empty(max(max_num_seqs, 1), dtype=torch.int32, pin_memory=pin)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.forwards = 0
        self.last_logits = None
        self.last_timing = (0.0, 0.0)
        self._t_exec = 0.0
        if self.on_gpu:
            sc = K.scratch(self.dev)
            sc.ensure_gemm(8 * 1024 * 1024)
            max_splits = max(4, K.decode_plan(max_num_seqs, cfg.num_kv_heads, cfg.max_model_len)[0])
            sc.ensure_decode(max_num_seqs * cfg.num_heads * max_splits * 128 + 64 * cfg.num_heads * 64 * 128,
                             max_num_seqs * cfg.num_heads * max_splits + 64 * cfg.num_heads * 64)
        self.graph_sizes = [g for g in (graph_sizes or DEFAULT_GRAPH_SIZES) if g <= max_num_seqs]
        # decode graphs are captured per length class (the longest sequence
        # of the step): the split count of the decode attention is fixed in a
        # graph, and short batches should not launch the empty splits of
        # long ones
        self.len_classes = sorted({c for c in (8192, 16384) if c < cfg.max_model_len} | {cfg.max_model_len})
        self.graphs: dict[int, tuple] = {}
        self.graph_launches: dict[int, int] = {}
        self.use_graphs = use_graphs and self.on_gpu
        if self.use_graphs:
            self._capture_all()

    # ------------------------------------------------------------------ packing
    def _pack(self, sched: SchedulerOutput, bt_updates: tuple[list[int], list[int]]):
        ps = self.page_size
        ids, pos, slots = [], [], []
        logits_rows = []
        sampled = []
        # prefill meta
        q_start, q_len, ctx_len, p_rows = [], [], [], []
        row = 0
        for c in sched.prefills:
            r = c.req
            toks = r.tokens_range(c.start, c.start + c.num_tokens)
            ids.extend(toks)
            ps_arr = np.arange(c.start, c.start + c.num_tokens, dtype=np.int64)
            pos.extend(ps_arr.tolist())
            pages = np.asarray(r.blocks.pages, dtype=np.int64)
            slots.extend((pages[ps_arr // ps] * ps + ps_arr % ps).tolist())
            q_start.append(row)
            q_len.append(c.num_tokens)
            ctx_len.append(c.start + c.num_tokens)
            p_rows.append(r.table_row)
            row += c.num_tokens
            if c.needs_logits:
                logits_rows.append(row - 1)
                sampled.append(c)
        Tp = row
        d_lens, d_rows = [], []
        for c in sched.decodes:
            r = c.req
            p = c.start
            ids.append(r.token_at(p))
            pos.append(p)
            slots.append(r.blocks.pages[p // ps] * ps + p % ps)
            d_lens.append(p + 1)
            d_rows.append(r.table_row)
            logits_rows.append(row)
            sampled.append(c)
            row += 1
        return ids, pos, slots, logits_rows, sampled, Tp, (q_start, q_len, ctx_len, p_rows), (d_lens, d_rows)

    def _sampling_arrays(self, sampled) -> tuple[np.ndarray, np.ndarray]:
        temps = np.zeros(len(sampled), dtype=np.float32)
        seeds = np.zeros(len(sampled), dtype=np.int64)
        for i, c in enumerate(sampled):
            sp = c.req.sampling
            temps[i] = sp.temperature
            # deterministic across processes (tensor-parallel ranks sample alike)
            base = sp.seed if sp.seed is not None else zlib.crc32(c.req.request_id.encode()) & 0x7FFFFFFF
            seeds[i] = base * 1000003 + len(c.req.output_token_ids)
        return temps, seeds

    # ------------------------------------------------------------------ execution
    def idle_forward(self) -> None:
        """One forward over a single padding token (no cache write, reads
        the dummy table row) whose result is dropped: keeps a rank whose
        scheduler has nothing to run in step with the collectives inside the
        model (expert-parallel MoE layers under data-parallel attention)."""
        dev = self.dev
        one = torch.ones(1, dtype=torch.int32, device=dev)
        zero = torch.zeros(1, dtype=torch.int32, device=dev)
        fb = ForwardBatch(token_ids=zero, positions=zero, slots=-one, logits_idx=zero, num_prefill_tokens=0,
                          d_block_table=self.block_table, d_seq_lens=one, d_splits=1, num_decode=1)
        fb.d_bt_rows = torch.full((1,), self.dummy_row, dtype=torch.int32, device=dev)
        self.model.forward(fb, self.k_cache, self.v_cache, None)
        self.forwards += 1

    def execute(self, sched: SchedulerOutput, bt_updates: tuple[list[int], list[int]],
                layer_hook=None) -> StepResult:
        """``layer_hook(layer)``: called by the model right after each
        layer's KV write (forces the eager path)."""
        self.forwards += 1
        self._t_exec = time.perf_counter()
        self._layer_hook = layer_hook
        ids, pos, slots, logits_rows, sampled, Tp, pmeta, dmeta = self._pack(sched, bt_updates)
        T = len(ids)
        S = len(logits_rows)
        temps, seeds = self._sampling_arrays(sampled)
        if Tp == 0 and self.use_graphs and T > 0 and T <= self.graph_sizes[-1] and layer_hook is None:
            toks = self._run_graph(ids, pos, slots, dmeta, temps, seeds, bt_updates)
        else:
            toks = self._run_eager(ids, pos, slots, logits_rows, Tp, pmeta, dmeta, temps, seeds, bt_updates)
        return StepResult(rows=sampled, token_ids=toks[:S])

    def _h2d(self, n: int) -> None:
        if self.on_gpu:
            self.d_in[:n].copy_(self.h_in[:n], non_blocking=True)
            # the copy reads the pinned buffer when the stream reaches it: the
            # next step may refill the buffer only after that (a step that
            # samples nothing - an inner prompt chunk - does not wait for its
            # kernels, so the host can be a step ahead)
            self._h2d_ev = torch.cuda.Event()
            self._h2d_ev.record()
            self.h2d_bytes += 4 * n
        else:
            self.d_in[:n].copy_(self.h_in[:n])

    def _host_in(self) -> np.ndarray:
        """The pinned input buffer, once the previous step's copy of it is done."""
        ev = getattr(self, "_h2d_ev", None)
        if ev is not None:
            ev.synchronize()
            self._h2d_ev = None
        return self.h_in.numpy()

    def _d2h(self, src: torch.Tensor, n: int) -> list[int]:
        if n == 0:
            return []
        if self.on_gpu:
            self.h_out[:n].copy_(src[:n], non_blocking=True)
            t0 = time.perf_counter()
            torch.cuda.current_stream().synchronize()
            # host time spent issuing this step, and waiting for the device
            self.last_timing = (t0 - self._t_exec, time.perf_counter() - t0)
            self.d2h_bytes += 4 * n
            return self.h_out[:n].tolist()
        return src[:n].tolist()

    def _run_eager(self, ids, pos, slots, logits_rows, Tp, pmeta, dmeta, temps, seeds, bt_updates) -> list[int]:
        T, S = len(ids), len(logits_rows)
        q_start, q_len, ctx_len, p_rows = pmeta
        d_lens, d_rows = dmeta
        tiles = K.prefill_tiles(q_len, getattr(self.model, "prefill_tile_rows", None)) if Tp > 0 else []
        upd_idx, upd_val = bt_updates
        parts = [("ids", ids), ("pos", pos), ("slots", slots), ("lidx", logits_rows), ("qs", q_start),
                 ("ql", q_len), ("cl", ctx_len), ("prow", p_rows), ("tiles", [x for t in tiles for x in t]),
                 ("dl", d_lens), ("drow", d_rows), ("ui", upd_idx), ("uv", upd_val),
                 ("temp", temps.view(np.int32).tolist()), ("seed", seeds.view(np.int32).tolist())]
        h = self._host_in()
        off = 0
        views = {}
        for name, arr in parts:
            n = len(arr)
            if name == "seed" and off % 2:
                off += 1
            if n:
                h[off:off + n] = arr
            views[name] = (off, n)
            off += n
        if off > self.in_cap:
            raise RuntimeError("step inputs exceed the packed buffer")
        self._h2d(off)
        d = self.d_in

        def v(name):
            o, n = views[name]
            return d[o:o + n]

        if views["ui"][1]:
            K.scatter_i32(self.block_table, v("ui"), v("uv"))
        fb = ForwardBatch(token_ids=v("ids"), positions=v("pos"), slots=v("slots"), logits_idx=v("lidx"),
                          num_prefill_tokens=Tp)
        fb.layer_hook = getattr(self, "_layer_hook", None)
        if Tp > 0:
            fb.p_q_start, fb.p_q_len, fb.p_ctx_len = v("qs"), v("ql"), v("cl")
            fb.p_block_table = self.block_table
            fb.p_tiles = v("tiles").view(-1, 2)
            fb.p_host_meta = (list(q_len), list(ctx_len))
            fb.p_bt_rows = v("prow")
        B = len(d_lens)
        if B > 0:
            fb.d_block_table = self.block_table
            fb.d_seq_lens = v("dl")
            fb.d_bt_rows = v("drow")
            fb.num_decode = B
            if self.on_gpu:
                fb.d_splits, fb.d_tps = K.decode_plan(B, self.cfg.num_kv_heads, max(d_lens))
        logits = self.model.forward(fb, self.k_cache, self.v_cache, self.bufs)
        self.last_logits = logits
        temp = v("temp").view(torch.float32)
        so, sn = views["seed"]
        seed_t = d[so:so + sn].view(torch.int64)
        out = K.sample(logits, temp, seed_t)
        return self._d2h(out, S)

    # ------------------------------------------------------------------ CUDA graphs
    def _graph_layout(self, B: int) -> dict:
        names = ["ids", "pos", "slots", "lidx", "dl", "drow", "temp"]
        lay = {n: (i * B, B) for i, n in enumerate(names)}
        off = len(names) * B
        off += off % 2
        lay["seed"] = (off, 2 * B)
        lay["_end"] = off + 2 * B
        return lay

    def _graph_inputs(self, B: int):
        lay = self._graph_layout(B)
        base = self.g_in

        def v(name):
            o, n = lay[name]
            return base[o:o + n]

        return lay, v

    def _capture_all(self) -> None:
        # Garbage from earlier engines in this process (graphs, exported
        # caches) frees device memory when it is collected; a collection in
        # the middle of a capture would put cudaFree into it and invalidate
        # the capture. Collect now and keep the collector off until done.
        import gc

        gc.collect()
        gc_on = gc.isenabled()
        gc.disable()
        try:
            self._capture_all_sizes()
        finally:
            if gc_on:
                gc.enable()

    def _capture_all_sizes(self) -> None:
        maxB = self.graph_sizes[-1]
        self.g_in = torch.zeros(self._graph_layout(maxB)["_end"] + 16, dtype=torch.int32, device=self.dev)
        self.g_out = torch.zeros(maxB, dtype=torch.int32, device=self.dev)
        pool = torch.cuda.graph_pool_handle()
        stream = torch.cuda.Stream(self.dev)
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for B in reversed(self.graph_sizes):
                for cls in self.len_classes:
                    self._capture_one(B, cls, pool, stream)
        torch.cuda.current_stream().wait_stream(stream)
        torch.cuda.synchronize()

    def _capture_one(self, B: int, cls: int, pool, stream) -> None:
        lay, v = self._graph_inputs(B)
        # benign placeholder values: every row reads the dummy table row
        self.g_in.zero_()
        v("dl").fill_(1)
        v("drow").fill_(self.dummy_row)
        v("slots").fill_(-1)
        v("lidx").copy_(torch.arange(B, dtype=torch.int32, device=self.dev))
        splits, tps = K.decode_plan(B, self.cfg.num_kv_heads, cls)
        fb = ForwardBatch(token_ids=v("ids"), positions=v("pos"), slots=v("slots"), logits_idx=v("lidx"),
                          num_prefill_tokens=0, d_block_table=self.block_table, d_seq_lens=v("dl"),
                          d_splits=splits, d_tps=tps, num_decode=B)
        fb.d_bt_rows = v("drow")
        so, sn = lay["seed"]

        def run():
            logits = self.model.forward(fb, self.k_cache, self.v_cache, self.bufs)
            K.sample(logits, v("temp").view(torch.float32), self.g_in[so:so + sn].view(torch.int64),
                     out=self.g_out[:B])

        run()  # warm-up outside capture (tensor-map cache, lazy init)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        n0 = K.LAUNCHES[0]
        with torch.cuda.graph(g, pool=pool, stream=stream):
            run()
        self.graph_launches[(B, cls)] = K.LAUNCHES[0] - n0
        self.graphs[(B, cls)] = (g, lay)

    def release_graphs(self) -> None:
        """Drop the captured graphs (a graph holding NCCL calls must be
        released before its process group is destroyed)."""
        if self.graphs:
            torch.cuda.synchronize(self.dev)
            self.graphs.clear()

    def _run_graph(self, ids, pos, slots, dmeta, temps, seeds, bt_updates) -> list[int]:
        B = len(ids)
        Bg = self.graph_sizes[bisect.bisect_left(self.graph_sizes, B)]
        d_lens, d_rows = dmeta
        cls = self.len_classes[min(bisect.bisect_left(self.len_classes, max(d_lens)), len(self.len_classes) - 1)]
        g, lay = self.graphs[(Bg, cls)]
        pad = Bg - B
        h = self._host_in()
        h[: lay["_end"]] = 0

        def put(name, arr, fill):
            o, n = lay[name]
            h[o:o + len(arr)] = arr
            if fill is not None and n > len(arr):
                h[o + len(arr):o + n] = fill

        put("ids", ids, 0)
        put("pos", pos, 0)
        put("slots", slots, -1)
        put("lidx", list(range(Bg)), None)
        put("dl", d_lens, 1)
        put("drow", d_rows, self.dummy_row)
        put("temp", temps.view(np.int32), 0)
        so, _ = lay["seed"]
        h[so:so + 2 * B] = seeds.view(np.int32)
        end = lay["_end"]
        upd_idx, upd_val = bt_updates
        nu = len(upd_idx)
        h[end:end + nu] = upd_idx
        h[end + nu:end + 2 * nu] = upd_val
        self._h2d(end + 2 * nu)
        self.g_in[:end].copy_(self.d_in[:end])
        if nu:
            K.scatter_i32(self.block_table, self.d_in[end:end + nu], self.d_in[end + nu:end + 2 * nu])
        g.replay()
        K.LAUNCHES[0] += self.graph_launches[(Bg, cls)]
        del pad
        return self._d2h(self.g_out, B)
