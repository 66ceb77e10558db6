"""Tensor-parallel group of one node: NCCL for the baseline collectives and a
symmetric NVLink region for the fused ones.

``TPComm`` owns, per rank, one cudaMalloc'd region exported with CUDA IPC
and mapped by every peer:

    [parity 0 | parity 1] x [source rank 0 .. world-1] x [max_rows, hidden] bf16
    arrival counters [parity][source rank] (u32)

The row-parallel GEMMs of a layer (attention output, MLP down) alternate
parities. ``gemm_allreduce_add_rmsnorm`` runs

    ib_gemm_bf16_push   (tcgen05 GEMM whose epilogue stores every tile into
                         this rank's slot on every rank, then signals)
    ib_ar_add_rmsnorm   (waits for every rank's arrival, sums the partials
                         in fp32, adds the residual, RMSNorm)

for up to ``max_rows`` tokens (decode and small prefill steps). Larger
batches, up to ``max_rows_rs``, take the two-shot form when it moves fewer
bytes (world >= 4, or ``INFERA_TP_TWO_SHOT=1``):

    ib_gemm_*_push_rs     (the epilogue stores each 128-row block of the
                           output only into its owner's slot, owner =
                           block % world: a reduce-scatter fused into the GEMM)
    ib_ar_add_rmsnorm_rs  (the owner sums its blocks' partials, adds the
                           residual, RMSNorm, and stores the normalised rows
                           into every rank's x buffer: the all-gather)
    ib_tp_wait            (bounded wait for every owner's rows)

Per rank that sends 2 (W-1)/W of the activation over NVLink instead of the
one-shot's (W-1) times it. The residual stays valid only on each row
block's owner, which is the only rank that reads it again. Anything larger
takes the baseline: GEMM, ``torch.distributed.all_reduce`` (NCCL), add +
RMSNorm. Reference counterpart: the engines' TP all-reduce
(vLLM / SGLang over RCCL on the reference's hardware); the fused form is
this framework's.
"""

from __future__ import annotations

import ctypes
import os

import torch
import torch.distributed as dist

from infera_b200.ops import _native
from infera_b200.ops import kernels as K

MAX_PEERS = 8
FLAG_BYTES = 256  # 2 parities x 8 sources x 4 B, padded


class TPComm:
    def __init__(self, rank: int, world: int, device: torch.device, hidden: int, max_rows: int = 256,
                 nccl_group=None, gloo_group=None, fused: bool = True, max_rows_rs: int = 0,
                 two_shot: bool | None = None):
        if world > MAX_PEERS:
            raise ValueError(f"tensor parallel size {world} > {MAX_PEERS}")
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.hidden = hidden
        self.max_rows = max_rows
        self.cap = max(max_rows, max_rows_rs)
        if two_shot is None:
            two_shot = world >= 4 or os.environ.get("INFERA_TP_TWO_SHOT") == "1"
        self.two_shot = two_shot and max_rows_rs > max_rows
        self.x_round = [0, 0]
        self.nccl = nccl_group
        self.gloo = gloo_group
        self.fused = fused and self.device.type == "cuda" and os.environ.get("INFERA_TP_FUSED", "1") != "0"
        self.base = None
        self.peers: list[int] = []
        # vocab-parallel LM head: GEMM whose epilogue stores each rank's column
        # block into every rank's full logits buffer (ensure_gather)
        self.g_base = None
        self.g_peers: list[int] = []
        self.g_opened: list[int] = []
        self.g_rows = self.g_cols = 0
        if self.fused:
            self._setup_symmetric()

    # ------------------------------------------------------------------ setup
    def _exchange(self, base: int) -> tuple[list[int], list[int]]:
        """CUDA-IPC handles of ``base`` all round: (every rank's mapping of
        its region, the mappings this rank opened)."""
        lib = _native.kernels()
        handle = (ctypes.c_char * 64)()
        _native.check(lib.ib_ipc_handle(ctypes.c_void_p(base), handle), "ib_ipc_handle")
        allh = [bytes(handle)]
        if self.world > 1:
            allh = [None] * self.world
            dist.all_gather_object(allh, bytes(handle), group=self.gloo)
        peers, opened = [], []
        for r, h in enumerate(allh):
            if r == self.rank:
                peers.append(base)
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(h)
            _native.check(lib.ib_ipc_open(buf, ctypes.byref(p)), f"ib_ipc_open(rank {r})")
            peers.append(p.value)
            opened.append(p.value)
        return peers, opened

    def ensure_gather(self, rows: int, cols: int) -> None:
        """Allocate (once, on every rank at the same point: it exchanges IPC
        handles) the symmetric [rows, cols] bf16 buffer of the fused GEMM ->
        all-gather, plus its arrival counter."""
        if not self.fused or self.world == 1 or self.g_base is not None:
            return
        lib = _native.kernels()
        ptr = ctypes.c_void_p()
        _native.check(lib.ib_sym_alloc(rows * cols * 2 + FLAG_BYTES, ctypes.byref(ptr)), "ib_sym_alloc")
        self.g_base = ptr.value
        self.g_rows, self.g_cols = rows, cols
        self.g_peers, self.g_opened = self._exchange(self.g_base)
        self.g_ctr = torch.zeros(4, dtype=torch.int32, device=self.device)   # done_ctr, consumed
        if self.world > 1:
            dist.barrier(group=self.gloo)

    def _setup_symmetric(self) -> None:
        lib = _native.kernels()
        self.slot_elems = self.cap * self.hidden
        self.data_bytes = 2 * self.world * self.slot_elems * 2
        self.x_bytes = self.slot_elems * 2 if self.two_shot else 0   # per parity
        total = self.data_bytes + FLAG_BYTES + 2 * self.x_bytes
        ptr = ctypes.c_void_p()
        _native.check(lib.ib_sym_alloc(total, ctypes.byref(ptr)), "ib_sym_alloc")
        self.base = ptr.value
        handle = (ctypes.c_char * 64)()
        _native.check(lib.ib_ipc_handle(ctypes.c_void_p(self.base), handle), "ib_ipc_handle")
        mine = bytes(handle)
        if self.world > 1:
            allh = [None] * self.world
            dist.all_gather_object(allh, mine, group=self.gloo)
        else:
            allh = [mine]
        self._opened = []
        for r, h in enumerate(allh):
            if r == self.rank:
                self.peers.append(self.base)
                continue
            p = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(h)
            _native.check(lib.ib_ipc_open(buf, ctypes.byref(p)), f"ib_ipc_open(rank {r})")
            self.peers.append(p.value)
            self._opened.append(p.value)
        # local counters: done_ctr[2], consumed[2], fin_ctr[2]
        self.ctr = torch.zeros(8, dtype=torch.int32, device=self.device)
        if self.world > 1:
            dist.barrier(group=self.gloo)

    def close(self) -> None:
        if self.base is None:
            return
        lib = _native.kernels()
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.gloo)
        for p in self._opened + self.g_opened:
            lib.ib_ipc_close(ctypes.c_void_p(p))
        lib.ib_sym_free(ctypes.c_void_p(self.base))
        self.base = None
        if self.g_base is not None:
            lib.ib_sym_free(ctypes.c_void_p(self.g_base))
            self.g_base = None

    # ------------------------------------------------------------------ ops
    def _slot(self, rank_base: int, parity: int, src: int) -> int:
        return rank_base + ((parity * self.world + src) * self.slot_elems) * 2

    def _flag(self, rank_base: int, parity: int, src: int) -> int:
        return rank_base + self.data_bytes + (parity * MAX_PEERS + src) * 4

    def _xflag(self, rank_base: int, parity: int) -> int:
        return rank_base + self.data_bytes + 128 + parity * 4

    def _xbuf(self, rank_base: int, parity: int) -> int:
        return rank_base + self.data_bytes + FLAG_BYTES + parity * self.x_bytes

    def uses_fused(self, rows: int) -> bool:
        return self.fused and rows <= self.max_rows

    def uses_two_shot(self, rows: int) -> bool:
        return self.fused and self.two_shot and self.max_rows < rows <= self.cap

    def gemm_allreduce_add_rmsnorm(self, x: torch.Tensor, w: torch.Tensor, h: torch.Tensor, norm_w: torch.Tensor,
                                   eps: float, out: torch.Tensor, parity: int, tmp: torch.Tensor | None = None
                                   ) -> torch.Tensor:
        """h += all_reduce(x @ w.T); out = rmsnorm(h) * norm_w (h updated in place)."""
        M, Kd = x.shape
        N = w.shape[0]
        if self.uses_two_shot(M):
            return self._two_shot(x, w, h, norm_w, eps, out, parity)
        if not self.uses_fused(M):
            o = K.linear(x, w, out=None if tmp is None else tmp[:M])
            if self.world > 1:
                dist.all_reduce(o, group=self.nccl)
            return K.add_rmsnorm(o, h, norm_w, eps, out=out)
        assert N == self.hidden and h.is_contiguous() and out.is_contiguous()
        lib = _native.kernels()
        sc = K.scratch(x.device)
        peer_out = (ctypes.c_void_p * MAX_PEERS)(*[self._slot(self.peers[d], parity, self.rank)
                                                   for d in range(self.world)])
        peer_flag = (ctypes.c_void_p * MAX_PEERS)(*[self._flag(self.peers[d], parity, self.rank)
                                                    for d in range(self.world)])
        ctr = self.ctr.data_ptr()
        stream = K._stream()
        if isinstance(w, torch.Tensor):
            splits = K._gemm_splits(M, N, Kd, 0)
            ws = sc.ensure_gemm(M * N if splits > 1 else 1)
            rc = lib.ib_gemm_bf16_push(x.data_ptr(), w.data_ptr(), M, N, Kd, x.stride(0), w.stride(0), self.hidden,
                                       self.world, peer_out, peer_flag, ctypes.c_void_p(ctr + 4 * parity),
                                       ws.data_ptr(), sc.status.data_ptr(), stream)
            _native.check(rc, "ib_gemm_bf16_push")
        else:  # fp8 block-scaled weight: quantise the activation, same push epilogue
            from infera_b200.ops import fp8

            q, sf = fp8.quant_act(x)
            splits = fp8._splits(M, N, Kd)
            ws = sc.ensure_gemm(M * N if splits > 1 else 1)
            rc = lib.ib_gemm_fp8_push(q.data_ptr(), sf.data_ptr(), sf.stride(0), w.q.data_ptr(), w.sf.data_ptr(), M,
                                      N, Kd, q.stride(0), w.q.stride(0), self.hidden, self.world, peer_out, peer_flag,
                                      ctypes.c_void_p(ctr + 4 * parity), ws.data_ptr(), sc.status.data_ptr(), stream)
            _native.check(rc, "ib_gemm_fp8_push")
        rc = lib.ib_ar_add_rmsnorm(ctypes.c_void_p(self._slot(self.base, parity, 0)), self.slot_elems, self.hidden,
                                   ctypes.c_void_p(self._flag(self.base, parity, 0)),
                                   ctypes.c_void_p(ctr + 4 * (2 + parity)), ctypes.c_void_p(ctr + 4 * (4 + parity)),
                                   self.world, M, N, h.data_ptr(), norm_w.data_ptr(), eps, out.data_ptr(),
                                   sc.status.data_ptr(), stream)
        _native.check(rc, "ib_ar_add_rmsnorm")
        K._count(3 if splits > 1 else 2)
        return out

    def _two_shot(self, x, w, h, norm_w, eps, out, parity: int) -> torch.Tensor:
        M, Kd = x.shape
        N = w.shape[0]
        assert N == self.hidden and h.is_contiguous() and out.is_contiguous()
        lib = _native.kernels()
        sc = K.scratch(x.device)
        peer_out = (ctypes.c_void_p * MAX_PEERS)(*[self._slot(self.peers[d], parity, self.rank)
                                                   for d in range(self.world)])
        peer_flag = (ctypes.c_void_p * MAX_PEERS)(*[self._flag(self.peers[d], parity, self.rank)
                                                    for d in range(self.world)])
        ctr = self.ctr.data_ptr()
        stream = K._stream()
        if isinstance(w, torch.Tensor):
            splits = K._gemm_splits(M, N, Kd, 0)
            ws = sc.ensure_gemm(M * N if splits > 1 else 1)
            rc = lib.ib_gemm_bf16_push_rs(x.data_ptr(), w.data_ptr(), M, N, Kd, x.stride(0), w.stride(0),
                                          self.hidden, self.world, peer_out, peer_flag,
                                          ctypes.c_void_p(ctr + 4 * parity), ws.data_ptr(), sc.status.data_ptr(),
                                          stream)
            _native.check(rc, "ib_gemm_bf16_push_rs")
        else:
            from infera_b200.ops import fp8

            q, sf = fp8.quant_act(x)
            splits = fp8._splits(M, N, Kd)
            ws = sc.ensure_gemm(M * N if splits > 1 else 1)
            rc = lib.ib_gemm_fp8_push_rs(q.data_ptr(), sf.data_ptr(), sf.stride(0), w.q.data_ptr(), w.sf.data_ptr(),
                                         M, N, Kd, q.stride(0), w.q.stride(0), self.hidden, self.world, peer_out,
                                         peer_flag, ctypes.c_void_p(ctr + 4 * parity), ws.data_ptr(),
                                         sc.status.data_ptr(), stream)
            _native.check(rc, "ib_gemm_fp8_push_rs")
        x_peer = (ctypes.c_void_p * MAX_PEERS)(*[self._xbuf(self.peers[d], parity) for d in range(self.world)])
        x_flag = (ctypes.c_void_p * MAX_PEERS)(*[self._xflag(self.peers[d], parity) for d in range(self.world)])
        rc = lib.ib_ar_add_rmsnorm_rs(ctypes.c_void_p(self._slot(self.base, parity, 0)), self.slot_elems, self.hidden,
                                      ctypes.c_void_p(self._flag(self.base, parity, 0)),
                                      ctypes.c_void_p(ctr + 4 * (2 + parity)), ctypes.c_void_p(ctr + 4 * (4 + parity)),
                                      self.world, self.rank, M, N, h.data_ptr(), norm_w.data_ptr(), eps, x_peer,
                                      x_flag, sc.status.data_ptr(), stream)
        _native.check(rc, "ib_ar_add_rmsnorm_rs")
        self.x_round[parity] += 1
        target = (self.x_round[parity] * self.world) & 0xFFFFFFFF
        rc = lib.ib_tp_wait(ctypes.c_void_p(self._xflag(self.base, parity)), target, sc.status.data_ptr(), stream)
        _native.check(rc, "ib_tp_wait")
        out.copy_(self._x_view(parity, M))
        K._count(4 if splits > 1 else 3)
        return out

    def _x_view(self, parity: int, rows: int) -> torch.Tensor:
        from infera_b200.parallel.symmem import _View

        class _B:
            pass

        b = _B()
        b.ptr = self._xbuf(self.base, parity)
        t = torch.as_tensor(_View(b, (rows, self.hidden), "<i2"), device=self.device).view(torch.bfloat16)
        return t

    def uses_fused_gather(self, rows: int, cols_local: int, w) -> bool:
        return (self.g_base is not None and rows <= self.g_rows and cols_local * self.world == self.g_cols
                and isinstance(w, torch.Tensor))

    def gemm_allgather_cols(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[M, K] @ w_local[n, K].T on every rank -> [M, world * n] on every
        rank (rank r's columns at r * n): one tcgen05 GEMM whose epilogue
        stores each output tile straight into every rank's symmetric buffer
        at this rank's column block over NVLink, then a bounded wait for the
        other ranks' blocks (target kept on the device: graph-safe). Falls
        back to GEMM + NCCL all-gather when the buffer does not fit."""
        M, Kd = x.shape
        n = w.shape[0]
        if not self.uses_fused_gather(M, n, w):
            return self.all_gather_cols(K.linear(x, w), out=out)
        lib = _native.kernels()
        sc = K.scratch(x.device)
        flag_off = self.g_rows * self.g_cols * 2
        peer_out = (ctypes.c_void_p * MAX_PEERS)(*[self.g_peers[d] + self.rank * n * 2 for d in range(self.world)])
        peer_flag = (ctypes.c_void_p * MAX_PEERS)(*[self.g_peers[d] + flag_off for d in range(self.world)])
        splits = K._gemm_splits(M, n, Kd, 0)
        ws = sc.ensure_gemm(M * n if splits > 1 else 1)
        stream = K._stream()
        ctr = self.g_ctr.data_ptr()
        rc = lib.ib_gemm_bf16_push(x.data_ptr(), w.data_ptr(), M, n, Kd, x.stride(0), w.stride(0), self.g_cols,
                                   self.world, peer_out, peer_flag, ctypes.c_void_p(ctr), ws.data_ptr(),
                                   sc.status.data_ptr(), stream)
        _native.check(rc, "ib_gemm_bf16_push")
        rc = lib.ib_tp_wait_next(ctypes.c_void_p(self.g_base + flag_off), ctypes.c_void_p(ctr + 4), self.world,
                                 sc.status.data_ptr(), stream)
        _native.check(rc, "ib_tp_wait_next")
        K._count(3 if splits > 1 else 2)
        full = self._raw_view(self.g_base, (self.g_rows, self.g_cols))[:M]
        if out is not None:
            out.copy_(full)
            return out
        return full

    def _raw_view(self, ptr: int, shape) -> torch.Tensor:
        from infera_b200.parallel.symmem import _View

        class _B:
            pass

        b = _B()
        b.ptr = ptr
        return torch.as_tensor(_View(b, shape, "<i2"), device=self.device).view(torch.bfloat16)

    def all_gather_cols(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """[M, n] per rank -> [M, world * n] (rank r's columns at r*n), NCCL."""
        if self.world == 1:
            return x
        M, n = x.shape
        stacked = torch.empty(self.world * M, n, dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(stacked, x.contiguous(), group=self.nccl)
        full = stacked.view(self.world, M, n).permute(1, 0, 2).reshape(M, self.world * n)
        if out is not None:
            out.copy_(full)
            return out
        return full

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            dist.all_reduce(x, group=self.nccl)
        return x
