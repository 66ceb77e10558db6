"""Expert parallelism for the MoE FFN (DeepSeek-V3 / Kimi style, EP = N).

Every rank owns ``E / world`` experts and routes its own tokens (attention
stays data-parallel); one layer's MoE step is

    ids, w   = grouped top-k over all E experts        (ib_moe_topk)
    sorted   = this rank's (token, slot) rows by expert  (ib_moe_permute +
               gather): expert-major = destination-rank-major
    counts   = all-to-all of the per-(rank, local expert) row counts
    dispatch = all-to-all of the rows (variable splits)
    regroup  = [source][local expert] -> [local expert][source]
    experts  = two grouped GEMMs over the local experts (SwiGLU between)
    return   = the inverse regroup and all-to-all
    combine  = weighted sum per token (ib_moe_combine) + shared expert

Two data paths:

* baseline: NCCL all-to-all over NVLink (gloo on CPU for the tests); the
  split sizes need one small host read per layer;
* fused (``fused=True``, GPUs): the counts are all-gathered (NCCL, a few
  KB) and the rows move with this framework's kernels over NVLink peer
  memory - ``ib_ep_dispatch`` stores each sorted row straight into its
  destination's receive buffer at its [local expert][source] place (no
  regroup on the receiver; fp8 experts: the sender quantises and
  ``ib_ep_dispatch_q`` moves e4m3 rows with their scale columns), the up
  projection waits for the arrivals inside its own TMA producer - per
  local expert: the dispatch bumps a counter of expert e on its
  destination once its last row of e has landed, and the up projection
  (``ib_gemm_grouped_wait_ex``) waits on that counter before each of e's
  tiles, so a lightly loaded expert's tiles start before a heavy one's
  rows are in (one round counter with ``INFERA_EP_PER_EXPERT=0``) - and
  the down projection's epilogue
  (``ib_gemm_grouped_push``) stores each expert-output row straight back
  at its source's sorted row; arrival counters with bounded waits
  separate the phases, and nothing is read back to the host.

Reference counterpart: the engines' EP MoE (vLLM / SGLang over their a2a
backends).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

import ctypes

from infera_b200.models.moe import MoELayer
from infera_b200.ops import _native
from infera_b200.ops import kernels as K

# two u32 round counters at 0 / 4, then one u32 arrival counter per local
# expert from byte 64 (up to 240 local experts), padded
FLAGS = 1024
EFLAG_OFF = 64


class _SharedComm:
    """The symmetric buffers of one process's EP layers: every MoE layer of
    a model uses the same receive / return buffers, arrival counters and
    scratch (a DeepSeek-V3 shard has 58 MoE layers; 7.5 GB of buffers each
    would not fit). Sharing is safe because layers run one after another in
    the same order on every rank: a rank starts layer i+1's dispatch only
    after its layer-i wait saw every rank's returns, i.e. after every rank's
    layer-i up projection has read its receive buffer, and a rank's layer
    i+1 return stores into a peer need that peer's layer-i+1 dispatch, which
    its stream issues after its layer-i combine read the return buffer.
    The arrival counters are cumulative, so the round counter is shared."""

    def __init__(self):
        self.users = 0
        self.round = 0


_SHARED: dict[tuple, _SharedComm] = {}


class EPMoE:
    def __init__(self, full: MoELayer, rank: int, world: int, group=None, device: str | torch.device = "cuda",
                 fused: bool = False, max_tokens: int = 256, gloo_group=None):
        if full.E % world:
            raise ValueError(f"{full.E} experts do not split over {world} ranks")
        self.rank, self.world, self.group = rank, world, group
        self.E, self.El, self.k = full.E, full.E // world, full.k
        # routing parameters only: the other ranks' experts are not kept
        self.n_groups, self.topk_groups, self.scaling = full.n_groups, full.topk_groups, full.scaling
        dev = torch.device(device)
        # this rank's experts, relative to the ones the given layer holds
        # (the full layer, or already just this shard)
        lo, hi = rank * self.El - full.lo, (rank + 1) * self.El - full.lo
        if lo < 0 or hi > full.hi - full.lo:
            raise ValueError(f"layer holds experts [{full.lo}, {full.hi}), rank {rank} needs "
                             f"[{rank * self.El}, {(rank + 1) * self.El})")
        self.gate = full.gate.to(dev)
        self.bias = full.bias.to(dev)
        self.fp8 = getattr(full, "fp8", False)
        whole = (lo, hi) == (0, full.hi - full.lo)
        if self.fp8:  # stacked e4m3 experts: rows of experts lo..hi-1
            self.F = full.F
            self.w13 = (full.w13 if whole else full.w13.rows(lo * 2 * full.F, hi * 2 * full.F)).to(dev)
            self.w2 = (full.w2 if whole else full.w2.rows(lo * full.H, hi * full.H)).to(dev)
        else:
            self.w13 = full.w13[lo:hi].to(dev).contiguous()
            self.w2 = full.w2[lo:hi].to(dev).contiguous()
        self.shared = None if full.shared is None else tuple(t.to(dev) for t in full.shared)
        self.stats = {"sent_rows": 0, "recv_rows": 0}
        import os

        self.per_expert = os.environ.get("INFERA_EP_PER_EXPERT", "1") != "0"
        self.device = dev
        self.fused = fused and dev.type == "cuda"
        if self.fused:
            self._setup_symmetric(max_tokens * full.k * world, full.H, gloo_group)

    # ------------------------------------------------------------------ fused path
    def _setup_symmetric(self, max_rows: int, H: int, gloo_group) -> None:
        lib = _native.kernels()
        self.max_rows, self.H = max_rows, H
        self.buf_bytes = max_rows * H * 2
        # fp8 experts: the dispatched rows are e4m3 (first half of the
        # receive buffer) with their scale columns [H/128, max_rows] here
        self.sf_bytes = ((H // 128) * max_rows + 15) // 16 * 16 if self.fp8 else 0
        key = (self.device.index, self.world, self.E, max_rows, H, self.fp8, id(gloo_group))
        sh = _SHARED.get(key)
        if sh is not None:
            self._shared = sh
            sh.users += 1
            for name in ("base", "peers", "ctr", "local_done", "counts_all", "offs", "row_map"):
                setattr(self, name, getattr(sh, name))
            if self.El * 4 > FLAGS - EFLAG_OFF:
                self.per_expert = False
            return
        total = FLAGS + 2 * self.buf_bytes + self.sf_bytes
        p = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native.check(lib.ib_sym_alloc(total, ctypes.byref(p)), "ib_sym_alloc")
            self.base = p.value
            h = (ctypes.c_char * 64)()
            _native.check(lib.ib_ipc_handle(ctypes.c_void_p(self.base), h), "ib_ipc_handle")
        allh = [None] * self.world
        dist.all_gather_object(allh, bytes(h), group=gloo_group)
        self.peers = []
        for r, hb in enumerate(allh):
            if r == self.rank:
                self.peers.append(self.base)
                continue
            q = ctypes.c_void_p()
            buf = (ctypes.c_char * 64).from_buffer_copy(hb)
            with torch.cuda.device(self.device):
                _native.check(lib.ib_ipc_open(buf, ctypes.byref(q)), f"ib_ipc_open(rank {r})")
            self.peers.append(q.value)
        self.ctr = torch.zeros(4, dtype=torch.int32, device=self.device)  # done counters of the two phases
        if self.El * 4 > FLAGS - EFLAG_OFF:
            self.per_expert = False
        # per-expert rows stored so far this round (zeroed by the dispatch)
        self.local_done = torch.zeros(self.E, dtype=torch.int32, device=self.device)
        W, E = self.world, self.E
        self.counts_all = torch.zeros(W * E, dtype=torch.int32, device=self.device)
        self.offs = torch.zeros(E + self.El + 1 + W * E, dtype=torch.int32, device=self.device)
        self.row_map = torch.zeros(max_rows, dtype=torch.int32, device=self.device)
        sh = _SharedComm()
        sh.users = 1
        for name in ("base", "peers", "ctr", "local_done", "counts_all", "offs", "row_map"):
            setattr(sh, name, getattr(self, name))
        _SHARED[key] = sh
        self._shared = sh
        dist.barrier(group=gloo_group)

    def _local_done(self):
        return ctypes.c_void_p(self.local_done.data_ptr()) if self.per_expert else None

    def _recv_view(self, base: int) -> int:
        return base + FLAGS

    def _ret_view(self, base: int) -> int:
        return base + FLAGS + self.buf_bytes

    def _sf_view(self, base: int) -> int:
        return base + FLAGS + 2 * self.buf_bytes

    def _tensor_at(self, ptr: int, rows: int) -> torch.Tensor:
        from infera_b200.parallel.symmem import _View

        class _Buf:
            pass

        b = _Buf()
        b.ptr = ptr
        t = torch.as_tensor(_View(b, (rows, self.H), "<i2"), device=self.device).view(torch.bfloat16)
        return t

    def _forward_fused(self, x: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor) -> torch.Tensor:
        lib = _native.kernels()
        W, E, El, H = self.world, self.E, self.El, x.shape[1]
        sc = K.scratch(x.device)
        stream = K._stream()
        offsets, row_of_slot, token_of_row = K.moe_permute(ids, E)
        xs = K.gather_rows(x, token_of_row)
        R = xs.shape[0]
        counts = (offsets[1:] - offsets[:-1]).contiguous()
        dist.all_gather_into_tensor(self.counts_all, counts, group=self.group)
        dst_off = self.offs[:E]
        loc_off = self.offs[E:E + El + 1]
        src_off = self.offs[E + El + 1:]
        _native.check(lib.ib_ep_offsets(self.counts_all.data_ptr(), W, E, self.rank, dst_off.data_ptr(),
                                        loc_off.data_ptr(), src_off.data_ptr(), stream), "ib_ep_offsets")
        self._shared.round += 1
        target = self._shared.round * W
        recv_peers = (ctypes.c_void_p * 8)(*[self._recv_view(b) for b in self.peers])
        flagA = (ctypes.c_void_p * 8)(*[b for b in self.peers])
        eflags = (ctypes.c_void_p * 8)(*[b + EFLAG_OFF for b in self.peers]) if self.per_expert else None
        ctr = self.ctr.data_ptr()
        bn = K.grouped_bn(R, El)
        if self.fp8:
            from infera_b200.ops import fp8

            bn = min(192, max(32, ((bn + 31) // 32) * 32))
            # the sender quantises (half the bytes cross NVLink) and the
            # rows land with their scales where the up projection reads them
            q, qsf = fp8.quant_act(xs)
            sf_peers = (ctypes.c_void_p * 8)(*[self._sf_view(b) for b in self.peers])
            _native.check(lib.ib_ep_dispatch_q_ex(q.data_ptr(), R, H, qsf.data_ptr(), qsf.stride(0), H // 128,
                                                  offsets.data_ptr(), E, W, dst_off.data_ptr(), recv_peers, sf_peers,
                                                  self.max_rows, flagA, eflags, self._local_done(),
                                                  ctypes.c_void_p(ctr), stream), "ib_ep_dispatch_q_ex")
            w13, w13sf, ldw13 = self.w13.q.data_ptr(), self.w13.sf.data_ptr(), self.w13.q.stride(0)
            a13, sf13 = self._recv_view(self.base), self._sf_view(self.base)
            n13 = self.w13.q.shape[0] // El
        else:
            _native.check(lib.ib_ep_dispatch_ex(xs.data_ptr(), R, H, offsets.data_ptr(), E, W, dst_off.data_ptr(),
                                                recv_peers, flagA, eflags, self._local_done(), ctypes.c_void_p(ctr),
                                                stream), "ib_ep_dispatch_ex")
            w13, w13sf, ldw13 = self.w13.data_ptr(), None, self.w13.stride(1)
            a13, sf13 = self._recv_view(self.base), None
            n13 = self.w13.shape[1]
        # up projection (SwiGLU) over the received rows; its TMA producer and
        # scale stagers wait for the dispatch's arrivals themselves
        tab, num, cap = K.grouped_tiles(loc_off, El, n13, bn, self.max_rows)
        act = torch.empty(self.max_rows, n13 // 2, dtype=torch.bfloat16, device=x.device)
        wflag = self.base + (EFLAG_OFF if self.per_expert else 0)
        _native.check(lib.ib_gemm_grouped_wait_ex(a13, sf13, self.max_rows, w13, w13sf, act.data_ptr(), self.max_rows,
                                                  n13, H, El, H, ldw13, act.stride(0), 1,
                                                  tab.data_ptr(), num.data_ptr(), bn, cap, ctypes.c_void_p(wflag),
                                                  target, 1 if self.per_expert else 0, 0, sc.status.data_ptr(),
                                                  stream), "ib_gemm_grouped_wait_ex")
        # down projection whose epilogue stores each expert-output row straight
        # into its source's return buffer (the return all-to-all fused in)
        _native.check(lib.ib_ep_row_map(self.counts_all.data_ptr(), W, E, self.rank, loc_off.data_ptr(),
                                        src_off.data_ptr(), self.max_rows, self.row_map.data_ptr(), stream),
                      "ib_ep_row_map")
        ret_peers = (ctypes.c_void_p * 8)(*[self._ret_view(b) for b in self.peers])
        flagB = (ctypes.c_void_p * 8)(*[b + 4 for b in self.peers])
        if self.fp8:
            a_q, a_sf = fp8.quant_act(act)
            w2q, w2sf, sf_ld = self.w2.q, self.w2.sf.data_ptr(), a_sf.stride(0)
            a_ptr, sfa_ptr, lda = a_q.data_ptr(), a_sf.data_ptr(), a_q.stride(0)
        else:
            w2q, w2sf, sf_ld = self.w2, None, 0
            a_ptr, sfa_ptr, lda = act.data_ptr(), None, act.stride(0)
        tab, num, cap = K.grouped_tiles(loc_off, El, H, bn, self.max_rows)
        _native.check(lib.ib_gemm_grouped_push(a_ptr, sfa_ptr, sf_ld, w2q.data_ptr(), w2sf, self.max_rows, H,
                                               act.shape[1], El, lda, w2q.stride(-2), H, tab.data_ptr(),
                                               num.data_ptr(), bn, cap, self.row_map.data_ptr(), W, ret_peers, flagB,
                                               ctypes.c_void_p(ctr + 4), sc.status.data_ptr(), stream),
                      "ib_gemm_grouped_push")
        _native.check(lib.ib_ep_wait(ctypes.c_void_p(self.base + 4), target, sc.status.data_ptr(), stream),
                      "ib_ep_wait")
        ret = self._tensor_at(self._ret_view(self.base), self.max_rows)
        K._count(6)
        self.stats["sent_rows"] += R
        y = K.moe_combine(ret, row_of_slot, wts)
        if self.shared is not None:
            y = y + K.linear(K.linear(x, self.shared[0], swiglu=True), self.shared[1])
        return y

    def _experts(self, xr: torch.Tensor, loc_off: torch.Tensor, bn: int | None = None) -> torch.Tensor:
        """This rank's experts over rows grouped by local expert."""
        if self.fp8:
            from infera_b200.ops import fp8

            act = fp8.gemm_fp8_grouped(xr, self.w13, self.El, loc_off, swiglu=True, bn=bn)
            return fp8.gemm_fp8_grouped(act, self.w2, self.El, loc_off, bn=bn)
        act = K.gemm_grouped(xr, self.w13, loc_off, swiglu=True, bn=bn)
        return K.gemm_grouped(act, self.w2, loc_off, bn=bn)

    def close(self) -> None:
        if getattr(self, "base", None):
            sh = self._shared
            self.base = None
            sh.users -= 1
            if sh.users > 0:
                return
            for k, v in list(_SHARED.items()):
                if v is sh:
                    del _SHARED[k]
            lib = _native.kernels()
            torch.cuda.synchronize(self.device)
            for r, p in enumerate(sh.peers):
                if r != self.rank:
                    lib.ib_ipc_close(ctypes.c_void_p(p))
            lib.ib_sym_free(ctypes.c_void_p(sh.base))

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def route(self, x: torch.Tensor):
        logits = K.linear(x, self.gate)
        return K.moe_topk(logits, self.k, self.n_groups, self.topk_groups, self.bias, self.scaling)

    def forward(self, x: torch.Tensor, ids: torch.Tensor | None = None, wts: torch.Tensor | None = None
                ) -> torch.Tensor:
        W, El, H = self.world, self.El, x.shape[1]
        if ids is None:
            ids, wts = self.route(x)
        if self.fused:
            if x.shape[0] * self.k * W > self.max_rows:
                raise ValueError("more tokens than the symmetric buffers hold (raise max_tokens)")
            return self._forward_fused(x, ids, wts)
        offsets, row_of_slot, token_of_row = K.moe_permute(ids, self.E)
        xs = K.gather_rows(x, token_of_row)
        send_counts = (offsets[1:] - offsets[:-1]).to(torch.int64).view(W, El).contiguous()
        recv_counts = torch.empty_like(send_counts)
        self._a2a(recv_counts, send_counts)
        sc = send_counts.cpu()
        rc = recv_counts.cpu()
        send_splits = sc.sum(1).tolist()
        recv_splits = rc.sum(1).tolist()
        recv = torch.empty(sum(recv_splits), H, dtype=x.dtype, device=x.device)
        self._a2a(recv, xs, recv_splits, send_splits)
        # regroup [src][expert] -> [expert][src] so each local expert's rows are contiguous
        src_base = torch.zeros(W, El, dtype=torch.int64)
        if W * El:
            flat = rc.reshape(-1)
            src_base.view(-1)[1:] = torch.cumsum(flat, 0)[:-1]
        exp_order = rc.t().contiguous()                       # [El, W]
        dst_base = torch.zeros(El, W, dtype=torch.int64)
        dst_base.view(-1)[1:] = torch.cumsum(exp_order.reshape(-1), 0)[:-1]
        perm = torch.empty(int(rc.sum()), dtype=torch.int64)  # position in recv -> position in grouped
        for s in range(W):
            for e in range(El):
                n = int(rc[s, e])
                if n:
                    perm[src_base[s, e]:src_base[s, e] + n] = torch.arange(dst_base[e, s], dst_base[e, s] + n)
        perm_d = perm.to(x.device)
        xr = torch.empty_like(recv)
        xr[perm_d] = recv
        loc_off = torch.zeros(El + 1, dtype=torch.int32)
        loc_off[1:] = torch.cumsum(exp_order.sum(1), 0).to(torch.int32)
        loc_off = loc_off.to(x.device)
        if xr.shape[0]:
            out_r = self._experts(xr, loc_off)
            back = out_r[perm_d]
        else:
            back = torch.empty(0, H, dtype=x.dtype, device=x.device)
        ret = torch.empty(xs.shape[0], H, dtype=x.dtype, device=x.device)
        self._a2a(ret, back.contiguous(), send_splits, recv_splits)
        self.stats["sent_rows"] += xs.shape[0]
        self.stats["recv_rows"] += recv.shape[0]
        y = K.moe_combine(ret, row_of_slot, wts)
        if self.shared is not None:
            y = y + K.linear(K.linear(x, self.shared[0], swiglu=True), self.shared[1])
        return y
