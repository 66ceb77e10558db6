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

The collectives are NCCL's all-to-all over NVLink (gloo on CPU for the
tests). The split sizes need one small host read per layer. Reference
counterpart: the engines' EP MoE (vLLM / SGLang over their a2a backends).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from infera_b200.models.moe import MoELayer
from infera_b200.ops import kernels as K


class EPMoE:
    def __init__(self, full: MoELayer, rank: int, world: int, group=None, device: str | torch.device = "cuda"):
        if full.E % world:
            raise ValueError(f"{full.E} experts do not split over {world} ranks")
        self.rank, self.world, self.group = rank, world, group
        self.E, self.El, self.k = full.E, full.E // world, full.k
        self.full = full
        dev = torch.device(device)
        lo, hi = rank * self.El, (rank + 1) * self.El
        self.gate = full.gate.to(dev)
        self.bias = full.bias.to(dev)
        self.w13 = full.w13[lo:hi].to(dev).contiguous()
        self.w2 = full.w2[lo:hi].to(dev).contiguous()
        self.shared = None if full.shared is None else tuple(t.to(dev) for t in full.shared)
        self.stats = {"sent_rows": 0, "recv_rows": 0}

    def _a2a(self, out: torch.Tensor, inp: torch.Tensor, out_splits=None, in_splits=None) -> None:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def route(self, x: torch.Tensor):
        f = self.full
        logits = K.linear(x, self.gate)
        return K.moe_topk(logits, f.k, f.n_groups, f.topk_groups, self.bias, f.scaling)

    def forward(self, x: torch.Tensor, ids: torch.Tensor | None = None, wts: torch.Tensor | None = None
                ) -> torch.Tensor:
        W, El, H = self.world, self.El, x.shape[1]
        if ids is None:
            ids, wts = self.route(x)
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
            act = K.gemm_grouped(xr, self.w13, loc_off, swiglu=True)
            out_r = K.gemm_grouped(act, self.w2, loc_off)
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
