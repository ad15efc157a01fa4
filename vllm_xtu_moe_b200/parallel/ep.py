"""Expert-parallel MoE layer over the GPUs of one node.

Rank r holds experts [r*El, (r+1)*El) of E (kernel layout, see ``ops.moe``).  Two
implementations of one layer call on a batch of this rank's tokens:

``EPMoE.forward`` (the product): the dispatch and the combine are fused with the
grouped GEMMs over NVLink peer memory (``csrc/comm/ep_moe.cu`` + the peer-store
epilogue of ``xtu_grouped_gemm_ex``):
    route (count all-gather + barrier)  ->  dispatch (P2P row stores)  ->  barrier
    ->  gate/up GEMM + SwiGLU on the received rows  ->  down GEMM whose epilogue
    stores each weighted row into its source rank's slot buffer  ->  barrier
    ->  per-token combine (+ shared expert) on every rank.
No host synchronisation: buffers are sized for the worst case (every pair of every
rank routed to one owner), the launch sequence is fixed, and it can be captured in
a CUDA graph.

``EPMoE.forward_collective`` (the baseline, also runs on gloo/CPU): counts and rows
travel through ``all_to_all_single`` (NCCL on GPUs), the local experts run on the
received rows, and the weighted rows come back through a second all-to-all — the
shape of the reference's expert-parallel paths (vllm_xiaotu_moe/hybrid_model.py:
254-326, 2019-2044), which reduce [T, H] partials instead.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import _native as N
from ..ops import gemm as G
from ..ops import moe as M
from .comm import PeerGroup


def shard_experts(fmt: str, w13: torch.Tensor, w2: torch.Tensor, s13, s2, rank: int, world: int,
                  device) -> M.ExpertWeights:
    """Checkpoint-layout experts of all E -> this rank's El experts in kernel layout."""
    E = w13.shape[0]
    El = E // world
    sl = slice(rank * El, (rank + 1) * El)
    pick = lambda t: None if t is None else t[sl].to(device)
    return M.prepare_experts(fmt, pick(w13), pick(w2), pick(s13), pick(s2))


class EPMoE:
    def __init__(self, experts: M.ExpertWeights, num_experts: int, top_k: int, max_tokens: int,
                 pg: PeerGroup | None = None, group=None, act_limit: float = 0.0):
        self.ex = experts
        self.E = num_experts
        self.K = top_k
        self.El = experts.num_experts
        self.H = experts.hidden
        self.I = experts.inter
        self.max_tokens = max_tokens
        self.act_limit = act_limit
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        assert self.El * self.world == self.E, "experts must divide evenly over the ranks"
        self.pair_cap = max_tokens * top_k
        self.recv_cap = self.world * self.pair_cap
        self.pg = pg
        if pg is not None:
            self._alloc_fused()

    # ------------------------------------------------------------------ fused path
    @staticmethod
    def heap_bytes(num_experts: int, top_k: int, hidden: int, max_tokens: int, world: int) -> int:
        pc = max_tokens * top_k
        rc = world * pc
        return PeerGroup.heap_bytes_for(world * num_experts * 4, rc * hidden * 2, rc * 4, rc * 4, pc * hidden * 2)

    def _alloc_fused(self):
        pg, d = self.pg, self.pg.device
        self.cnt = pg.alloc((self.world, self.E), torch.int32)
        self.xp = pg.alloc((self.recv_cap, self.H), torch.bfloat16)
        self.rsrc = pg.alloc((self.recv_cap,), torch.int32)
        self.rw = pg.alloc((self.recv_cap,), torch.float32)
        self.slots = pg.alloc((self.pair_cap, self.H), torch.bfloat16)
        self.send_base = torch.zeros(self.E, dtype=torch.int32, device=d)
        self.cursor = torch.zeros(self.E, dtype=torch.int32, device=d)
        self.seg = torch.zeros(self.El + 1, dtype=torch.int32, device=d)
        self.h = torch.empty(self.recv_cap, self.I, dtype=torch.bfloat16, device=d)
        self.mx = G.max_mtiles(self.recv_cap, self.El)
        self.tiles = torch.empty(self.mx * 4, dtype=torch.int32, device=d)
        self.ntiles = torch.zeros(1, dtype=torch.int32, device=d)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                shared: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x.shape
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the layer's capacity ({self.max_tokens})")
        pg = self.pg
        s = N.stream_ptr(x.device)
        st = pg.status.data_ptr()
        ids = ids.to(torch.int32).contiguous()
        weights = weights.float().contiguous()
        N.call("xtu_ep_route", ids.data_ptr(), T * self.K, self.E, self.El, self.rank, self.world, self.cnt.ptr(),
               pg.flags.ptr(), pg.epoch.data_ptr(), self.send_base.data_ptr(), self.cursor.data_ptr(),
               self.seg.data_ptr(), st, pg.timeout_ns, s)
        N.call("xtu_ep_dispatch", ids.data_ptr(), weights.data_ptr(), T, self.K, self.El, self.E, self.rank,
               x.data_ptr(),
               H, x.stride(0), self.send_base.data_ptr(), self.cursor.data_ptr(), self.xp.ptr(), self.rsrc.ptr(),
               self.rw.ptr(), self.pair_cap, s)
        pg.barrier()                                    # every owner holds its rows
        ex = self.ex
        fp8 = ex.fmt == "fp8"
        tiles = G.build_mtiles(self.seg, self.recv_cap, self.tiles, self.ntiles)
        G.grouped_gemm(self.xp.local, ex.w13, self.seg, w_scale=ex.s13 if fp8 else None, epilogue=G.EPI_SWIGLU,
                       out=self.h, act_limit=self.act_limit, tiles=tiles)
        t, cnt, mx = tiles
        N.call("xtu_grouped_gemm_ex", self.h.data_ptr(), ex.w2.data_ptr(), N.ptr(ex.s2 if fp8 else None), None,
               1 if fp8 else 0, self.slots.local.data_ptr(), H, self.recv_cap, H, self.I, self.El, t.data_ptr(),
               cnt.data_ptr(), mx, G.EPI_BF16, self.rw.local.data_ptr(), self.rsrc.local.data_ptr(),
               float(self.act_limit), 1.0, 0.0, self.slots.ptr(), self.pair_cap, st, s)
        pg.barrier()                                    # every source holds its weighted rows
        ws_like = _SlotView(self.slots.local, H)
        return M.moe_combine(ws_like, ids, 0, self.E, shared=shared, out=out)

    # ------------------------------------------------------------------ collective baseline
    def forward_collective(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                           shared: torch.Tensor | None = None) -> torch.Tensor:
        T, H = x.shape
        K, W, El = self.K, self.world, self.El
        flat = ids.reshape(-1).long()
        dest = flat // El
        order = torch.argsort(dest, stable=True)
        send_counts = torch.bincount(dest, minlength=W)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        rows = x[order // K].contiguous()
        meta = torch.stack([flat[order].float(), weights.reshape(-1)[order].float()], 1).contiguous()
        r_rows = torch.empty(sum(rc), H, dtype=x.dtype, device=x.device)
        r_meta = torch.empty(sum(rc), 2, dtype=torch.float32, device=x.device)
        dist.all_to_all_single(r_rows, rows, rc, sc, group=self.group)
        dist.all_to_all_single(r_meta, meta, rc, sc, group=self.group)
        R = r_rows.shape[0]
        lo = self.rank * El
        r_ids = r_meta[:, 0].round().int().view(R, 1)
        r_w = r_meta[:, 1].contiguous().view(R, 1)
        if R > 0:
            y = M.fused_moe(r_rows, r_ids, r_w, self.ex, lo=lo, act_limit=self.act_limit)
        else:
            y = torch.empty(0, H, dtype=x.dtype, device=x.device)
        back = torch.empty(T * K, H, dtype=y.dtype, device=x.device)
        dist.all_to_all_single(back, y.contiguous(), sc, rc, group=self.group)
        pair_rows = torch.empty_like(back)
        pair_rows[order] = back
        out = pair_rows.view(T, K, H).float().sum(1)
        if shared is not None:
            out = out + shared.float()
        return out.to(x.dtype)


class _SlotView:
    """The two fields of MoEWorkspace that moe_combine reads."""

    def __init__(self, slots: torch.Tensor, hidden: int):
        self.slots = slots
        self.hidden = hidden
