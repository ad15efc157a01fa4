"""Streamed prefill ring: sub-layer expert tiles copied host -> GPU on a copy stream,
double (or N-) buffered, overlapped with the expert GEMMs of the previous tile.

For a long prefill chunk of a layer whose experts live on the host tier, every
expert is needed, so they are streamed through ``nslots`` GPU slots of ``tile_e``
experts each (``XIAOTU_GPF_STAGE_TILE_E``, default 48; ``XIAOTU_GPF_STAGE_NSLOTS``,
>= 2).  Per tile: the copy stream waits for the slot's ``free`` event, DMAs the
tile's experts from the page-locked host copy and records ``ready``; the compute
stream waits ``ready``, runs permute + grouped GEMMs for the pairs of those experts,
and records ``free``.  One combine at the end sums every pair's slot row.  Slots
are allocated once (``staging_bytes`` is the single source of truth for the VRAM
they take), like the reference's tile ring (vllm_xiaotu_moe/gpu_prefill.py:2911-3095).
"""
from __future__ import annotations

import torch

from ..ops import moe as M
from .host import HostExperts, alloc_expert_slots, expert_slot_bytes


def staging_bytes(fmt: str, H: int, I: int, tile_e: int, nslots: int) -> int:
    return expert_slot_bytes(fmt, H, I) * tile_e * nslots


class ExpertRing:
    def __init__(self, fmt: str, H: int, I: int, tile_e: int, nslots: int, device):
        assert nslots >= 2, "the ring needs at least two slots to overlap copy and compute"
        self.fmt, self.H, self.I, self.tile_e, self.nslots = fmt, H, I, tile_e, nslots
        self.slots = [alloc_expert_slots(fmt, tile_e, H, I, device) for _ in range(nslots)]
        self.ready = [torch.cuda.Event() for _ in range(nslots)]
        self.free = [torch.cuda.Event() for _ in range(nslots)]
        self.copy_stream = torch.cuda.Stream(device=device)
        self.bytes = staging_bytes(fmt, H, I, tile_e, nslots)
        self.copied_bytes = 0

    def run_layer(self, host: HostExperts, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                  ws: M.MoEWorkspace, *, shared=None, act_limit=0.0, out=None, lo: int = 0) -> torch.Tensor:
        """All routed experts of one layer through the ring; returns the combined output.
        ``lo``: global id of the host tier's first expert (pairs outside [lo, lo + E) are
        another rank's)."""
        E = host.E
        main = torch.cuda.current_stream()
        ntiles = (E + self.tile_e - 1) // self.tile_e
        for s in range(self.nslots):
            self.free[s].record(main)
        for t in range(ntiles):
            s = t % self.nslots
            e0, e1 = t * self.tile_e, min(E, (t + 1) * self.tile_e)
            slot = self.slots[s]
            self.copy_stream.wait_event(self.free[s])
            for e in range(e0, e1):
                host.copy_slot(e, slot, e - e0, self.copy_stream)
            self.copied_bytes += (e1 - e0) * host.expert_bytes()
            self.ready[s].record(self.copy_stream)
            main.wait_event(self.ready[s])
            n = e1 - e0
            cut = lambda t: None if t is None else t[:n]
            view = slot if n == self.tile_e else M.ExpertWeights(
                slot.fmt, slot.w13[:n], slot.w2[:n], cut(slot.s13), cut(slot.s2), True, cut(slot.gs13), cut(slot.gs2))
            M.moe_experts_partial(x, ids, weights, view, ws, lo=lo + e0, act_limit=act_limit)
            self.free[s].record(main)
        return M.moe_combine(ws, ids, lo, lo + E, shared=shared, out=out)
