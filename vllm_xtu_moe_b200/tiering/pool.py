"""GPU-resident hot-expert pool of one layer (the reference's ``LayerPool``,
vllm_xiaotu_moe/expert_pool.py:139-448, rebuilt on this framework's kernels).

* ``nslots`` expert slots are allocated once, before the KV cache is sized, and are
  never freed or resized afterwards.
* ``slotmap[e]`` (device int32): slot of expert e, or -1 when e is served by the CPU
  tier.  The route-split kernel turns each step's top-k ids into pool-slot ids and CPU
  ids with it and counts hits per expert on the device (graph-capturable, no syncs).
* Every ``window`` steps, ``maybe_adapt`` reads the hit counts once (one D2H), asks
  ``plan_swap`` for (evict, load), copies the loaded experts from the host copy into the
  evicted slots on a side stream, waits for the copies, and only then flips the slot
  map entries -- so a step never sees a half-loaded slot.
"""
from __future__ import annotations

import torch

from ..ops import moe as M
from .host import HostExperts, alloc_expert_slots
from .policy import plan_swap, pool_hits


class LayerPool:
    def __init__(self, host: HostExperts, experts: list[int], device, *, window: int = 0, hyst: float = 0.25,
                 maxswap: int = 0):
        self.host = host
        self.E = host.E
        self.nslots = len(experts)
        self.window, self.hyst, self.maxswap = window, hyst, maxswap
        self.slots = alloc_expert_slots(host.fmt, self.nslots, host.H, host.I, device)
        self.expert_of = list(experts)
        sm = torch.full((self.E,), -1, dtype=torch.int32)
        for s, e in enumerate(experts):
            sm[e] = s
        self.slotmap = sm.to(device)
        self.hits = torch.zeros(self.E, dtype=torch.int32, device=device)
        self.steps = 0
        self.swaps_in = 0
        self.hit_pairs = self.total_pairs = 0    # pairs counted at past window ends
        self.side = torch.cuda.Stream(device=device)
        for s, e in enumerate(experts):
            self._load(e, s)
        self.side.synchronize()

    def nbytes(self) -> int:
        return self.nslots * self.host.expert_bytes()

    def _load(self, e: int, s: int) -> None:
        self.host.copy_slot(e, self.slots, s, self.side)

    def hit_counts(self) -> tuple[int, int]:
        """(pairs served by the pool, all routed pairs) since the pool was built (synchronises)."""
        h, t = pool_hits(self.hits.cpu().tolist(), self.expert_of)
        return self.hit_pairs + h, self.total_pairs + t

    def maybe_adapt(self, preserve_oldest: bool = False) -> tuple[list[int], list[int]]:
        """Called by the host once per step (outside graph capture)."""
        self.steps += 1
        if self.window <= 0 or self.nslots == 0 or self.steps % self.window:
            return [], []
        counts_t = self.hits.cpu()
        self.hits.zero_()
        counts = {e: int(c) for e, c in enumerate(counts_t.tolist()) if c}
        h, t = pool_hits(counts, self.expert_of)
        self.hit_pairs += h
        self.total_pairs += t
        evict, load = plan_swap(self.expert_of, counts, self.nslots, hyst=self.hyst, maxswap=self.maxswap,
                                preserve_oldest=preserve_oldest)
        if not evict:
            return [], []
        slots = [self.expert_of.index(v) for v in evict]
        # stop routing evicted experts to their slots before the slots are overwritten
        for v in evict:
            self.slotmap[v] = -1
        self.side.wait_stream(torch.cuda.current_stream())
        for e, s in zip(load, slots):
            self._load(e, s)
        self.side.synchronize()
        for e, s in zip(load, slots):       # flip the table last
            self.expert_of[s] = e
            self.slotmap[e] = s
        self.swaps_in += len(load)
        return evict, load
