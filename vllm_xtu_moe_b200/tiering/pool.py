"""GPU-resident hot-expert pool of one layer (the reference's ``LayerPool``,
vllm_xiaotu_moe/expert_pool.py:139-448, rebuilt on this framework's kernels).

* ``nslots`` expert slots are allocated once, before the KV cache is sized, and are
  never freed or resized afterwards.
* ``slotmap[e]`` (device int32): slot of expert e, or -1 when e is served by the CPU
  tier.  The route-split kernel turns each step's top-k ids into pool-slot ids and CPU
  ids with it and counts hits per expert on the device (graph-capturable, no syncs).
* Adaptation never blocks the host or the compute stream.  At the end of every
  ``window`` steps, ``maybe_adapt`` queues an asynchronous copy of the hit counts into
  pinned host memory (and re-zeroes them on the device, in stream order); a later call
  whose copy has landed asks ``plan_swap`` for (evict, load), points the evicted experts
  at the CPU tier (slot map -1, in stream order), and copies the loaded experts from the
  host copy into the freed slots on a side stream that first waits for the compute
  stream; a later call whose copies have landed flips the slot map entries of the loaded
  experts -- so a step never sees a half-loaded slot, and the experts in transit are
  served by the CPU tier meanwhile.  ``flush`` completes whatever is in flight.
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
        self._counts_host = None          # pinned landing buffer of the hit counts
        self._counts_ev = None            # their copy in flight
        self._swap_ev = None              # the expert copies of a swap in flight
        self._swap: list[tuple[int, int]] = []
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
        """Called by the host once per step (outside graph capture); returns the (evict,
        load) swap it issued this call, if any."""
        self._finish_swap()
        self.steps += 1
        if self.window <= 0 or self.nslots == 0:
            return [], []
        if self.steps % self.window == 0 and self._counts_ev is None:
            main = torch.cuda.current_stream()
            if self._counts_host is None:
                self._counts_host = torch.empty(self.E, dtype=torch.int32, pin_memory=True)
            self._counts_host.copy_(self.hits, non_blocking=True)
            self.hits.zero_()
            self._counts_ev = torch.cuda.Event()
            self._counts_ev.record(main)
        if self._counts_ev is None or self._swap_ev is not None or not self._counts_ev.query():
            return [], []
        self._counts_ev = None
        counts = {e: int(c) for e, c in enumerate(self._counts_host.tolist()) if c}
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
        self._swap_ev = torch.cuda.Event()
        self._swap_ev.record(self.side)
        self._swap = list(zip(load, slots))
        return evict, load

    def _finish_swap(self, wait: bool = False) -> None:
        """Flip the slot map for a swap whose copies have landed (the table changes last)."""
        if self._swap_ev is None:
            return
        if wait:
            self._swap_ev.synchronize()
        elif not self._swap_ev.query():
            return
        for e, s in self._swap:
            self.expert_of[s] = e
            self.slotmap[e] = s
        self.swaps_in += len(self._swap)
        self._swap_ev, self._swap = None, []

    def flush(self) -> None:
        """Complete the swap in flight (the slot map then matches ``expert_of``)."""
        self._finish_swap(wait=True)
