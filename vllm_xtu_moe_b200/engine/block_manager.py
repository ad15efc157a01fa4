"""Paged KV-cache block allocation (fixed-size blocks, free list) and
recurrent-state slot allocation.

Models with sliding-window layers get a second, small pool for those layers
(``swa_blocks`` blocks, ``window`` tokens): a request keeps a sliding-window block only
while some query it still has to compute can see it.  Before each step, blocks wholly
below ``num_computed - window + 1`` (the lowest key the step's first query sees) go back
to the pool, so a sequence holds about window / block_size + its current chunk of them,
whatever its length; the global-attention layers keep the whole context as before."""
from __future__ import annotations


def swa_pool_blocks(max_seqs: int, window: int, block_size: int, max_batched_tokens: int) -> int:
    """Blocks a sliding-window pool needs: per sequence the window's history (+1 partly
    used block, +1 for the chunk's boundary) and, over all sequences, one step's tokens."""
    return max_seqs * ((window + block_size - 1) // block_size + 2) + (max_batched_tokens + block_size - 1) // block_size


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, max_seqs: int, swa_blocks: int = 0, window: int = 0):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free = list(range(num_blocks - 1, -1, -1))
        self.free_slots = list(range(max_seqs - 1, -1, -1))
        self.window = window if swa_blocks > 0 else 0
        self.swa_free = list(range(swa_blocks - 1, -1, -1))
        self.num_swa_blocks = swa_blocks

    def blocks_needed(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    def _swa_keep_from(self, req) -> int:
        """First logical block the request's next step can still read in a window layer."""
        first_query = min(req.num_computed, max(0, req.total_len - 1))
        return max(0, first_query - self.window + 1) // self.block_size

    def _swa_need(self, req, upto_tokens: int) -> int:
        lo, hi = self._swa_keep_from(req), self.blocks_needed(upto_tokens)
        return sum(1 for j in range(lo, hi) if j not in req.swa_blocks)

    def can_allocate(self, req, upto_tokens: int) -> bool:
        """Would ``ensure(req, upto_tokens)`` succeed?  (Changes nothing.)"""
        if self.blocks_needed(upto_tokens) - len(req.blocks) > len(self.free):
            return False
        if self.window:
            keep = self._swa_keep_from(req)
            releasable = sum(1 for j in req.swa_blocks if j < keep)
            return self._swa_need(req, upto_tokens) <= len(self.swa_free) + releasable
        return True

    def ensure(self, req, upto_tokens: int) -> bool:
        need = self.blocks_needed(upto_tokens) - len(req.blocks)
        if need > len(self.free):
            return False
        if self.window:
            keep = self._swa_keep_from(req)
            for j in [j for j in req.swa_blocks if j < keep]:     # out of every future window
                self.swa_free.append(req.swa_blocks.pop(j))
            if self._swa_need(req, upto_tokens) > len(self.swa_free):
                return False
            for j in range(keep, self.blocks_needed(upto_tokens)):
                if j not in req.swa_blocks:
                    req.swa_blocks[j] = self.swa_free.pop()
        for _ in range(max(0, need)):
            req.blocks.append(self.free.pop())
        return True

    def acquire_slot(self, req) -> bool:
        if req.slot >= 0:
            return True
        if not self.free_slots:
            return False
        req.slot = self.free_slots.pop()
        return True

    def release(self, req) -> None:
        self.free.extend(reversed(req.blocks))
        req.blocks = []
        self.swa_free.extend(req.swa_blocks.values())
        req.swa_blocks = {}
        if req.slot >= 0:
            self.free_slots.append(req.slot)
            req.slot = -1

    @property
    def num_free(self) -> int:
        return len(self.free)
