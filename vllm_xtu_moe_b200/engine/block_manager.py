"""Paged KV-cache block allocation (fixed-size blocks, free list) and
recurrent-state slot allocation."""
from __future__ import annotations


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, max_seqs: int):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free = list(range(num_blocks - 1, -1, -1))
        self.free_slots = list(range(max_seqs - 1, -1, -1))

    def blocks_needed(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    def can_allocate(self, req, upto_tokens: int) -> bool:
        need = self.blocks_needed(upto_tokens) - len(req.blocks)
        return need <= len(self.free)

    def ensure(self, req, upto_tokens: int) -> bool:
        need = self.blocks_needed(upto_tokens) - len(req.blocks)
        if need > len(self.free):
            return False
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
        if req.slot >= 0:
            self.free_slots.append(req.slot)
            req.slot = -1

    @property
    def num_free(self) -> int:
        return len(self.free)
