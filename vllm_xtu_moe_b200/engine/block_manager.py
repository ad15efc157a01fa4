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
    """``prefix_caching``: full blocks are keyed by a hash chained over their tokens and the
    tokens before them; a new request starts from the longest cached chain of its prompt
    (those blocks shared, reference-counted, never written again) and computes the rest.
    A released block whose hash is known stays cached until its slot is needed (least
    recently released first)."""

    def __init__(self, num_blocks: int, block_size: int, max_seqs: int, swa_blocks: int = 0, window: int = 0,
                 prefix_caching: bool = False):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.free = list(range(num_blocks - 1, -1, -1))
        self.free_slots = list(range(max_seqs - 1, -1, -1))
        self.prefix_caching = prefix_caching
        self.hash_to_block: dict[int, int] = {}
        self.block_hash: dict[int, int] = {}
        self.refs: dict[int, int] = {}
        self.cached_free: dict[int, None] = {}      # released blocks with a hash, oldest first
        self.prefix_hits = 0                        # prompt tokens served from cached blocks
        self.window = window if swa_blocks > 0 else 0
        self.swa_free = list(range(swa_blocks - 1, -1, -1))
        self.num_swa_blocks = swa_blocks

    def blocks_needed(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    # ------------------------------------------------------------------ prefix caching
    def _hashes(self, tokens: list[int], n_blocks: int) -> list[int]:
        bs, h, out = self.block_size, 0, []
        for j in range(n_blocks):
            h = hash((h, tuple(tokens[j * bs:(j + 1) * bs])))
            out.append(h)
        return out

    def _take(self) -> int:
        """A block for new data: a never-cached free block first, else the oldest cached one."""
        if self.free:
            return self.free.pop()
        b = next(iter(self.cached_free))
        del self.cached_free[b]
        del self.hash_to_block[self.block_hash.pop(b)]
        return b

    def _available(self) -> int:
        return len(self.free) + len(self.cached_free)

    def match_prefix(self, req) -> int:
        """Start a new request from its longest cached prefix (at least its last prompt
        token is left to compute).  Returns the prompt tokens served from the cache."""
        if not self.prefix_caching or req.blocks:
            return 0
        n_full = (len(req.prompt) - 1) // self.block_size
        got = []
        for h in self._hashes(req.prompt, n_full):
            b = self.hash_to_block.get(h)
            if b is None:
                break
            got.append(b)
        for b in got:
            if self.refs.get(b, 0) == 0:
                self.cached_free.pop(b, None)
            self.refs[b] = self.refs.get(b, 0) + 1
        req.blocks = got
        req.num_computed = len(got) * self.block_size
        req._hash_chain = self._hashes(req.prompt, len(got))
        self.prefix_hits += req.num_computed
        return req.num_computed

    def _register_full_blocks(self, req) -> None:
        """Hash the request's blocks whose tokens are all computed (they will not change);
        the chain is extended incrementally, so a step hashes only its new full blocks."""
        n_full = min(req.num_computed // self.block_size, len(req.blocks))
        chain = req.__dict__.setdefault("_hash_chain", [])
        if n_full <= len(chain):
            return
        bs = self.block_size
        toks = req.all_tokens
        h = chain[-1] if chain else 0
        for j in range(len(chain), n_full):
            h = hash((h, tuple(toks[j * bs:(j + 1) * bs])))
            chain.append(h)
            b = req.blocks[j]
            if b in self.block_hash or h in self.hash_to_block:
                continue
            self.block_hash[b] = h
            self.hash_to_block[h] = b

    def _swa_keep_from(self, req) -> int:
        """First logical block the request's next step can still read in a window layer."""
        first_query = min(req.num_computed, max(0, req.total_len - 1))
        return max(0, first_query - self.window + 1) // self.block_size

    def _swa_need(self, req, upto_tokens: int) -> int:
        lo, hi = self._swa_keep_from(req), self.blocks_needed(upto_tokens)
        return sum(1 for j in range(lo, hi) if j not in req.swa_blocks)

    def can_allocate(self, req, upto_tokens: int) -> bool:
        """Would ``ensure(req, upto_tokens)`` succeed?  (Changes nothing.)"""
        if self.blocks_needed(upto_tokens) - len(req.blocks) > self._available():
            return False
        if self.window:
            keep = self._swa_keep_from(req)
            releasable = sum(1 for j in req.swa_blocks if j < keep)
            return self._swa_need(req, upto_tokens) <= len(self.swa_free) + releasable
        return True

    def ensure(self, req, upto_tokens: int) -> bool:
        need = self.blocks_needed(upto_tokens) - len(req.blocks)
        if need > self._available():
            return False
        if self.prefix_caching:
            self._register_full_blocks(req)
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
            b = self._take()
            self.refs[b] = 1
            req.blocks.append(b)
        return True

    def acquire_slot(self, req) -> bool:
        if req.slot >= 0:
            return True
        if not self.free_slots:
            return False
        req.slot = self.free_slots.pop()
        return True

    def release(self, req) -> None:
        if self.prefix_caching:
            self._register_full_blocks(req)
        for b in reversed(req.blocks):
            n = self.refs.get(b, 1) - 1
            if n > 0:
                self.refs[b] = n
                continue
            self.refs.pop(b, None)
            if b in self.block_hash:
                self.cached_free[b] = None       # kept for reuse until its slot is needed
            else:
                self.free.append(b)
        req.blocks = []
        req.__dict__.pop("_hash_chain", None)
        self.swa_free.extend(req.swa_blocks.values())
        req.swa_blocks = {}
        if req.slot >= 0:
            self.free_slots.append(req.slot)
            req.slot = -1

    @property
    def num_free(self) -> int:
        return self._available()
