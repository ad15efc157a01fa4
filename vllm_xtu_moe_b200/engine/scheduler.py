"""Continuous-batching scheduler with chunked prefill.

Each step is either a prefill step (chunks of waiting/prefilling requests, up
to ``max_batched_tokens`` tokens in total) or a decode step (every request in
the decode phase, one token each plus any speculative draft tokens).  Prefill
goes first, like the reference's serving setup (vLLM chunked prefill with
MBT 8192, scripts/serve_v41.sh:637-664).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass

from .block_manager import BlockManager
from .sequence import Request, Status


@dataclass
class ScheduledChunk:
    req: Request
    start: int          # first token position of the chunk
    length: int         # tokens in the chunk


@dataclass
class StepPlan:
    is_decode: bool
    chunks: list[ScheduledChunk]

    @property
    def num_tokens(self) -> int:
        return sum(c.length for c in self.chunks)


class Scheduler:
    def __init__(self, blocks: BlockManager, max_batched_tokens: int = 16384, max_seqs: int = 64,
                 num_spec: int = 0):
        self.blocks = blocks
        self.max_batched_tokens = max_batched_tokens
        self.max_seqs = max_seqs
        self.num_spec = num_spec
        self.waiting: deque[Request] = deque()
        self.running: list[Request] = []
        self.finished: list[Request] = []

    def capacity_tokens(self) -> int:
        """Most tokens (prompt + output + one step's drafts) one request may ever hold."""
        return self.blocks.num_blocks * self.blocks.block_size

    def add(self, req: Request) -> None:
        """Queue a request; one that could not fit in the whole KV pool even alone is
        rejected here (it would otherwise wait forever for blocks)."""
        need = len(req.prompt) + req.params.max_tokens + self.num_spec + 1
        if self.blocks.blocks_needed(need) > self.blocks.num_blocks:
            raise ValueError(f"request needs {need} tokens of KV cache; the pool holds {self.capacity_tokens()}")
        self.waiting.append(req)

    def has_work(self) -> bool:
        return bool(self.waiting) or bool(self.running)

    def schedule(self) -> StepPlan | None:
        # 1) prefill chunks (requests already prefilling first, then new ones)
        budget = self.max_batched_tokens
        chunks: list[ScheduledChunk] = []
        blocked = False          # a request already prefilling could not get its next chunk's blocks
        for r in self.running:
            if r.status == Status.PREFILL and budget > 0:
                n = min(r.prefill_remaining, budget)
                if self.blocks.ensure(r, r.num_computed + n):
                    chunks.append(ScheduledChunk(r, r.num_computed, n))
                    budget -= n
                else:
                    blocked = True
        # new requests are admitted only while no admitted one is starved of blocks
        while not blocked and self.waiting and budget > 0 and len(self.running) < self.max_seqs:
            r = self.waiting[0]
            if not self.blocks.acquire_slot(r):
                break
            self.blocks.match_prefix(r)          # prefix caching: skip the cached blocks
            n = min(len(r.prompt) - r.num_computed, budget)
            if not self.blocks.ensure(r, r.num_computed + n):
                self.blocks.release(r)           # give the shared prefix back; retry later
                r.num_computed = 0
                break
            self.waiting.popleft()
            r.status = Status.PREFILL
            self.running.append(r)
            chunks.append(ScheduledChunk(r, r.num_computed, n))
            budget -= n
        if chunks:
            return StepPlan(False, chunks)
        # 2) decode
        dec = [r for r in self.running if r.status == Status.DECODE]
        if not dec:
            pre = [r for r in self.running if r.status == Status.PREFILL]
            if blocked and len(pre) > 1:
                # prompts in prefill hold the pool between them and none can go on: the newest
                # goes back to the queue (its blocks freed, recomputed later); the oldest alone
                # always fits, since add() rejects requests larger than the pool
                self._preempt(pre[-1])
                return self.schedule()
            return None
        out = []
        for r in dec:
            q = 1 + len(r.draft)
            if not self.blocks.ensure(r, r.total_len + q):
                # out of blocks: preempt the newest request (recompute later)
                self._preempt(dec[-1])
                return self.schedule()
            out.append(ScheduledChunk(r, r.total_len - 1, q))
        return StepPlan(True, out)

    def _preempt(self, r: Request) -> None:
        self.running.remove(r)
        self.blocks.release(r)
        r.prompt = r.prompt + r.output
        r.output = []
        r.num_computed = 0
        r.status = Status.WAITING
        self.waiting.appendleft(r)

    def abort(self, rid: int) -> Request | None:
        """Drop request `rid` (waiting or running) and free its blocks; None if unknown."""
        for q in (self.waiting, self.running):
            for r in list(q):
                if r.rid == rid:
                    q.remove(r)
                    self.blocks.release(r)
                    r.status = Status.FINISHED
                    return r
        return None

    def finish(self, r: Request) -> None:
        r.status = Status.FINISHED
        if r in self.running:
            self.running.remove(r)
        self.blocks.release(r)
        self.finished.append(r)
