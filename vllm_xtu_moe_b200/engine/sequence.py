"""Requests and sampling parameters."""
from __future__ import annotations

import enum
import itertools
from dataclasses import dataclass, field


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0      # 0 = greedy
    top_p: float = 1.0
    top_k: int = 0                # 0 = no top-k filter
    ignore_eos: bool = True
    eos_token_id: int | None = None
    seed: int | None = None
    stop_token_ids: tuple = ()    # finish after any of these tokens (even with ignore_eos)
    logprobs: int | None = None   # return each token's log-probability and this many top alternatives


class Status(enum.Enum):
    WAITING = 0
    PREFILL = 1
    DECODE = 2
    FINISHED = 3


_ids = itertools.count()


@dataclass
class Request:
    prompt: list[int]
    params: SamplingParams
    rid: int = field(default_factory=lambda: next(_ids))
    output: list[int] = field(default_factory=list)
    status: Status = Status.WAITING
    num_computed: int = 0          # tokens whose KV is in the cache
    blocks: list[int] = field(default_factory=list)
    swa_blocks: dict = field(default_factory=dict)   # logical block -> block of the sliding-window pool
    slot: int = -1                 # recurrent-state slot
    # timing (seconds, host clock) for TTFT / TPOT accounting
    t_submit: float = 0.0
    t_first: float = 0.0
    t_done: float = 0.0
    # speculative decoding
    draft: list[int] = field(default_factory=list)
    accepted: int = 0
    proposed: int = 0
    # per output token: (log-probability, {token: log-probability} of the top alternatives)
    logprobs: list = field(default_factory=list)

    @property
    def all_tokens(self) -> list[int]:
        return self.prompt + self.output

    @property
    def total_len(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def prefill_remaining(self) -> int:
        return len(self.prompt) - self.num_computed

    def finished(self) -> bool:
        p = self.params
        if len(self.output) >= p.max_tokens:
            return True
        if not p.ignore_eos and p.eos_token_id is not None and self.output and self.output[-1] == p.eos_token_id:
            return True
        if p.stop_token_ids and self.output and self.output[-1] in p.stop_token_ids:
            return True
        return False
