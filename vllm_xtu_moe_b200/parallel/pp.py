"""Pipeline parallelism: the decoder's layers cut into contiguous stages, one per rank.

Stage r holds layers ``[lo_r, hi_r)`` (their weights, KV caches and recurrent states
only); the first stage also embeds the tokens, the last one applies the final norm, the
LM head and the MTP layers.  Between stages the step's ``(hidden, residual)`` pair
travels as ONE ``[2, T, H]`` tensor by point-to-point send/recv of the process group
(NCCL between GPUs over NVLink, gloo on CPU).  Every rank runs the same scheduler on
the same requests; the last stage broadcasts the sampled token ids so the schedulers
stay in step.

``forward_microbatches`` streams several micro-batches through the stages with
non-blocking sends, so stage r computes micro-batch i + 1 while micro-batch i is in
flight to stage r + 1 (the GPipe forward schedule).

The reference serves with PP = 1 everywhere and has no pipeline kernel of its own;
this is the framework's own stage runtime over the same engine contract as
:class:`models.model.MoETransformer` (``forward`` / ``logits`` / cache allocation).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.model import MoETransformer
from ..ops import basic as B


def stage_bounds(num_layers: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced split: the first ``num_layers % world`` stages take one more."""
    if world > num_layers:
        raise ValueError(f"{world} pipeline stages for {num_layers} layers")
    base, extra = divmod(num_layers, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


class PipelineStage(MoETransformer):
    """One rank's stage of a pipelined model, usable wherever the engine takes a model.

    Built from a full model object (its tensors are shared, not copied; the other
    stages' layers are dropped from this object).  ``group`` defaults to the world."""

    is_pipeline_stage = True

    def __init__(self, full: MoETransformer, rank: int, world: int, group=None,
                 bounds: tuple[int, int] | None = None):
        lo, hi = bounds or stage_bounds(len(full.layers), world, rank)
        last = rank == world - 1
        super().__init__(full.cfg, full.embed_tokens, full.layers[lo:hi], full.norm, full.lm_head,
                         full.mtp if last else [])
        self.act_dtype = full.act_dtype
        self.lo, self.hi = lo, hi
        self.rank, self.world, self.group = rank, world, group
        self.first, self.last = rank == 0, last

    # ------------------------------------------------------------------ peers
    def _peer(self, r: int) -> int:
        return dist.get_global_rank(self.group, r) if self.group is not None else r

    def _recv(self, T: int) -> tuple[torch.Tensor, torch.Tensor]:
        buf = torch.empty(2, T, self.cfg.hidden_size, dtype=self.act_dtype, device=self.device)
        dist.recv(buf, src=self._peer(self.rank - 1), group=self.group)
        return buf[0], buf[1]

    def _pack(self, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
        return torch.stack([x, residual]).contiguous()

    # ------------------------------------------------------------------ engine contract
    def kv_bytes_per_token(self, layers: range | None = None, skip_swa: bool = False, kv_dtype: str = "bf16") -> int:
        return super().kv_bytes_per_token(range(self.lo, self.hi) if layers is None else layers, skip_swa, kv_dtype)

    def allocate_caches(self, num_blocks: int, block_size: int, max_seqs: int, device=None,
                        layers: range | None = None, swa_blocks: int = 0, kv_dtype: str = "bf16") -> list:
        return super().allocate_caches(num_blocks, block_size, max_seqs, device,
                                       range(self.lo, self.hi) if layers is None else layers, swa_blocks, kv_dtype)

    def _run_layers(self, x, residual, meta, caches):
        for layer, kv in zip(self.layers, caches):
            x, residual = layer(x, residual, meta, kv, self.rope)
        return x, residual

    def _stage_in(self, ids: torch.Tensor):
        if self.first:
            return self.embed(ids), None
        return self._recv(ids.shape[0])

    def forward(self, ids: torch.Tensor, meta, caches: list, return_prenorm: bool = False):
        """This stage's part of one step.  Non-last stages send their output on and
        return None (or (None, None)); the last returns the normed hidden states."""
        x, residual = self._stage_in(ids)
        x, residual = self._run_layers(x, residual, meta, caches)
        if not self.last:
            dist.send(self._pack(x, residual), dst=self._peer(self.rank + 1), group=self.group)
            return (None, None) if return_prenorm else None
        h, pre = self.norm(x, residual)
        return (h, pre) if return_prenorm else h

    def sample(self, ids: torch.Tensor, meta, caches: list, logit_rows: torch.Tensor | None) -> torch.Tensor:
        """One engine step through the whole pipeline: every rank returns the greedy token
        ids of ``logit_rows`` (int32), computed on the last stage and broadcast."""
        h = self.forward(ids, meta, caches)
        n = 0 if logit_rows is None else int(logit_rows.numel())
        tok = torch.empty(n, dtype=torch.int32, device=self.device)
        if n == 0:
            return tok
        if self.last:
            tok.copy_(B.argmax(self.logits(h.index_select(0, logit_rows))).to(torch.int32))
        dist.broadcast(tok, src=self._peer(self.world - 1), group=self.group)
        return tok

    def forward_microbatches(self, batches: list, caches: list) -> list:
        """GPipe forward of several micro-batches ``[(ids, meta), ...]`` (each with its own
        sequences / cache slots).  Returns the last stage's normed hidden states per
        micro-batch (None elsewhere).  Sends are non-blocking: the stage starts on the
        next micro-batch while the previous one travels on."""
        outs, pending = [], []
        for ids, meta in batches:
            x, residual = self._stage_in(ids)
            x, residual = self._run_layers(x, residual, meta, caches)
            if self.last:
                outs.append(self.norm(x, residual)[0])
            else:
                buf = self._pack(x, residual)
                pending.append((buf, dist.isend(buf, dst=self._peer(self.rank + 1), group=self.group)))
                outs.append(None)
        for _, work in pending:
            work.wait()
        return outs
