"""Model runner: step plan -> device metadata -> forward -> sampling.

* Metadata for a step (token ids, positions, KV slot mapping, block tables,
  sequence lengths) is built on the host into pinned staging buffers and copied
  to the device with one async copy per tensor.
* Decode steps run as CUDA graphs captured per batch size (static input
  buffers; every kernel sizes its grid from upper bounds and reads the real
  lengths from device memory), which removes the launch overhead of ~10
  kernels x layers per token.
* Greedy sampling runs on the device (argmax kernel); speculative decoding with
  the model's MTP layer (k drafts, greedy verification) is handled by
  :class:`SpecDecoder` in ``spec_decode.py``.
"""
from __future__ import annotations

import dataclasses

import math
from dataclasses import dataclass

import torch

from ..models.model import MoETransformer
from ..ops import basic as B
from ..ops import _native as N
from ..ops.attention import AttnMetadata, choose_splits, decode_ctas_per_sm
from . import sampling as S
from .block_manager import swa_pool_blocks
from .scheduler import StepPlan


@dataclass
class RunnerConfig:
    block_size: int = 64
    num_blocks: int = 0            # 0: size from memory budget
    max_seqs: int = 16
    max_batched_tokens: int = 16384
    max_model_len: int = 32768
    use_cuda_graph: bool = True
    graph_batch_sizes: tuple = (1, 2, 4, 8, 16)
    kv_mem_fraction: float = 0.9   # of free memory after weights, for the KV cache
    num_spec: int = 0
    # sliding-window layers keep only their window in a small pool of their own (models
    # with "swa" layers); False: they share the full-context pool
    swa_bounded: bool = True
    swa_blocks: int = 0            # set by the runner: blocks of that pool (0 = no pool)
    # reuse the KV blocks of a cached prompt prefix (models without linear-attention
    # state or a sliding-window pool, whose per-request state a shared prefix cannot carry)
    prefix_caching: bool = False
    # "bf16" or "fp8" (e4m3, per-layer K / V scales; GQA layers -- MLA latents stay bf16)
    kv_cache_dtype: str = "bf16"


class ModelRunner:
    def __init__(self, model: MoETransformer, rc: RunnerConfig):
        self.model = model
        self.rc = rc
        self.pipeline = bool(getattr(model, "is_pipeline_stage", False))
        if self.pipeline and rc.num_spec > 0:
            raise ValueError("speculative decoding with pipeline stages is not supported")
        self.device = model.device
        self.cuda = self.device.type == "cuda"
        if rc.num_spec + 1 > rc.block_size:
            raise ValueError("num_spec + 1 must fit in one KV block (the block table keeps one block of slack "
                             "for a step's draft rows past max_model_len)")
        self.max_blocks_per_seq = (rc.max_model_len + rc.block_size - 1) // rc.block_size + 1
        cfg = model.cfg
        has_swa = cfg.sliding_window > 0 and cfg.layer_types is not None and "swa" in cfg.layer_types
        rc.swa_blocks = (swa_pool_blocks(rc.max_seqs, cfg.sliding_window, rc.block_size, rc.max_batched_tokens)
                         if has_swa and rc.swa_bounded else 0)
        if rc.num_blocks <= 0:
            rc.num_blocks = self._auto_blocks()
        self.caches = model.allocate_caches(rc.num_blocks, rc.block_size, rc.max_seqs, swa_blocks=rc.swa_blocks,
                                            kv_dtype=rc.kv_cache_dtype)
        if rc.swa_blocks:
            for l in model.layers:
                if getattr(l.attn, "window", 0) > 0:
                    l.attn.bounded = True
        self.mtp_caches = (model.allocate_mtp_caches(rc.num_blocks, rc.block_size, rc.max_seqs,
                                                     kv_dtype=rc.kv_cache_dtype) if model.mtp else [])
        max_rows = max(rc.max_batched_tokens, rc.max_seqs * (1 + rc.num_spec))
        model.prepare_workspaces(max_rows)
        self.graphs: dict[int, tuple] = {}
        self._static = None
        # bytes of the per-step host<->device copies (pinned H2D metadata and ids, D2H tokens)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.steps = 0

    # ------------------------------------------------------------------
    def _auto_blocks(self) -> int:
        per_tok = max(1, self.model.kv_bytes_per_token(skip_swa=self.rc.swa_blocks > 0,
                                                       kv_dtype=self.rc.kv_cache_dtype))
        if self.model.mtp:
            c = self.model.cfg
            last = c.num_layers - 1     # MTP layers: the last decoder layer's attention type
            gb = 1 if self.rc.kv_cache_dtype == "fp8" else 2
            per_tok += len(self.model.mtp) * ((c.kv_heads(last) * (c.head_dim + c.gqa_v_dim) * gb) if not c.is_mla
                                              else (c.kv_lora_rank + c.qk_rope_head_dim) * 2)
        need = self.rc.max_seqs * self.max_blocks_per_seq
        if not self.cuda:
            return need
        free, _ = torch.cuda.mem_get_info(self.device)
        reserve = 6 << 30   # activations, workspaces, graphs
        budget = max(0, int((free - reserve) * self.rc.kv_mem_fraction))
        nb = budget // (per_tok * self.rc.block_size)
        return int(max(16, min(nb, need)))

    # ------------------------------------------------------------------
    def build_meta(self, plan: StepPlan):
        """Host lists -> device tensors for one step."""
        bs = self.rc.block_size
        ids, pos, slots = [], [], []
        q_start = [0]
        kv_len, seq_slots, fresh = [], [], []
        tables = []
        swa = self.rc.swa_blocks > 0
        swa_slots, swa_tables = [], []
        for ch in plan.chunks:
            r = ch.req
            toks = r.all_tokens
            if plan.is_decode:
                step_toks = [toks[-1]] + list(r.draft)
            else:
                step_toks = toks[ch.start:ch.start + ch.length]
            n = len(step_toks)
            ids.extend(step_toks)
            p0 = ch.start
            for i in range(n):
                p = p0 + i
                pos.append(p)
                slots.append(r.blocks[p // bs] * bs + p % bs)
                if swa:
                    swa_slots.append(r.swa_blocks[p // bs] * bs + p % bs)
            if swa:    # logical blocks below the window read a placeholder (block 0), always masked
                swa_tables.append([r.swa_blocks.get(j, 0) for j in range(len(r.blocks))])
            q_start.append(q_start[-1] + n)
            kv_len.append(p0 + n)
            seq_slots.append(max(r.slot, 0))
            fresh.append(1 if p0 == 0 else 0)
            tables.append(r.blocks)
        Bn = len(plan.chunks)
        maxb = max(len(t) for t in tables)
        bt = torch.zeros(Bn, max(maxb, 1), dtype=torch.int32)
        for i, t in enumerate(tables):
            if t:
                bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        d = self.device
        nb = self.cuda

        def T(x, dt=torch.int32):
            t = torch.tensor(x, dtype=dt)
            if not nb:
                return t
            self.h2d_bytes += t.numel() * t.element_size()
            return t.pin_memory().to(d, non_blocking=True)

        if nb:
            self.h2d_bytes += bt.numel() * bt.element_size()
        self.steps += 1
        meta = AttnMetadata(num_seqs=Bn, q_start=T(q_start), kv_len=T(kv_len),
                            block_table=bt.pin_memory().to(d, non_blocking=True) if nb else bt,
                            slot_mapping=T(slots), positions=T(pos), max_q_len=max(q_start[i + 1] - q_start[i] for i in range(Bn)),
                            max_kv_len=max(kv_len), is_decode=plan.is_decode, q_start_host=q_start, kv_len_host=kv_len,
                            seq_slots=T(seq_slots), seq_fresh=T(fresh))
        if swa:
            sbt = torch.zeros_like(bt)
            for i, t in enumerate(swa_tables):
                if t:
                    sbt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
            if nb:
                self.h2d_bytes += sbt.numel() * sbt.element_size()
            meta.swa_block_table = sbt.pin_memory().to(d, non_blocking=True) if nb else sbt
            meta.swa_slot_mapping = T(swa_slots)
        if plan.is_decode and self.cuda:
            meta.num_splits = choose_splits(Bn, max(1, self.model.cfg.num_kv_heads), meta.max_kv_len,
                                            ctas_per_sm=decode_ctas_per_sm(self.model.cfg, meta.max_q_len))
        return T(ids), meta

    # ------------------------------------------------------------------
    @torch.inference_mode()
    def forward(self, ids, meta, logit_rows: torch.Tensor | None):
        if self.pipeline:   # pipeline stage: tokens come back from the last stage
            return self.model.sample(ids, meta, self.caches, logit_rows), None, None, None
        h, pre = self.model.forward(ids, meta, self.caches, return_prenorm=True)
        if logit_rows is not None:
            hs = h.index_select(0, logit_rows)
            logits = self.model.logits(hs)
            return B.argmax(logits), h, pre, logits
        return None, h, pre, None

    @torch.inference_mode()
    def execute(self, plan: StepPlan):
        """Run one step; returns (sampled token ids per row that produced logits (host list), extras)."""
        ids, meta = self.build_meta(plan)
        if plan.is_decode:
            rows = None  # every row produces logits
            reqs = [ch.req for ch in plan.chunks]
            if self.cuda and self.rc.use_cuda_graph and self.rc.num_spec == 0 and not self.pipeline:
                tok, logits = self._decode_graph(ids, meta)
                if logits is not None and S.needs_sampling(reqs):
                    tok = S.sample_rows(logits, reqs, tok)
                self._logprobs(logits, tok, reqs)
                return tok, None
            tok, h, pre, logits = self.forward(ids, meta, torch.arange(ids.shape[0], device=self.device))
            if logits is not None and S.needs_sampling(reqs):
                tok = S.sample_rows(logits, reqs, tok)
            self._logprobs(logits, tok, reqs)
            return tok, (h, pre, meta)
        # prefill: logits only for chunks that finish their prompt
        rows, reqs = [], []
        for i, ch in enumerate(plan.chunks):
            if ch.start + ch.length == len(ch.req.prompt):
                rows.append(meta.q_start_host[i + 1] - 1)
                reqs.append(ch.req)
        rt = torch.tensor(rows, dtype=torch.long, device=self.device) if rows else None
        tok, h, pre, logits = self.forward(ids, meta, rt)
        if logits is not None and S.needs_sampling(reqs):
            tok = S.sample_rows(logits, reqs, tok)
        self._logprobs(logits, tok, reqs)
        return tok, (h, pre, meta, rows)

    def _logprobs(self, logits, tok, reqs) -> None:
        """Record each row's token log-probability (and alternatives) for requests asking."""
        k = S.wants_logprobs(reqs) if logits is not None else -1
        if k < 0:
            return
        for r, lp in zip(reqs, S.row_logprobs(logits, tok, k)):
            if r.params.logprobs is not None:
                n = r.params.logprobs
                r.logprobs.append((lp[0], dict(list(lp[1].items())[:n])))

    # ------------------------------------------------------------------
    # CUDA-graph decode (one token per sequence)
    # ------------------------------------------------------------------
    def _graph_bs(self, n: int) -> int | None:
        for b in self.rc.graph_batch_sizes:
            if b >= n and b <= self.rc.max_seqs:
                return b
        return None

    def _alloc_static(self):
        ms = max(self.rc.graph_batch_sizes)
        d = self.device
        self._static = dict(
            ids=torch.zeros(ms, dtype=torch.int32, device=d),
            pos=torch.zeros(ms, dtype=torch.int32, device=d),
            slots=torch.full((ms,), -1, dtype=torch.int32, device=d),
            swa_slots=torch.full((ms,), -1, dtype=torch.int32, device=d),
            swa_bt=torch.zeros(ms, self.max_blocks_per_seq, dtype=torch.int32, device=d),
            q_start=torch.arange(ms + 1, dtype=torch.int32, device=d),
            kv_len=torch.ones(ms, dtype=torch.int32, device=d),
            bt=torch.zeros(ms, self.max_blocks_per_seq, dtype=torch.int32, device=d),
            seq_slots=torch.full((ms,), -1, dtype=torch.int32, device=d),
            fresh=torch.zeros(ms, dtype=torch.int32, device=d),
            out=torch.zeros(ms, dtype=torch.int32, device=d),
            rows=torch.arange(ms, dtype=torch.long, device=d),   # logit rows (must outlive the graphs)
        )

    def _static_meta(self, b: int) -> AttnMetadata:
        s = self._static
        splits = choose_splits(b, max(1, self.model.cfg.num_kv_heads), self.rc.max_model_len,
                               ctas_per_sm=decode_ctas_per_sm(self.model.cfg))
        return AttnMetadata(num_seqs=b, q_start=s["q_start"][:b + 1], kv_len=s["kv_len"][:b],
                            block_table=s["bt"][:b], slot_mapping=s["slots"][:b], positions=s["pos"][:b],
                            max_q_len=1, max_kv_len=self.rc.max_model_len, is_decode=True,
                            seq_slots=s["seq_slots"][:b], seq_fresh=s["fresh"][:b], num_splits=splits,
                            swa_block_table=s["swa_bt"][:b] if self.rc.swa_blocks else None,
                            swa_slot_mapping=s["swa_slots"][:b] if self.rc.swa_blocks else None)

    def _capture(self, b: int):
        if self._static is None:
            self._alloc_static()
        s = self._static
        meta = self._static_meta(b)
        rows = s["rows"][:b]
        # warm up (allocations happen outside the capture).  The warm-up passes execute, so
        # they run with no recurrent-state slots (-1): the step's real sequences must not have
        # their linear-attention state advanced by a pass that is not the step itself (their
        # KV-cache writes repeat what the replay writes, so those are harmless)
        warm = dataclasses.replace(meta, seq_slots=torch.full((b,), -1, dtype=torch.int32, device=self.device))
        for _ in range(2):
            tok, *_ = self.forward(s["ids"][:b], warm, rows)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        n0 = N.launches()
        with torch.cuda.graph(g):
            tok, _, _, logits = self.forward(s["ids"][:b], meta, rows)
            s["out"][:b].copy_(tok)
        kernels = N.launches() - n0
        N.add_launches(-kernels)      # capture enqueues nothing; replays are counted below
        # `logits` is a graph output: after each replay it holds that step's logits rows
        self.graphs[b] = (g, meta, kernels, logits)

    def _decode_graph(self, ids, meta):
        n = meta.num_seqs
        b = self._graph_bs(n)
        if b is None:
            tok, _, _, logits = self.forward(ids, meta, torch.arange(ids.shape[0], device=self.device))
            return tok, logits
        if self._static is None:
            self._alloc_static()
        s = self._static
        s["ids"][:n].copy_(ids)
        s["pos"][:n].copy_(meta.positions)
        s["slots"][:b].fill_(-1)
        s["slots"][:n].copy_(meta.slot_mapping)
        s["kv_len"][:b].fill_(1)
        s["kv_len"][:n].copy_(meta.kv_len)
        w = meta.block_table.shape[1]
        s["bt"][:n, :w].copy_(meta.block_table)
        s["seq_slots"][:b].fill_(-1)
        s["seq_slots"][:n].copy_(meta.seq_slots)
        if self.rc.swa_blocks:
            s["swa_slots"][:b].fill_(-1)
            s["swa_slots"][:n].copy_(meta.swa_slot_mapping)
            s["swa_bt"][:n, :w].copy_(meta.swa_block_table)
        s["fresh"][:b].zero_()
        if b not in self.graphs:
            self._capture(b)
        g, _, kernels, logits = self.graphs[b]
        g.replay()
        N.add_launches(kernels)
        return s["out"][:n], (logits[:n] if logits is not None else None)

    def release_graphs(self):
        self.graphs.clear()
