"""Speculative decoding with the model's MTP ("next-n") layer, greedy verification.

The reference runs GLM MTP k=1..4 and DeepSeek drafters through vLLM's proposer
(scripts/serve_v41.sh:41-47; hybrid_model.py:121-237 detects and places the draft
layers).  Here the drafter is the model's own ``MTPLayer`` and the loop is:

* MTP row semantics: the row at position p reads (h_p, token_{p+1}) and predicts
  token_{p+2}.  Its attention has its own paged KV cache that shares the main
  cache's block tables, so one ``AttnMetadata`` serves both.
* After a prefill chunk the MTP layer runs over the same rows (token ids shifted by
  one; the last row of a finished prompt uses the sampled token) and, for finished
  prompts, drafts k tokens (row 1 from the main hidden state, rows 2..k chained from
  the MTP layer's own output).
* A decode step verifies [last, d_1..d_k] in one main forward (k+1 query rows per
  sequence).  The verification kernel counts, per sequence, the leading drafts equal
  to the target's greedy tokens (a) and emits t_0..t_a.  The MTP layer then runs over
  the same k+1 rows with the target tokens as inputs; the row of the last accepted
  position gives the next d_1, and the chain gives the rest.  Rows past the accepted
  prefix leave stale KV entries at positions that the next step overwrites before
  any row can attend to them.

Linear-attention (DeltaNet) models are not drafted: their recurrent state would
need a rollback for rejected drafts.
"""
from __future__ import annotations

import torch

from ..ops import _native as N
from ..ops import basic as B
from ..ops.attention import AttnMetadata, choose_splits, decode_ctas_per_sm


def verify_greedy(target: torch.Tensor, ids: torch.Tensor, q_start: torch.Tensor, num_seqs: int, k: int):
    """-> (accepted [B] int32, last_row [B] int32): leading drafts equal to the target's tokens.

    Row q_start[b] + j of ``ids`` holds d_j (j >= 1); row q_start[b] + j of ``target``
    holds the target's token for the position after it.
    """
    acc = torch.empty(num_seqs, dtype=torch.int32, device=target.device)
    row = torch.empty(num_seqs, dtype=torch.int32, device=target.device)
    if target.is_cuda:
        N.call("xtu_spec_verify", target.data_ptr(), ids.data_ptr(), q_start.data_ptr(), num_seqs, k,
               acc.data_ptr(), row.data_ptr(), N.stream_ptr(target.device))
        return acc, row
    qs = q_start.tolist()
    for b in range(num_seqs):
        a = 0
        while a < k and qs[b] + a + 1 < qs[b + 1] and int(ids[qs[b] + a + 1]) == int(target[qs[b] + a]):
            a += 1
        acc[b] = a
        row[b] = qs[b] + a
    return acc, row


class SpecDecoder:
    def __init__(self, runner, k: int, blocks):
        self.runner = runner
        self.blocks = blocks
        self.model = runner.model
        self.k = k
        if not self.model.mtp:
            raise ValueError("speculative decoding needs a model with an MTP layer")
        if any(self.model.cfg.layer_type(i) == "linear" for i in range(self.model.cfg.num_layers)):
            raise NotImplementedError("MTP drafting with linear-attention layers (no state rollback)")
        self.mtp = self.model.mtp[0]
        self.caches = runner.mtp_caches[0]

    # ------------------------------------------------------------------ MTP passes
    def _mtp(self, tok_ids: torch.Tensor, hidden: torch.Tensor, meta: AttnMetadata) -> torch.Tensor:
        emb = self.model.embed(tok_ids)
        return self.mtp(emb, hidden, meta, self.caches, self.model.rope)

    def _chain(self, reqs, first: torch.Tensor, hid: torch.Tensor) -> list[list[int]]:
        """Drafts 2..k for each request, starting from draft 1 and the MTP hidden row."""
        drafts = [first]
        n = len(reqs)
        d = self.runner.device
        if self.k > 1:
            bs = self.runner.rc.block_size
            for r in reqs:
                self.blocks.ensure(r, r.total_len + self.k + 1)
            tables = [r.blocks for r in reqs]
            maxb = max(len(t) for t in tables)
            bt = torch.zeros(n, maxb, dtype=torch.int32)
            for i, t in enumerate(tables):
                bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
            bt = bt.to(d)
            q_start = torch.arange(n + 1, dtype=torch.int32, device=d)
            tok = first
            for j in range(1, self.k):
                pos = [r.total_len - 2 + j for r in reqs]
                if any(p // bs >= len(r.blocks) for p, r in zip(pos, reqs)):
                    break
                slots = [r.blocks[p // bs] * bs + p % bs for p, r in zip(pos, reqs)]
                kv = [p + 1 for p in pos]
                meta = AttnMetadata(num_seqs=n, q_start=q_start, kv_len=torch.tensor(kv, dtype=torch.int32, device=d),
                                    block_table=bt, slot_mapping=torch.tensor(slots, dtype=torch.int32, device=d),
                                    positions=torch.tensor(pos, dtype=torch.int32, device=d), max_q_len=1,
                                    max_kv_len=max(kv), is_decode=True, q_start_host=list(range(n + 1)),
                                    kv_len_host=kv)
                if self.runner.cuda:
                    meta.num_splits = choose_splits(n, max(1, self.model.cfg.num_kv_heads), max(kv),
                                                    ctas_per_sm=decode_ctas_per_sm(self.model.cfg))
                hid = self._mtp(tok, hid, meta)
                tok = B.argmax(self.model.logits(hid))
                drafts.append(tok)
        return torch.stack(drafts, dim=1).tolist()

    # ------------------------------------------------------------------ engine hooks
    def after_prefill(self, r, extra) -> None:
        r.draft = []

    @torch.inference_mode()
    def prefill_mtp(self, plan, extra) -> None:
        h, _, meta, rows = extra
        ids = []
        fin, fin_rows = [], []
        for i, ch in enumerate(plan.chunks):
            toks = ch.req.all_tokens
            nxt = toks[ch.start + 1: ch.start + ch.length + 1]
            if len(nxt) < ch.length:         # unfinished prompt whose next chunk is not known yet: pad
                nxt = nxt + [0] * (ch.length - len(nxt))
            ids.extend(nxt)
            if ch.start + ch.length == len(ch.req.prompt) and not ch.req.finished():
                fin.append(ch.req)
                fin_rows.append(meta.q_start_host[i + 1] - 1)
        tid = torch.tensor(ids, dtype=torch.int32, device=self.runner.device)
        out = self._mtp(tid, h, meta)
        if not fin:
            return
        rows_t = torch.tensor(fin_rows, dtype=torch.long, device=self.runner.device)
        hid = out.index_select(0, rows_t)
        first = B.argmax(self.model.logits(hid))
        for r, d in zip(fin, self._chain(fin, first, hid)):
            r.draft = d
            r.proposed += len(d)

    @torch.inference_mode()
    def decode_step(self, plan, scheduler) -> list:
        import time
        rn = self.runner
        ids, meta = rn.build_meta(plan)
        n_rows = ids.shape[0]
        tgt, h, _, _ = rn.forward(ids, meta, torch.arange(n_rows, device=rn.device))
        k = max(len(ch.req.draft) for ch in plan.chunks)
        acc, last = verify_greedy(tgt, ids, meta.q_start, meta.num_seqs, k)
        out = self._mtp(tgt.to(torch.int32), h, meta)
        hid = out.index_select(0, last.long())
        first = B.argmax(self.model.logits(hid))
        tgt_h = tgt.tolist()
        acc_h = acc.tolist()
        now = time.perf_counter()
        done = []
        live, live_idx = [], []
        for i, ch in enumerate(plan.chunks):
            r = ch.req
            q0 = meta.q_start_host[i]
            a = min(acc_h[i], len(r.draft))
            r.accepted += a
            for t in tgt_h[q0:q0 + a + 1]:
                if r.finished():
                    break
                r.output.append(int(t))
            r.num_computed = r.total_len - 1
            r.draft = []
            if r.finished():
                r.t_done = now
                scheduler.finish(r)
                done.append(r)
            else:
                live.append(r)
                live_idx.append(i)
        if live:
            sel = torch.tensor(live_idx, dtype=torch.long, device=rn.device)
            drafts = self._chain(live, first.index_select(0, sel), hid.index_select(0, sel))
            for r, d in zip(live, drafts):
                r.draft = d
                r.proposed += len(d)
        return done
