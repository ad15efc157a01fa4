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

Sampled requests (temperature > 0) verify by rejection sampling against the point-mass
draft distribution of the greedy drafter (Leviathan et al. 2023, Chen et al. 2023):
draft d_j is kept with probability p_j(d_j) (p_j the request's filtered sampling
distribution at that row), the first rejected position emits a draw from p_j with d_j
removed and renormalised, and a fully accepted chain adds a draw from the last row's p;
every emitted token is then an exact sample of the request's distribution.  Those steps
run eagerly (the sampling draws are made with the request's own generator).

Linear-attention (DeltaNet / KDA) layers carry a recurrent state that rejected drafts
must not advance: a verification step keeps the state after each of its rows
(``DeltaNetState.spec_ssm`` / ``spec_conv``, written by the recurrent and conv-state
kernels), and once the acceptance is known a kernel installs, per sequence, the states
after its last accepted row (``xtu_deltanet_spec_commit``; inside the replayed graph).

On a GPU a decode step whose requests all carry k drafts replays one CUDA graph per batch
bucket: the verification forward, the acceptance kernel, the MTP pass over the verified
rows and the k - 1 chained draft passes, whose positions, KV slots and lengths a kernel
derives on the device from the acceptance (``xtu_spec_chain_meta``).  The host copies the
step's metadata in, replays, and reads back one int32 buffer (target tokens, accepted
counts, next drafts).
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


def verify_sampled(logits: torch.Tensor, drafts: list[int], params, generator: torch.Generator) -> list[int]:
    """Rejection-sampling verification of one request's greedy drafts.

    logits [len(drafts) + 1, V]: row j is the target's distribution for the position that
    draft j (0-based) fills; row len(drafts) the one after the last draft.  Returns the
    emitted tokens: the accepted drafts, then one drawn token (2 host reads)."""
    from .sampling import filtered_probs
    n = len(drafts)
    probs = torch.stack([filtered_probs(logits[j], params.temperature, params.top_k, params.top_p)
                         for j in range(n + 1)])
    d = torch.tensor(drafts, dtype=torch.long, device=logits.device)
    u = torch.rand(n, generator=generator, device=logits.device)
    keep = (u < probs[torch.arange(n, device=logits.device), d]).tolist() if n else []
    a = 0
    while a < n and keep[a]:
        a += 1
    p = probs[a].clone()
    if a < n:                                 # residual of the point-mass draft: p without d_a
        p[d[a]] = 0.0
        tot = p.sum()
        p = p / tot if float(tot) > 0 else probs[a]
    x = int(torch.multinomial(p, 1, generator=generator)[0])
    return drafts[:a] + [x]


class SpecDecoder:
    def __init__(self, runner, k: int, blocks):
        self.runner = runner
        self.blocks = blocks
        self.model = runner.model
        self.k = k
        if not self.model.mtp:
            raise ValueError("speculative decoding needs a model with an MTP layer")
        from ..models.deltanet import DeltaNetState
        # recurrent layers: k + 1 state copies per slot for the rollback of rejected drafts
        self.states = [c for c in runner.caches if isinstance(c, DeltaNetState)]
        for st in self.states:
            st.enable_spec(max(k, runner.rc.num_spec))
        self.mtp = self.model.mtp[0]
        self.caches = runner.mtp_caches[0]
        rc = runner.rc
        self.use_graph = runner.cuda and rc.use_cuda_graph and not runner.pipeline and k >= 1
        self.graphs: dict[int, tuple] = {}
        self._st = None
        self.graph_steps = 0
        self.eager_steps = 0

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
    def _commit(self, accepted: torch.Tensor, slots: torch.Tensor) -> None:
        for st in self.states:
            st.commit_spec(accepted, slots)

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

    # ------------------------------------------------------------------ graph-replayed step
    def _graph_bucket(self, plan) -> int | None:
        if not self.use_graph:
            return None
        k = self.k
        if any(len(ch.req.draft) != k for ch in plan.chunks):
            return None
        n = len(plan.chunks)
        for b in self.runner.rc.graph_batch_sizes:
            if n <= b <= self.runner.rc.max_seqs:
                return b
        return None

    def _alloc_static(self):
        rn, k = self.runner, self.k
        ms = max(b for b in rn.rc.graph_batch_sizes if b <= rn.rc.max_seqs)
        R = ms * (k + 1)
        d = rn.device
        mb = rn.max_blocks_per_seq
        self._st = dict(
            ms=ms, ids=torch.zeros(R, dtype=torch.int32, device=d), pos=torch.zeros(R, dtype=torch.int32, device=d),
            slots=torch.full((R,), -1, dtype=torch.int32, device=d),
            q_start=torch.arange(0, (ms + 1) * (k + 1), k + 1, dtype=torch.int32, device=d),
            kv_len=torch.full((ms,), k + 1, dtype=torch.int32, device=d),
            bt=torch.zeros(ms, mb, dtype=torch.int32, device=d),
            seq_slots=torch.full((ms,), -1, dtype=torch.int32, device=d),
            fresh=torch.zeros(ms, dtype=torch.int32, device=d),
            base=torch.zeros(ms, dtype=torch.int32, device=d),
            rows=torch.arange(R, dtype=torch.long, device=d),
            cq=torch.arange(ms + 1, dtype=torch.int32, device=d),
            cpos=torch.zeros(max(1, k - 1), ms, dtype=torch.int32, device=d),
            cslot=torch.full((max(1, k - 1), ms), -1, dtype=torch.int32, device=d),
            ckv=torch.ones(max(1, k - 1), ms, dtype=torch.int32, device=d),
            # one read-back buffer per bucket: [target rows | accepted | drafts]
            out={})

    def _graph_body(self, b: int):
        """The step for a batch bucket of b sequences (runs eagerly to warm up, then captured)."""
        rn, k, st, m = self.runner, self.k, self._st, self.model
        R = b * (k + 1)
        cfg = m.cfg
        splits = choose_splits(b, max(1, cfg.num_kv_heads), rn.rc.max_model_len,
                               ctas_per_sm=decode_ctas_per_sm(cfg, k + 1))
        meta = AttnMetadata(num_seqs=b, q_start=st["q_start"][:b + 1], kv_len=st["kv_len"][:b],
                            block_table=st["bt"][:b], slot_mapping=st["slots"][:R], positions=st["pos"][:R],
                            max_q_len=k + 1, max_kv_len=rn.rc.max_model_len, is_decode=True,
                            seq_slots=st["seq_slots"][:b], seq_fresh=st["fresh"][:b], num_splits=splits,
                            spec_rows=k + 1)
        out = st["out"][b]
        tgt_o, acc_o, drf_o = out[:R], out[R:R + b], out[R + b:].view(b, k)
        tgt, h, _, _ = rn.forward(st["ids"][:R], meta, st["rows"][:R])
        last = torch.empty(b, dtype=torch.int32, device=rn.device)
        N.call("xtu_spec_verify", tgt.data_ptr(), st["ids"].data_ptr(), meta.q_start.data_ptr(), b, k,
               acc_o.data_ptr(), last.data_ptr(), N.stream_ptr(rn.device))
        self._commit(acc_o, st["seq_slots"][:b])
        hid = self._mtp(tgt, h, meta).index_select(0, last.long())
        tok = B.argmax(m.logits(hid))
        drf_o[:, 0].copy_(tok)
        if k > 1:
            bt = st["bt"]
            N.call("xtu_spec_chain_meta", st["base"].data_ptr(), acc_o.data_ptr(), bt.data_ptr(), bt.stride(0),
                   bt.shape[1], rn.rc.block_size, b, k, st["cpos"].data_ptr(), st["cslot"].data_ptr(),
                   st["ckv"].data_ptr(), N.stream_ptr(rn.device))
            # cpos / cslot / ckv are [k-1, ms]: pass j's b rows start at (j-1) * b in the flat view
            cp, cs, ck = (st[n].view(-1) for n in ("cpos", "cslot", "ckv"))
            csplits = choose_splits(b, max(1, cfg.num_kv_heads), rn.rc.max_model_len,
                                    ctas_per_sm=decode_ctas_per_sm(cfg))
            for j in range(1, k):
                o = (j - 1) * b
                mj = AttnMetadata(num_seqs=b, q_start=st["cq"][:b + 1], kv_len=ck[o:o + b],
                                  block_table=bt[:b], slot_mapping=cs[o:o + b], positions=cp[o:o + b], max_q_len=1,
                                  max_kv_len=rn.rc.max_model_len, is_decode=True, num_splits=csplits)
                hid = self._mtp(tok, hid, mj)
                tok = B.argmax(m.logits(hid))
                drf_o[:, j].copy_(tok)
        tgt_o.copy_(tgt)

    def _replay(self, plan, b: int):
        """Fill the bucket's static inputs from the plan, replay its graph (capturing it on
        first use) and return the host copy of [target rows | accepted | drafts]."""
        rn, k = self.runner, self.k
        if self._st is None:
            self._alloc_static()
        st = self._st
        ids, meta = rn.build_meta(plan)
        n = meta.num_seqs
        R, Rn = b * (k + 1), n * (k + 1)
        if b not in st["out"]:
            st["out"][b] = torch.zeros(R + b + b * k, dtype=torch.int32, device=rn.device)
        st["ids"][:Rn].copy_(ids)
        st["pos"][:Rn].copy_(meta.positions)
        st["slots"][:R].fill_(-1)
        st["slots"][:Rn].copy_(meta.slot_mapping)
        st["kv_len"][:b].fill_(k + 1)
        st["kv_len"][:n].copy_(meta.kv_len)
        w = meta.block_table.shape[1]
        st["bt"][:n, :w].copy_(meta.block_table)
        st["seq_slots"][:b].fill_(-1)
        if meta.seq_slots is not None:        # recurrent-state slots (linear-attention layers)
            st["seq_slots"][:n].copy_(meta.seq_slots)
        st["fresh"][:b].zero_()
        base = torch.tensor([ch.req.total_len for ch in plan.chunks] + [0] * (b - n), dtype=torch.int32)
        rn.h2d_bytes += base.numel() * 4
        st["base"][:b].copy_(base.pin_memory(), non_blocking=True)
        if b not in self.graphs:
            for _ in range(2):           # warm-up (allocations happen outside the capture)
                self._graph_body(b)
            torch.cuda.synchronize(rn.device)
            g = torch.cuda.CUDAGraph()
            n0 = N.launches()
            with torch.cuda.graph(g):
                self._graph_body(b)
            kernels = N.launches() - n0
            N.add_launches(-kernels)
            self.graphs[b] = (g, kernels)
        g, kernels = self.graphs[b]
        g.replay()
        N.add_launches(kernels)
        host = st["out"][b].cpu()
        rn.d2h_bytes += host.numel() * 4
        return meta, host

    def release_graphs(self):
        self.graphs.clear()

    @torch.inference_mode()
    def decode_step(self, plan, scheduler) -> list:
        if any(ch.req.params.temperature > 0.0 for ch in plan.chunks):
            return self._decode_step_eager(plan, scheduler)
        b = self._graph_bucket(plan)
        if b is not None:
            # the chain writes draft KV up to total_len + 2k - 1: hold those blocks first
            if all(self.blocks.ensure(ch.req, ch.req.total_len + 2 * self.k + 1) for ch in plan.chunks):
                return self._decode_step_graph(plan, scheduler, b)
        return self._decode_step_eager(plan, scheduler)

    def _decode_step_graph(self, plan, scheduler, b: int) -> list:
        import time
        k = self.k
        meta, host = self._replay(plan, b)
        self.graph_steps += 1
        R = b * (k + 1)
        tgt_h = host[:R].tolist()
        acc_h = host[R:R + b].tolist()
        drafts = host[R + b:].view(b, k).tolist()
        now = time.perf_counter()
        done = []
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
                r.draft = drafts[i]
                r.proposed += k
        return done

    def _decode_step_eager(self, plan, scheduler) -> list:
        import time
        self.eager_steps += 1
        rn = self.runner
        ids, meta = rn.build_meta(plan)
        meta.spec_rows = meta.max_q_len
        n_rows = ids.shape[0]
        tgt, h, _, logits = rn.forward(ids, meta, torch.arange(n_rows, device=rn.device))
        k = max(len(ch.req.draft) for ch in plan.chunks)
        emit = tgt.to(torch.int32)
        if any(ch.req.params.temperature > 0.0 for ch in plan.chunks):
            # sampled requests: rejection sampling; their emitted tokens feed the MTP pass
            from .sampling import _generator
            acc_l, last_l = [], []
            emit_h = emit.tolist()
            greedy_acc, _ = verify_greedy(tgt, ids, meta.q_start, meta.num_seqs, k)
            greedy_acc = greedy_acc.tolist()
            for i, ch in enumerate(plan.chunks):
                r = ch.req
                q0, q1 = meta.q_start_host[i], meta.q_start_host[i + 1]
                if r.params.temperature > 0.0:
                    nd = min(len(r.draft), q1 - q0 - 1)
                    toks = verify_sampled(logits[q0:q0 + nd + 1], [int(t) for t in r.draft[:nd]], r.params,
                                          _generator(r, logits.device))
                    emit_h[q0:q0 + len(toks)] = toks
                    a = len(toks) - 1
                else:
                    a = greedy_acc[i]
                acc_l.append(a)
                last_l.append(q0 + a)
            emit = torch.tensor(emit_h, dtype=torch.int32, device=rn.device)
            acc = torch.tensor(acc_l, dtype=torch.int32)
            last = torch.tensor(last_l, dtype=torch.long, device=rn.device)
        else:
            acc, last = verify_greedy(tgt, ids, meta.q_start, meta.num_seqs, k)
        if self.states and meta.seq_slots is not None:
            self._commit(acc.to(device=rn.device, dtype=torch.int32), meta.seq_slots)
        out = self._mtp(emit, h, meta)
        hid = out.index_select(0, last.long())
        first = B.argmax(self.model.logits(hid))
        tgt_h = emit.tolist()
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
