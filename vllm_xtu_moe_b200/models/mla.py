"""Multi-head latent attention (DeepSeek-V3 family) over a paged latent cache.

Cache: one latent "head" per token, ``[num_blocks, 1, block_size, kv_lora + rope]``
(the normalised compressed KV followed by the RoPE'd shared key).  Prefill
expands the latent into per-head K/V (qk dim = nope + rope, v dim = v_head_dim)
and runs causal attention; decode absorbs W_UK into the query and W_UV into the
output so attention runs directly over the 576-wide latent (MQA-like: all 128
heads share one KV "head"), which is what makes MLA decode bandwidth-cheap.

An fp8 latent cache (``kv_cache_dtype="fp8"``) stores e4m3 rows (latent / latent_scale,
one scale per layer): half the bytes per cached token, so twice the context fits.  Each
step dequantises its sequences' blocks into a bf16 scratch cache that the latent kernels
read (``csrc/cuda/mla_fp8.cu``); the trade is capacity, not bandwidth.
"""
from __future__ import annotations

import dataclasses
import math

import torch

from ..ops import _native as N
from ..ops import basic as B
from ..ops import gemm as G
from ..ops.attention import AttnMetadata, paged_attention
from .config import ModelConfig
from .layers import Linear


_LATENT_SCRATCH: dict = {}


def write_latent_fp8(entry: torch.Tensor, slot_mapping: torch.Tensor, cache: torch.Tensor, scale: float) -> None:
    """entry [T, 1, D] bf16 -> e4m3 rows entry / scale (saturated at +-448) of the paged
    latent cache [blocks, 1, bs, D] at each token's slot (slot < 0: skipped)."""
    T, _, D = entry.shape
    bs = cache.shape[2]
    if not entry.is_cuda:
        sm = slot_mapping.long()
        valid = sm >= 0
        cache[(sm // bs)[valid], 0, (sm % bs)[valid]] = B.to_e4m3(entry[valid, 0], 1.0 / scale)
        return
    x = entry.reshape(T, D).to(torch.bfloat16).contiguous()
    N.call("xtu_mla_latent_write_fp8", x.data_ptr(), x.stride(0), T, D, slot_mapping.data_ptr(),
           cache.shape[0] * bs, cache.data_ptr(), float(1.0 / scale), N.status_buffer(x.device).data_ptr(),
           N.stream_ptr(x.device))


def dequant_latent_cache(cache: torch.Tensor, meta: AttnMetadata, scale: float):
    """The blocks of the step's sequences of an e4m3 latent cache -> (bf16 cache [B * maxb,
    1, bs, D] with block j of sequence b at b * maxb + j, metadata with that block table).
    The scratch cache and block table are shared by all layers (one layer runs at a time)
    and keep their addresses, so a captured decode graph replays them."""
    nb, _, bs, D = cache.shape
    Bn, maxb = meta.block_table.shape
    dev = cache.device
    key = (dev, Bn * maxb, bs, D)
    sc = _LATENT_SCRATCH.get(key)
    if sc is None:
        sc = (torch.zeros(Bn * maxb, 1, bs, D, dtype=torch.bfloat16, device=dev),
              torch.arange(Bn * maxb, dtype=torch.int32, device=dev).view(Bn, maxb))
        _LATENT_SCRATCH[key] = sc
    out, bt = sc
    if cache.is_cuda:
        N.call("xtu_mla_latent_dequant_gather", cache.data_ptr(), D, meta.block_table.data_ptr(),
               meta.block_table.stride(0), meta.kv_len.data_ptr(), Bn, maxb, nb, float(scale), out.data_ptr(),
               N.status_buffer(dev).data_ptr(), N.stream_ptr(dev))
    else:
        kl = meta.kv_len_host if meta.kv_len_host is not None else meta.kv_len.tolist()
        for b in range(Bn):
            for j in range((int(kl[b]) + bs - 1) // bs):
                out[b * maxb + j] = (cache[int(meta.block_table[b, j])].float() * scale).to(torch.bfloat16)
    return out, dataclasses.replace(meta, block_table=bt)


class DSAIndexer:
    """DeepSeek-V3.2 lightning indexer of one MLA layer: index queries from the q latent
    (wq_b: q_lora -> n_heads x 128), one index key per token (wk: hidden -> 128, LayerNorm
    with bias), per-head weights (weights_proj: hidden -> n_heads, times n_heads^-1/2 and the
    softmax scale 128^-1/2); RoPE (non-interleaved) on the first qk_rope_head_dim dims of both.
    Its keys live in a paged cache of their own ([blocks, 1, 64, 128], the latent cache's
    block tables).  Scores and selection: :mod:`..ops.dsa`."""

    def __init__(self, cfg: ModelConfig, wq_b: Linear, wk: Linear, k_norm_w: torch.Tensor, k_norm_b: torch.Tensor,
                 weights_proj: Linear):
        self.cfg = cfg
        self.wq_b, self.wk, self.weights_proj = wq_b, wk, weights_proj
        self.k_norm_w, self.k_norm_b = k_norm_w, k_norm_b
        self.nh, self.d = cfg.index_n_heads, cfg.index_head_dim
        self.topk = cfg.index_topk
        self.w_scale = self.nh ** -0.5 * self.d ** -0.5
        self._ws = {}

    def keys_and_queries(self, x: torch.Tensor, qa: torch.Tensor, meta: AttnMetadata, idx_cache: torch.Tensor,
                         rope: torch.Tensor):
        """Writes the step's index keys into the cache; returns (q [T, nh, d] bf16, w [T, nh] fp32)."""
        import torch.nn.functional as F
        T = x.shape[0]
        c = self.cfg
        q = self.wq_b(qa).view(T, self.nh, self.d)
        k = F.layer_norm(self.wk(x).float(), (self.d,), self.k_norm_w.float(), self.k_norm_b.float(),
                         1e-6).to(torch.bfloat16).view(T, 1, self.d)
        rot = c.qk_rope_head_dim if c.mla_rope else 0
        if rot:
            if x.is_cuda:
                B.rope_and_cache(q, k, k, meta.positions, rope, rot, True)
            else:
                q = B.apply_rope_ref(q, meta.positions, rope, rot, True)
                k = B.apply_rope_ref(k, meta.positions, rope, rot, True)
        B.write_cache_rows(k.contiguous(), meta.slot_mapping, idx_cache)
        w = (self.weights_proj(x).float() * self.w_scale).contiguous()
        return q.contiguous(), w

    def select(self, q: torch.Tensor, w: torch.Tensor, meta: AttnMetadata, idx_cache: torch.Tensor,
               max_len: int):
        """-> (rows [T, topk] flat latent-cache rows, lens [T]) of every query row."""
        from ..ops import dsa as D
        T = q.shape[0]
        ld = (max_len + 63) // 64 * 64
        key = (T, ld, q.device)
        ws = self._ws.get(key)
        if ws is None:
            ws = dict(scores=torch.empty(T, ld, dtype=torch.float32, device=q.device),
                      rows=torch.empty(T, self.topk, dtype=torch.int32, device=q.device),
                      lens=torch.empty(T, dtype=torch.int32, device=q.device))
            if q.is_cuda:
                self._ws[key] = ws
        seq = D.seq_of_rows(meta.q_start, T)
        scores = D.index_scores(q, w, idx_cache, meta, seq, ld, out=ws["scores"])
        return D.topk_rows(scores, meta, seq, self.topk, ws["rows"], ws["lens"])

    def tensors(self):
        return (self.wq_b.tensors() + self.wk.tensors() + self.weights_proj.tensors() +
                [self.k_norm_w, self.k_norm_b])


class MLAAttention:
    def __init__(self, cfg: ModelConfig, q_a: Linear | None, q_a_norm: torch.Tensor | None, q_b: Linear,
                 kv_a: Linear, kv_a_norm: torch.Tensor, kv_b: Linear, o: Linear, indexer: DSAIndexer | None = None):
        self.cfg = cfg
        self.indexer = indexer
        self.q_a, self.q_a_norm, self.q_b = q_a, q_a_norm, q_b
        self.kv_a, self.kv_a_norm, self.kv_b, self.o = kv_a, kv_a_norm, kv_b, o
        self.nh = cfg.num_heads
        self.dn, self.dr, self.dv, self.dc = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
        mscale = 1.0
        rs = cfg.rope_scaling
        if rs and rs.get("type", rs.get("rope_type")) == "yarn" and rs.get("mscale_all_dim"):
            f = float(rs["factor"])
            m = 0.1 * float(rs["mscale_all_dim"]) * math.log(f) + 1.0 if f > 1 else 1.0
            mscale = m * m
        self.scale = mscale / math.sqrt(self.dn + self.dr)
        self.latent_scale = 1.0    # fp8 latent cache: stored value = latent / latent_scale
        self._w_uk = None
        self._w_uv = None
        self._w_ukT = None
        self._dec = {}

    def _absorbed(self):
        """W_UK [nh, dn, dc] and W_UV [nh, dv, dc] (fp32 -> bf16) from kv_b [nh*(dn+dv), dc]."""
        if self._w_uk is None:
            w = self.kv_b.dense_weight().view(self.nh, self.dn + self.dv, self.dc)
            self._w_uk = w[:, : self.dn].to(torch.bfloat16).contiguous()
            self._w_uv = w[:, self.dn:].to(torch.bfloat16).contiguous()
            self._w_ukT = self._w_uk.transpose(1, 2).contiguous()      # [nh, dc, dn]: q_nope -> latent
        return self._w_uk, self._w_uv

    def _decode_plan(self, T: int, device):
        """Static per-T tensors of the absorbed decode GEMMs: head h's T rows form group h
        (rows h*T .. h*T+T-1 of the head-major operand), and row (h, t) lands in row t*nh + h."""
        key = (T, device)
        p = self._dec.get(key)
        if p is None:
            nh = self.nh
            seg = torch.arange(0, (nh + 1) * T, T, dtype=torch.int32, device=device)
            hh, tt = torch.meshgrid(torch.arange(nh, device=device), torch.arange(T, device=device), indexing="ij")
            dest = (tt * nh + hh).reshape(-1).to(torch.int32).contiguous()
            mx = G.max_mtiles(nh * T, nh)
            p = dict(seg=seg, dest=dest, tiles=torch.empty(mx * 4, dtype=torch.int32, device=device),
                     cnt=torch.zeros(1, dtype=torch.int32, device=device))
            self._dec[key] = p
        return p

    def _absorb_q(self, q_nope: torch.Tensor, q_rope: torch.Tensor) -> torch.Tensor:
        """[T, nh, dc + dr] decode queries: q_nope W_UK per head (a grouped tcgen05 GEMM whose
        epilogue scatters each head's rows into token order) next to the RoPE'd part."""
        T = q_nope.shape[0]
        nh, dc, dr = self.nh, self.dc, self.dr
        p = self._decode_plan(T, q_nope.device)
        a = q_nope.transpose(0, 1).reshape(nh * T, self.dn).contiguous()   # head-major rows
        qfull = torch.empty(T, nh, dc + dr, dtype=torch.bfloat16, device=q_nope.device)
        tiles = G.build_mtiles(p["seg"], nh * T, p["tiles"], p["cnt"])
        G.grouped_gemm(a, self._w_ukT, p["seg"], out=qfull.view(T * nh, dc + dr)[:, :dc], row_dest=p["dest"],
                       out_rows=T * nh, tiles=tiles)
        qfull[:, :, dc:].copy_(q_rope)
        return qfull

    def _absorb_o(self, o_lat: torch.Tensor) -> torch.Tensor:
        """[T, nh, dv] outputs: o_lat W_UV^T per head (grouped GEMM, rows scattered to token order)."""
        T = o_lat.shape[0]
        nh, dv = self.nh, self.dv
        p = self._decode_plan(T, o_lat.device)
        a = o_lat.transpose(0, 1).reshape(nh * T, self.dc).contiguous()
        o = torch.empty(T, nh, dv, dtype=torch.bfloat16, device=o_lat.device)
        tiles = G.build_mtiles(p["seg"], nh * T, p["tiles"], p["cnt"])
        G.grouped_gemm(a, self._w_uv, p["seg"], out=o.view(T * nh, dv), row_dest=p["dest"], out_rows=T * nh,
                       tiles=tiles)
        return o

    def __call__(self, x: torch.Tensor, meta: AttnMetadata, kv: tuple, rope: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        nh, dn, dr, dv, dc = self.nh, self.dn, self.dr, self.dv, self.dc
        if self.q_a is not None:
            qa = B.rmsnorm(self.q_a(x), self.q_a_norm, self.cfg.norm_eps)
            q = self.q_b(qa).view(T, nh, dn + dr)
        else:
            q = self.q_b(x).view(T, nh, dn + dr)
        ckv = self.kv_a(x)                                   # [T, dc + dr]
        latent = B.rmsnorm(ckv[:, :dc], self.kv_a_norm, self.cfg.norm_eps)
        k_rope = ckv[:, dc:].contiguous().view(T, 1, dr)
        q_rope = q[:, :, dn:].contiguous()
        if not self.cfg.mla_rope:
            pass                         # NoPE MLA: the rope dims take part in the scores unrotated
        elif x.is_cuda:
            B.rope_and_cache(q_rope, k_rope, k_rope, meta.positions, rope, dr, self.cfg.rope_neox)
        else:
            q_rope = B.apply_rope_ref(q_rope, meta.positions, rope, dr, self.cfg.rope_neox)
            k_rope = B.apply_rope_ref(k_rope, meta.positions, rope, dr, self.cfg.rope_neox)
        entry = torch.cat([latent, k_rope.view(T, dr)], dim=-1).view(T, 1, dc + dr)
        k_cache = kv[0]
        self._write_latent(entry, meta, k_cache)
        if k_cache.dtype == torch.float8_e4m3fn:
            # fp8 latent cache: the step's sequences' blocks, dequantised into a bf16 scratch
            # cache that the latent attention kernels read (block table remapped)
            k_cache, meta = dequant_latent_cache(k_cache, meta, self.latent_scale)
        q_nope = q[:, :, :dn]
        if self.indexer is not None:
            # DSA: the indexer sees every token; attention is sparse once a context can hold
            # more than index_topk tokens (before that the selection is the whole context)
            qi, wi = self.indexer.keys_and_queries(x, qa, meta, kv[1], rope)
            if meta.max_kv_len > self.indexer.topk:
                rows, lens = self.indexer.select(qi, wi, meta, kv[1], meta.max_kv_len)
                o = self._sparse(q_nope, q_rope, k_cache, rows, lens)
                return self.o(o.reshape(T, nh * dv))
        if meta.is_decode:
            w_uk, w_uv = self._absorbed()
            if x.is_cuda and dc % 128 == 0 and dn % 64 == 0 and dv % 16 == 0:
                qfull = self._absorb_q(q_nope, q_rope)
                o_lat = paged_attention(qfull, k_cache, None, meta, self.scale, v_dim=dc)  # [T, nh, dc]
                o = self._absorb_o(o_lat)
            else:
                qn = torch.einsum("thd,hdc->thc", q_nope.float(), w_uk.float()).to(torch.bfloat16)
                qfull = torch.cat([qn, q_rope.to(torch.bfloat16)], dim=-1).contiguous()   # [T, nh, dc+dr]
                o_lat = paged_attention(qfull, k_cache, None, meta, self.scale, v_dim=dc)
                o = torch.einsum("thc,hvc->thv", o_lat.float(), w_uv.float()).to(torch.bfloat16)
        else:
            o = self._prefill(q_nope, q_rope, meta, k_cache)
        return self.o(o.reshape(T, nh * dv))

    def _sparse(self, q_nope, q_rope, k_cache, rows, lens):
        """Absorbed attention of every query row over its selected latent rows (DSA), in
        chunks of query rows (each chunk's gathered rows are index_topk x 576 per row)."""
        from ..ops import dsa as D
        T = q_nope.shape[0]
        nh, dn, dv, dc = self.nh, self.dn, self.dv, self.dc
        w_uk, w_uv = self._absorbed()
        native = q_nope.is_cuda and dc % 128 == 0 and dn % 64 == 0 and dv % 16 == 0
        ch = T if T <= 64 else 256
        outs = []
        for s0 in range(0, T, ch):
            s1 = min(T, s0 + ch)
            qn, qr = q_nope[s0:s1], q_rope[s0:s1]
            if native:
                qfull = self._absorb_q(qn, qr)
            else:
                qfull = torch.cat([torch.einsum("thd,hdc->thc", qn.float(), w_uk.float()).to(torch.bfloat16),
                                   qr.to(torch.bfloat16)], dim=-1).contiguous()
            plan = None
            if q_nope.is_cuda:
                key = ("sparse", s1 - s0, q_nope.device)
                plan = self._dec.get(key)
                if plan is None:
                    plan = D.SparsePlan(s1 - s0, rows.shape[1], dc + self.dr, q_nope.device)
                    self._dec[key] = plan
            o_lat = D.sparse_mla(qfull, k_cache, rows[s0:s1], lens[s0:s1], self.scale, dc, plan)
            if native:
                outs.append(self._absorb_o(o_lat))
            else:
                outs.append(torch.einsum("thc,hvc->thv", o_lat.float(), w_uv.float()).to(torch.bfloat16))
        return outs[0] if len(outs) == 1 else torch.cat(outs)

    def _write_latent(self, entry, meta, k_cache):
        if k_cache.dtype == torch.float8_e4m3fn:
            write_latent_fp8(entry, meta.slot_mapping, k_cache, self.latent_scale)
            return
        B.write_cache_rows(entry.to(k_cache.dtype).contiguous(), meta.slot_mapping, k_cache)

    def _prefill(self, q_nope, q_rope, meta, k_cache):
        if q_nope.is_cuda and (self.dn + self.dr, self.dv) in ((192, 128), (128, 128), (64, 64), (256, 256)):
            return self._prefill_flash(q_nope, q_rope, meta, k_cache)
        return self._prefill_ref(q_nope, q_rope, meta, k_cache)

    def _prefill_flash(self, q_nope, q_rope, meta, k_cache):
        """All sequences of the step at once: their latent context blocks are gathered into
        one matrix, expanded by ONE kv_b GEMM into per-head K [., nh, dn+dr] and V [., nh, dv],
        laid out as a paged cache (sequence b owns a contiguous run of 64-token blocks), and
        ONE causal flash-attention launch covers every sequence (no [q, k] score matrix)."""
        nh, dn, dr, dv, dc = self.nh, self.dn, self.dr, self.dv, self.dc
        kl = meta.kv_len_host if meta.kv_len_host is not None else meta.kv_len.tolist()
        bs = k_cache.shape[2]
        d = q_nope.device
        nbs = [(n + bs - 1) // bs for n in kl]
        tot = sum(nbs)
        if tot == 0:
            return torch.zeros(q_nope.shape[0], nh, dv, dtype=torch.bfloat16, device=d)
        mx = max(nbs)
        # each sequence's first nb_b block ids, in order, and its run in the expanded cache
        sel = torch.zeros(meta.num_seqs, mx, dtype=torch.bool)
        new_bt = torch.zeros(meta.num_seqs, mx, dtype=torch.int32)
        off = 0
        for b, nb in enumerate(nbs):
            sel[b, :nb] = True
            new_bt[b, :nb] = torch.arange(off, off + nb, dtype=torch.int32)
            off += nb
        blocks = meta.block_table[:, :mx][sel.to(d)].long()                  # [tot]
        ent = k_cache[blocks, 0].reshape(tot * bs, dc + dr)
        kvb = self.kv_b(ent[:, :dc].contiguous()).view(tot * bs, nh, dn + dv)
        k = torch.cat([kvb[:, :, :dn], ent[:, dc:].view(tot * bs, 1, dr).expand(tot * bs, nh, dr)], dim=-1)
        kc = k.view(tot, bs, nh, dn + dr).permute(0, 2, 1, 3).contiguous()
        vc = kvb[:, :, dn:].reshape(tot, bs, nh, dv).permute(0, 2, 1, 3).contiguous()
        q = torch.cat([q_nope, q_rope.to(q_nope.dtype)], dim=-1).contiguous()
        m2 = AttnMetadata(num_seqs=meta.num_seqs, q_start=meta.q_start, kv_len=meta.kv_len,
                          block_table=new_bt.to(d, non_blocking=True), slot_mapping=meta.slot_mapping,
                          positions=meta.positions, max_q_len=meta.max_q_len, max_kv_len=meta.max_kv_len,
                          is_decode=False, q_start_host=meta.q_start_host, kv_len_host=meta.kv_len_host)
        return paged_attention(q, kc, vc, m2, self.scale)

    def _prefill_ref(self, q_nope, q_rope, meta, k_cache):
        """Expand latent -> per-head K/V for every context token, causal attention."""
        nh, dn, dr, dv, dc = self.nh, self.dn, self.dr, self.dv, self.dc
        T = q_nope.shape[0]
        qs = meta.q_start_host if meta.q_start_host is not None else meta.q_start.tolist()
        kl = meta.kv_len_host if meta.kv_len_host is not None else meta.kv_len.tolist()
        out = torch.empty(T, nh, dv, dtype=torch.bfloat16, device=q_nope.device)
        bs = k_cache.shape[2]
        for b in range(meta.num_seqs):
            s0, s1 = qs[b], qs[b + 1]
            if s1 == s0:
                continue
            n = kl[b]
            nb = (n + bs - 1) // bs
            ent = k_cache[meta.block_table[b, :nb].long(), 0].reshape(nb * bs, dc + dr)[:n]
            kvb = self.kv_b(ent[:, :dc].contiguous()).view(n, nh, dn + dv)
            k = torch.cat([kvb[:, :, :dn], ent[:, dc:].view(n, 1, dr).expand(n, nh, dr)], dim=-1)
            v = kvb[:, :, dn:]
            q = torch.cat([q_nope[s0:s1], q_rope[s0:s1]], dim=-1)
            ql = s1 - s0
            s = torch.einsum("qhd,khd->hqk", q.float(), k.float()) * self.scale
            pos = torch.arange(n - ql, n, device=q.device)
            mask = torch.arange(n, device=q.device)[None, :] > pos[:, None]
            p = torch.softmax(s.masked_fill(mask[None], float("-inf")), dim=-1)
            out[s0:s1] = torch.einsum("hqk,khd->qhd", p, v.float()).to(torch.bfloat16)
        return out

    def tensors(self):
        ts = self.q_b.tensors() + self.kv_a.tensors() + self.kv_b.tensors() + self.o.tensors() + [self.kv_a_norm]
        if self.q_a is not None:
            ts += self.q_a.tensors() + [self.q_a_norm]
        if self.indexer is not None:
            ts += self.indexer.tensors()
        return ts
