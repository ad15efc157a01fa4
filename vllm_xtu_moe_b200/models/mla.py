"""Multi-head latent attention (DeepSeek-V3 family) over a paged latent cache.

Cache: one latent "head" per token, ``[num_blocks, 1, block_size, kv_lora + rope]``
(the normalised compressed KV followed by the RoPE'd shared key).  Prefill
expands the latent into per-head K/V (qk dim = nope + rope, v dim = v_head_dim)
and runs causal attention; decode absorbs W_UK into the query and W_UV into the
output so attention runs directly over the 576-wide latent (MQA-like: all 128
heads share one KV "head"), which is what makes MLA decode bandwidth-cheap.
"""
from __future__ import annotations

import math

import torch

from ..ops import basic as B
from ..ops.attention import AttnMetadata, paged_attention
from .config import ModelConfig
from .layers import Linear


class MLAAttention:
    def __init__(self, cfg: ModelConfig, q_a: Linear | None, q_a_norm: torch.Tensor | None, q_b: Linear,
                 kv_a: Linear, kv_a_norm: torch.Tensor, kv_b: Linear, o: Linear):
        self.cfg = cfg
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
        self._w_uk = None
        self._w_uv = None

    def _absorbed(self):
        """W_UK [nh, dn, dc] and W_UV [nh, dv, dc] (fp32 -> bf16) from kv_b [nh*(dn+dv), dc]."""
        if self._w_uk is None:
            w = self.kv_b.dense_weight().view(self.nh, self.dn + self.dv, self.dc)
            self._w_uk = w[:, : self.dn].to(torch.bfloat16).contiguous()
            self._w_uv = w[:, self.dn:].to(torch.bfloat16).contiguous()
        return self._w_uk, self._w_uv

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
        q_nope = q[:, :, :dn]
        if meta.is_decode:
            w_uk, w_uv = self._absorbed()
            qn = torch.einsum("thd,hdc->thc", q_nope.float(), w_uk.float()).to(torch.bfloat16)
            qfull = torch.cat([qn, q_rope.to(torch.bfloat16)], dim=-1).contiguous()   # [T, nh, dc+dr]
            o_lat = paged_attention(qfull, k_cache, None, meta, self.scale, v_dim=dc)  # [T, nh, dc]
            o = torch.einsum("thc,hvc->thv", o_lat.float(), w_uv.float()).to(torch.bfloat16)
        else:
            o = self._prefill(q_nope, q_rope, meta, k_cache)
        return self.o(o.reshape(T, nh * dv))

    def _write_latent(self, entry, meta, k_cache):
        B.write_cache_rows(entry.to(k_cache.dtype).contiguous(), meta.slot_mapping, k_cache)

    def _prefill(self, q_nope, q_rope, meta, k_cache):
        if q_nope.is_cuda and (self.dn + self.dr, self.dv) in ((192, 128), (128, 128), (64, 64), (256, 256)):
            return self._prefill_flash(q_nope, q_rope, meta, k_cache)
        return self._prefill_ref(q_nope, q_rope, meta, k_cache)

    def _prefill_flash(self, q_nope, q_rope, meta, k_cache):
        """Expand each sequence's latent context into per-head K [n, nh, dn+dr] and V
        [n, nh, dv], lay them out as a paged cache of 64-token blocks, and run the causal
        flash kernel (no [q, k] score matrix is ever materialised)."""
        nh, dn, dr, dv, dc = self.nh, self.dn, self.dr, self.dv, self.dc
        T = q_nope.shape[0]
        qs = meta.q_start_host if meta.q_start_host is not None else meta.q_start.tolist()
        kl = meta.kv_len_host if meta.kv_len_host is not None else meta.kv_len.tolist()
        out = torch.empty(T, nh, dv, dtype=torch.bfloat16, device=q_nope.device)
        bs = k_cache.shape[2]
        d = q_nope.device
        for b in range(meta.num_seqs):
            s0, s1 = qs[b], qs[b + 1]
            if s1 == s0:
                continue
            n = kl[b]
            nb = (n + bs - 1) // bs
            ent = k_cache[meta.block_table[b, :nb].long(), 0].reshape(nb * bs, dc + dr)
            kvb = self.kv_b(ent[:, :dc].contiguous()).view(nb * bs, nh, dn + dv)
            k = torch.cat([kvb[:, :, :dn], ent[:, dc:].view(nb * bs, 1, dr).expand(nb * bs, nh, dr)], dim=-1)
            kc = k.view(nb, bs, nh, dn + dr).permute(0, 2, 1, 3).contiguous()
            vc = kvb[:, :, dn:].reshape(nb, bs, nh, dv).permute(0, 2, 1, 3).contiguous()
            q = torch.cat([q_nope[s0:s1], q_rope[s0:s1].to(q_nope.dtype)], dim=-1).contiguous()
            ql = s1 - s0
            m1 = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, ql], dtype=torch.int32, device=d),
                              kv_len=torch.tensor([n], dtype=torch.int32, device=d),
                              block_table=torch.arange(nb, dtype=torch.int32, device=d).view(1, nb),
                              slot_mapping=meta.slot_mapping[s0:s1], positions=meta.positions[s0:s1], max_q_len=ql,
                              max_kv_len=n, is_decode=False, q_start_host=[0, ql], kv_len_host=[n])
            out[s0:s1] = paged_attention(q, kc, vc, m1, self.scale)
        return out

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
        return ts
