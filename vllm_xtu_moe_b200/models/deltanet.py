"""Gated DeltaNet linear attention (Qwen3-Next "linear_attention" layers).

Per value head h, with L2-normalised q, k (q additionally scaled by 1/sqrt(dk)),
decay g_t = -exp(A_log) * softplus(a_t + dt_bias) and write strength
beta_t = sigmoid(b_t), the state S [dk, dv] evolves as

    S <- exp(g_t) * S
    S <- S + k_t (beta_t (v_t - S^T k_t))^T
    o_t = S^T q_t

followed by a gated RMSNorm (rmsnorm(o) * w * silu(z)) and the output
projection.  A causal depthwise conv (kernel 4, SiLU) runs over the
concatenated q/k/v channels first.  Recurrent state and conv state are kept
per request slot between steps (``DeltaNetState``).

Kimi Delta Attention (KDA, ``KimiDeltaAttention``) is the same recurrence with a decay per
key dimension: g_t [nv, dk] = -exp(A_log) * softplus(f_b(f_a(x)) + dt_bias), applied as
S <- Diag(exp(g_t)) S; its q, k, v come from separate projections (concatenated here),
beta from its own projection, and the output gate is sigmoid(g_b(g_a(x))) in place of
silu(z).

The per-token recurrence in ``_delta_rule_ref`` is the numerics oracle; on a
GPU (key head dim 128) the conv / recurrence kernels of ``csrc/cuda/deltanet.cu`` run.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from ..ops import _native as N
from ..ops.attention import AttnMetadata
from .config import ModelConfig
from .layers import Linear


class DeltaNetState:
    """Recurrent state [slots, nv, dk, dv] fp32 and conv state [slots, channels, kernel-1].

    With speculative decoding (``enable_spec(k)``) each slot also has k + 1 copies of both,
    ``spec_ssm`` / ``spec_conv``: a verification step writes the states after each of its
    (at most k + 1) tokens there, and ``commit_spec`` installs, per sequence, the ones after
    its last accepted token -- the rollback of rejected drafts."""

    def __init__(self, cfg: ModelConfig, max_slots: int, device):
        nv, dk, dv = cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        ch = 2 * cfg.linear_num_key_heads * dk + nv * dv
        self.ssm = torch.zeros(max_slots, nv, dk, dv, dtype=torch.float32, device=device)
        self.conv = torch.zeros(max_slots, ch, cfg.linear_conv_kernel - 1, dtype=torch.bfloat16, device=device)
        self.spec_ssm: torch.Tensor | None = None
        self.spec_conv: torch.Tensor | None = None

    def enable_spec(self, k: int) -> None:
        n = k + 1
        if self.spec_ssm is not None and self.spec_ssm.shape[1] >= n:
            return
        self.spec_ssm = torch.zeros(self.ssm.shape[0], n, *self.ssm.shape[1:], dtype=torch.float32,
                                    device=self.ssm.device)
        self.spec_conv = torch.zeros(self.conv.shape[0], n, *self.conv.shape[1:], dtype=torch.bfloat16,
                                     device=self.conv.device)

    def commit_spec(self, accepted: torch.Tensor, slots: torch.Tensor) -> None:
        """Per sequence b with slot >= 0: states <- the copies after position accepted[b]."""
        n = self.spec_ssm.shape[1]
        if self.ssm.is_cuda:
            from ..ops import _native as N
            N.call("xtu_deltanet_spec_commit", accepted.data_ptr(), slots.data_ptr(), slots.numel(), n,
                   self.spec_ssm.data_ptr(), self.ssm.data_ptr(), self.ssm[0].numel(), self.spec_conv.data_ptr(),
                   self.conv.data_ptr(), self.conv[0].numel(), N.stream_ptr(self.ssm.device))
            return
        for a, sl in zip(accepted.tolist(), slots.tolist()):
            if sl >= 0:
                a = min(max(int(a), 0), n - 1)
                self.ssm[sl].copy_(self.spec_ssm[sl, a])
                self.conv[sl].copy_(self.spec_conv[sl, a])

    def nbytes(self) -> int:
        n = self.ssm.numel() * 4 + self.conv.numel() * 2
        if self.spec_ssm is not None:
            n += self.spec_ssm.numel() * 4 + self.spec_conv.numel() * 2
        return n


def _delta_rule_ref(q, k, v, g, beta, state, per_token: torch.Tensor | None = None):
    """q,k [T, H, dk], v [T, H, dv], g [T, H] (or [T, H, dk]: a decay per key dim), beta [T, H];
    state [H, dk, dv] (updated in place); per_token [>= T, H, dk, dv]: the state after each token."""
    T = q.shape[0]
    out = torch.empty(T, v.shape[1], v.shape[2], dtype=torch.float32, device=q.device)
    S = state
    for t in range(T):
        S.mul_(torch.exp(g[t])[:, :, None] if g.dim() == 3 else torch.exp(g[t])[:, None, None])
        kv_mem = torch.einsum("hkv,hk->hv", S, k[t])
        delta = (v[t] - kv_mem) * beta[t][:, None]
        S.add_(torch.einsum("hk,hv->hkv", k[t], delta))
        out[t] = torch.einsum("hkv,hk->hv", S, q[t])
        if per_token is not None and t < per_token.shape[0]:
            per_token[t].copy_(S)
    return out


class GatedDeltaNet:
    def __init__(self, cfg: ModelConfig, in_qkvz: Linear, in_ba: Linear, conv_w: torch.Tensor, A_log: torch.Tensor,
                 dt_bias: torch.Tensor, norm_w: torch.Tensor, out: Linear):
        self.cfg = cfg
        self.in_qkvz, self.in_ba, self.conv_w = in_qkvz, in_ba, conv_w   # conv_w [channels, kernel]
        self.A_log, self.dt_bias, self.norm_w, self.out = A_log, dt_bias, norm_w, out
        self.nk, self.nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self.state: DeltaNetState | None = None

    def _split(self, qkvz, ba):
        T = qkvz.shape[0]
        nk, nv, dk, dv = self.nk, self.nv, self.dk, self.dv
        r = nv // nk
        x = qkvz.view(T, nk, 2 * dk + 2 * r * dv)
        q = x[:, :, :dk].reshape(T, nk * dk)
        k = x[:, :, dk:2 * dk].reshape(T, nk * dk)
        v = x[:, :, 2 * dk:2 * dk + r * dv].reshape(T, nv * dv)
        z = x[:, :, 2 * dk + r * dv:].reshape(T, nv, dv)
        bav = ba.view(T, nk, 2 * r)
        b = bav[:, :, :r].reshape(T, nv)
        a = bav[:, :, r:].reshape(T, nv)
        return q, k, v, z, b, a

    def _f32(self, name: str, t: torch.Tensor, device) -> torch.Tensor:
        """fp32 contiguous copy of a small parameter, made once per device."""
        c = getattr(self, name, None)
        if c is None or c.device != device:
            c = t.float().contiguous().to(device)
            setattr(self, name, c)
        return c

    def __call__(self, x: torch.Tensor, meta: AttnMetadata, kv, rope) -> torch.Tensor:
        state: DeltaNetState = kv
        T = x.shape[0]
        qkvz = self.in_qkvz(x)
        ba = self.in_ba(x)
        if x.is_cuda and N.has_symbol("xtu_deltanet_fwd") and self.dk == 128:
            # gates, conv, recurrence and gated RMSNorm in the deltanet kernels
            from ..ops.deltanet import deltanet_fwd
            d = x.device
            y = deltanet_fwd(qkvz.contiguous(), self._f32("_conv_w32", self.conv_w, d), None, None, meta, state,
                             self.nk, self.nv, self.dk, self.dv, ba=ba.contiguous(),
                             A_log32=self._f32("_A_log32", self.A_log, d),
                             dt_bias32=self._f32("_dt_bias32", self.dt_bias, d),
                             norm_w32=self._f32("_norm_w32", self.norm_w, d), eps=self.cfg.norm_eps)
            return self.out(y)
        q, k, v, z, b, a = self._split(qkvz, ba)
        beta = torch.sigmoid(b.float())
        g = -torch.exp(self.A_log.float()) * F.softplus(a.float() + self.dt_bias.float())
        mixed = torch.cat([q, k, v], dim=-1)        # [T, channels]
        o = self._core(mixed, g, beta, meta, state)  # [T, nv, dv] fp32
        o = self._gated_norm(o, z)
        return self.out(o.reshape(T, self.nv * self.dv))

    def _gated_norm(self, o, z):
        of = o.float()
        y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + self.cfg.norm_eps)
        y = y * self.norm_w.float() * F.silu(z.float())
        return y.to(torch.bfloat16)

    def _core(self, mixed, g, beta, meta, state):
        if mixed.is_cuda and N.native_required() and self.dk == 128:
            raise N.NativeLibraryMissing("xtu_deltanet_fwd missing from the CUDA library")
        return deltanet_ref(mixed, self.conv_w, g, beta, meta, state, self.nk, self.nv, self.dk, self.dv)

    def tensors(self):
        return (self.in_qkvz.tensors() + self.in_ba.tensors() + self.out.tensors() +
                [self.conv_w, self.A_log, self.dt_bias, self.norm_w])


class KimiDeltaAttention:
    """Kimi Delta Attention layer: conv + L2-normalised q/k, the delta rule with a decay per
    key dimension, RMSNorm of the output times sigmoid(output gate), output projection.
    Weights: in_qkv rows [Q | K | V] (q_proj, k_proj, v_proj), in_b [nv, H], the low-rank
    decay f_a [dk, H] / f_b [nv*dk, dk] with dt_bias [nv*dk] and A_log [nv], the low-rank
    gate g_a [dk, H] / g_b [nv*dv, dk], conv [channels, kernel], norm weight [dv]."""

    def __init__(self, cfg: ModelConfig, in_qkv: Linear, in_b: Linear, f_a: Linear, f_b: Linear, g_a: Linear,
                 g_b: Linear, conv_w: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
                 norm_w: torch.Tensor, out: Linear):
        self.cfg = cfg
        self.in_qkv, self.in_b, self.f_a, self.f_b, self.g_a, self.g_b = in_qkv, in_b, f_a, f_b, g_a, g_b
        self.conv_w, self.A_log, self.dt_bias, self.norm_w, self.out = conv_w, A_log, dt_bias, norm_w, out
        self.nk, self.nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim

    _f32 = GatedDeltaNet._f32

    def decay(self, x: torch.Tensor) -> torch.Tensor:
        """g [T, nv, dk] fp32."""
        T = x.shape[0]
        raw = self.f_b(self.f_a(x)).float().view(T, self.nv, self.dk)
        return -torch.exp(self.A_log.float()).view(1, self.nv, 1) * F.softplus(
            raw + self.dt_bias.float().view(1, self.nv, self.dk))

    def __call__(self, x: torch.Tensor, meta: AttnMetadata, kv, rope) -> torch.Tensor:
        state: DeltaNetState = kv
        T = x.shape[0]
        qkv = self.in_qkv(x)
        beta = torch.sigmoid(self.in_b(x).float())
        g = self.decay(x)
        gate = self.g_b(self.g_a(x)).view(T, self.nv, self.dv)
        if x.is_cuda and N.has_symbol("xtu_deltanet_fwd") and self.dk == 128:
            # conv, recurrence and the sigmoid-gated RMSNorm in the deltanet kernels
            from ..ops.deltanet import deltanet_fwd
            d = x.device
            y = deltanet_fwd(qkv.contiguous(), self._f32("_conv_w32", self.conv_w, d), g.contiguous(), beta, meta,
                             state, self.nk, self.nv, self.dk, self.dv, blocked=True,
                             norm_w32=self._f32("_norm_w32", self.norm_w, d), eps=self.cfg.norm_eps,
                             gate=gate.reshape(T, self.nv * self.dv).contiguous())
            return self.out(y)
        else:
            if x.is_cuda and N.native_required() and self.dk == 128:
                raise N.NativeLibraryMissing("xtu_deltanet_fwd missing from the CUDA library")
            o = deltanet_ref(qkv, self.conv_w, g, beta, meta, state, self.nk, self.nv, self.dk, self.dv)
        of = o.float()
        y = of * torch.rsqrt(of.pow(2).mean(-1, keepdim=True) + self.cfg.norm_eps)
        y = (y * self.norm_w.float() * torch.sigmoid(gate.float())).to(x.dtype)
        return self.out(y.reshape(T, self.nv * self.dv))

    def tensors(self):
        ts = []
        for lin in (self.in_qkv, self.in_b, self.f_a, self.f_b, self.g_a, self.g_b, self.out):
            ts += lin.tensors()
        return ts + [self.conv_w, self.A_log, self.dt_bias, self.norm_w]


def deltanet_ref(mixed, conv_w, g, beta, meta, state: DeltaNetState, nk, nv, dk, dv):
    """Causal conv (with carried state) + gated delta rule per sequence (fp32)."""
    T, ch = mixed.shape
    kw = conv_w.shape[1]
    qs = meta.q_start_host if meta.q_start_host is not None else meta.q_start.tolist()
    slots = meta.seq_slots.tolist()
    fresh = meta.seq_fresh.tolist() if meta.seq_fresh is not None else [0] * meta.num_seqs
    out = torch.empty(T, nv, dv, dtype=torch.float32, device=mixed.device)
    r = nv // nk
    for bi in range(meta.num_seqs):
        s0, s1 = qs[bi], qs[bi + 1]
        if s1 == s0:
            continue
        slot = slots[bi]
        if slot < 0:      # padding sequence of a captured decode graph: zero state, nothing kept
            conv_st, ssm_st = torch.zeros_like(state.conv[0]), torch.zeros_like(state.ssm[0])
        else:
            conv_st, ssm_st = state.conv[slot], state.ssm[slot]
        if fresh[bi]:
            conv_st.zero_()
            ssm_st.zero_()
        xs = mixed[s0:s1].float()                                  # [L, ch]
        hist = conv_st.float().t()                                 # [kw-1, ch]
        full = torch.cat([hist, xs], dim=0)                        # [kw-1+L, ch]
        L = s1 - s0
        w = conv_w.float()                                          # [ch, kw]
        conv = torch.zeros(L, ch, device=mixed.device)
        for j in range(kw):
            conv += full[j:j + L] * w[:, j]
        conv = F.silu(conv)
        spec = getattr(meta, "spec_rows", 0) > 0 and state.spec_ssm is not None and slot >= 0
        if spec:       # the conv state after each token j: inputs j+1 .. j+kw-1 of [history ++ step]
            for j in range(min(L, state.spec_conv.shape[1])):
                state.spec_conv[slot, j].copy_(full[j + 1:j + kw].t().to(state.conv.dtype))
        conv_st.copy_(full[-(kw - 1):].t().to(state.conv.dtype))
        q = conv[:, : nk * dk].view(L, nk, dk)
        k = conv[:, nk * dk: 2 * nk * dk].view(L, nk, dk)
        v = conv[:, 2 * nk * dk:].view(L, nv, dv)
        q = F.normalize(q, dim=-1) / math.sqrt(dk)
        k = F.normalize(k, dim=-1)
        q = q.repeat_interleave(r, dim=1)
        k = k.repeat_interleave(r, dim=1)
        out[s0:s1] = _delta_rule_ref(q, k, v, g[s0:s1], beta[s0:s1], ssm_st,
                                     state.spec_ssm[slot] if spec else None)
    return out
