"""Building blocks of the decoder: linear, norms, GQA attention, dense MLP, MoE block.

Weights are held as plain tensors in kernel layout (no nn.Module overhead on the
decode path).  Every forward uses the ops in :mod:`vllm_xtu_moe_b200.ops`, which
dispatch to the sm_100a kernels on a GPU and to PyTorch restatements on a CPU.
"""
from __future__ import annotations

import dataclasses

import math

import torch

from ..ops import basic as B
from ..ops import gemm as G
from ..ops import moe as M
from ..ops.attention import AttnMetadata, paged_attention
from ..ops.router import router_topk
from .config import ModelConfig


class Linear:
    """y = x W^T (+ b); W bf16 [N, K] or e4m3 [N, K] with fp32 block scales."""

    def __init__(self, weight: torch.Tensor, scale: torch.Tensor | None = None, bias: torch.Tensor | None = None):
        self.weight = weight
        self.scale = scale
        self.bias = bias

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    def __call__(self, x: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
        if not x.is_cuda and x.dtype == torch.float32:
            out_dtype = torch.float32   # CPU fp32-activation mode (exact-reference runs)
        return G.linear(x, self.weight, self.scale, out_dtype=out_dtype, bias=self.bias)

    def dense_weight(self) -> torch.Tensor:
        if self.scale is None:
            return self.weight.float()
        from ..ops.quant import dequant_fp8_block
        return dequant_fp8_block(self.weight, self.scale)

    def tensors(self):
        return [t for t in (self.weight, self.scale, self.bias) if t is not None]


class RMSNorm:
    def __init__(self, weight: torch.Tensor, eps: float, add_one: bool = False):
        self.weight, self.eps, self.add_one = weight, eps, add_one
        # set when the consumers are fp8-weight decode GEMVs: decode-size calls then also
        # write the f16 x 2^-8 copy those GEMVs read (attached as y.xtu_f16s)
        self.emit_f16s = False

    def __call__(self, x, residual=None):
        f16s = self.emit_f16s and x.is_cuda and x.dim() == 2 and x.shape[0] <= G.DECODE_MAX_M
        return B.rmsnorm(x, self.weight, self.eps, residual=residual, add_one=self.add_one, f16s=f16s)

    def tensors(self):
        return [self.weight]


class GQAAttention:
    """Grouped-query attention with partial RoPE, optional qkv bias, per-head q/k
    norm and a sigmoid output gate (Qwen3-Next), over the paged KV cache; optionally a
    sliding window, learned per-head sink logits and a value width other than the
    q/k width (MiMo-V2)."""

    def __init__(self, cfg: ModelConfig, qkv: Linear, o: Linear, q_norm: torch.Tensor | None = None,
                 k_norm: torch.Tensor | None = None, num_kv_heads: int | None = None, window: int = 0,
                 sinks: torch.Tensor | None = None):
        self.cfg = cfg
        self.qkv = qkv
        self.o = o
        self.q_norm, self.k_norm = q_norm, k_norm
        self.nh, self.hd, self.vd = cfg.num_heads, cfg.head_dim, cfg.gqa_v_dim
        self.nkv = num_kv_heads if num_kv_heads is not None else cfg.num_kv_heads
        self.window = window
        self.bounded = False        # set by the runner when this window layer has its own bounded pool
        self.sinks = sinks.float().contiguous() if sinks is not None else None
        self.scale = 1.0 / math.sqrt(self.hd)
        # dequantisation scales of an fp8 KV cache (checkpoint k_scale / v_scale; 1 by default)
        self.k_scale = 1.0
        self.v_scale = 1.0

    def __call__(self, x: torch.Tensor, meta: AttnMetadata, kv: tuple, rope: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        nh, nkv, hd, vd = self.nh, self.nkv, self.hd, self.vd
        y = self.qkv(x)
        gate = None
        if self.cfg.attn_output_gate:
            # per head: [q (hd) | gate (hd)] for nh heads, then k, v
            qg = y[:, : 2 * nh * hd].view(T, nh, 2 * hd)
            q = qg[:, :, :hd].contiguous()
            gate = qg[:, :, hd:]
            k = y[:, 2 * nh * hd: 2 * nh * hd + nkv * hd].view(T, nkv, hd)
            v = y[:, 2 * nh * hd + nkv * hd:].view(T, nkv, vd)
        else:
            q = y[:, : nh * hd].view(T, nh, hd)
            k = y[:, nh * hd: (nh + nkv) * hd].view(T, nkv, hd)
            v = y[:, (nh + nkv) * hd:].view(T, nkv, vd)
        k_cache, v_cache = kv
        if self.bounded:            # the sliding-window pool: its own block table and write slots
            if meta.swa_block_table is None:
                raise RuntimeError("a bounded sliding-window cache needs the step's window block table")
            meta = dataclasses.replace(meta, block_table=meta.swa_block_table, slot_mapping=meta.swa_slot_mapping)
        B.rope_and_cache(q, k, v, meta.positions, rope, self.cfg.rot_dim, self.cfg.rope_neox,
                         slot_mapping=meta.slot_mapping, k_cache=k_cache, v_cache=v_cache, q_norm_w=self.q_norm,
                         k_norm_w=self.k_norm, norm_eps=self.cfg.norm_eps, norm_add_one=self.cfg.norm_add_one,
                         k_scale=self.k_scale, v_scale=self.v_scale)
        o = paged_attention(q, k_cache, v_cache, meta, self.scale, window=self.window, sinks=self.sinks,
                            k_scale=self.k_scale, v_scale=self.v_scale)
        if gate is not None:
            B.gate_mul_(o, gate)
        return self.o(o.reshape(T, nh * vd))

    def tensors(self):
        ts = self.qkv.tensors() + self.o.tensors()
        return ts + [t for t in (self.q_norm, self.k_norm, self.sinks) if t is not None]


class DenseMLP:
    """SwiGLU MLP; gate/up rows interleaved in 128-row blocks when the width allows
    (the GEMM epilogue then applies SwiGLU)."""

    def __init__(self, gate_up: Linear, down: Linear, interleaved: bool, limit: float = 0.0):
        self.gate_up, self.down, self.interleaved, self.limit = gate_up, down, interleaved, limit
        self._seg = {}

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        T = x.shape[0]
        if (x.is_cuda and self.interleaved and T <= G.DECODE_MAX_M and x.shape[1] % 128 == 0
                and self.down.weight.shape[1] % 128 == 0):
            return M.dense_swiglu_gemv(x.contiguous(), self.gate_up.weight, self.gate_up.scale, self.down.weight,
                                       self.down.scale, self.limit, self._seg)
        if x.is_cuda and self.interleaved:
            seg = self._seg.get((x.device, T))
            if seg is None:
                seg = torch.tensor([0, T], dtype=torch.int32, device=x.device)
                self._seg[(x.device, T)] = seg
            w = self.gate_up.weight.unsqueeze(0)
            s = self.gate_up.scale.unsqueeze(0) if self.gate_up.scale is not None else None
            h = G.grouped_gemm(x.contiguous(), w, seg, w_scale=s, epilogue=G.EPI_SWIGLU, act_limit=self.limit,
                               out=torch.empty(T, w.shape[1] // 2, dtype=torch.bfloat16, device=x.device))
        else:
            y = self.gate_up(x)
            if self.interleaved:
                I = y.shape[1] // 2
                yb = y.view(T, I // 128, 2, 128)
                h = G.silu_and_mul_clamped(yb[:, :, 0], yb[:, :, 1], self.limit).reshape(T, I).to(x.dtype)
            else:
                h = B.silu_mul(y, self.limit)
        return self.down(h)

    def tensors(self):
        return self.gate_up.tensors() + self.down.tensors()


class MoEBlock:
    """Router + routed experts (+ shared expert, optionally sigmoid-gated).

    The routed experts are executed by an expert executor (see
    :mod:`vllm_xtu_moe_b200.tiering`) that decides, per call, which pairs run on
    GPU-resident experts, on the streamed ring, or on the CPU engine.  Without an
    executor, all experts are GPU resident.
    """

    def __init__(self, cfg: ModelConfig, layer_idx: int, gate: torch.Tensor, gate_bias: torch.Tensor | None,
                 experts: M.ExpertWeights | None, shared: DenseMLP | None, shared_gate: torch.Tensor | None):
        self.cfg = cfg
        self.layer_idx = layer_idx
        self.gate = gate                  # [E, H] bf16 (router weight, kept unquantized)
        self.gate_bias = gate_bias        # [E] fp32 correction bias
        self.experts = experts            # GPU-resident routed experts (None when tiered)
        self.shared = shared
        self.shared_gate = shared_gate    # [1, H] (Qwen3-Next)
        self.executor = None              # set by the tier planner
        self.ws: M.MoEWorkspace | None = None
        self.last_ids: torch.Tensor | None = None
        self.tracer = None                # utils.trace.Tracer (routing dump) when enabled
        self.trace_idx = layer_idx
        self.expert_lo = 0                # first global expert id held here (expert parallel over TP ranks)
        from ..utils.diagnostics import selfcheck_enabled
        self.selfcheck_pending = selfcheck_enabled()   # XIAOTU_MOE_SELFCHECK: verify one real call

    def route(self, x: torch.Tensor):
        logits = G.linear(x, self.gate, out_dtype=torch.float32)
        c = self.cfg
        return router_topk(logits, c.top_k, c.scoring, self.gate_bias, c.n_group, c.topk_group, c.norm_topk_prob,
                           c.routed_scale)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.selfcheck_pending and x.shape[0] <= 64:
            y = self._checked_call(x)
            if y is not None:
                return y
        c = self.cfg
        permuted = False
        if self.executor is None and M.decode_route_ok(x, self.gate, self.experts, c.top_k, c.n_group):
            # decode: router and permute in one launch, straight into the MoE workspace
            bias = self.gate_bias.float() if self.gate_bias is not None else None
            ids, w = M.route_decode(x, self.gate, bias, c.top_k, c.scoring, c.n_group, c.topk_group,
                                    c.norm_topk_prob, c.routed_scale, self.workspace(x), self.expert_lo,
                                    self.experts.num_experts)
            permuted = True
        else:
            ids, w = self.route(x)
        self.last_ids = ids
        if self.tracer is not None and self.tracer.routing is not None:
            self.tracer.routing.record(self.trace_idx, ids)
        sh = None
        if (self.shared is not None and self.shared_gate is None and self.executor is None and x.is_cuda
                and (x.shape[0] <= G.GEMV_MAX_M or permuted) and x.shape[0] <= G.DECODE_MAX_M
                and M.shared_fusable(self.shared, self.experts, self.cfg.swiglu_limit)):
            # decode: the shared expert runs inside the routed experts' GEMV launches
            return M.fused_moe(x, ids, w, self.experts, self.workspace(x), lo=self.expert_lo,
                               act_limit=self.cfg.swiglu_limit, shared_mlp=self.shared, permuted=permuted)
        if self.shared is not None:
            sh = self.shared(x)
            if self.shared_gate is not None:
                sh = B.shared_gate_(sh, x, self.shared_gate)
        if self.executor is not None:
            return self.executor(self, x, ids, w, sh)
        return M.fused_moe(x, ids, w, self.experts, self.workspace(x), lo=self.expert_lo, shared=sh,
                           act_limit=self.cfg.swiglu_limit, permuted=permuted)

    def _checked_call(self, x: torch.Tensor) -> torch.Tensor | None:
        """XIAOTU_MOE_SELFCHECK: this call's routed experts once more on the plain path (no
        shared expert), compared with an fp32 recomputation from the layer's own weights
        (utils.diagnostics.moe_selfcheck); returns the layer output, or None when the call
        does not qualify (then the normal path runs)."""
        from ..utils import diagnostics as D
        if x.is_cuda and torch.cuda.is_current_stream_capturing():
            return None
        ids, w = self.route(x)
        if self.executor is not None:
            routed = self.executor(self, x, ids, w, None)
        else:
            routed = M.fused_moe(x.contiguous(), ids.to(torch.int32).contiguous(), w.float().contiguous(),
                                 self.experts, self.workspace(x), lo=self.expert_lo, act_limit=self.cfg.swiglu_limit)
        if D.moe_selfcheck(self, x, ids, w, routed) is None:
            return None
        self.selfcheck_pending = False
        self.last_ids = ids
        if self.shared is None:
            return routed
        sh = self.shared(x)
        if self.shared_gate is not None:
            sh = B.shared_gate_(sh, x, self.shared_gate)
        return (routed.float() + sh.float()).to(x.dtype)

    def workspace(self, x: torch.Tensor) -> M.MoEWorkspace | None:
        if not x.is_cuda:
            return None
        T = x.shape[0]
        if self.ws is None or self.ws.max_tokens < T or self.ws.device != x.device:
            self.ws = M.MoEWorkspace(max(T, 16), self.cfg.top_k, self.experts.num_experts, self.cfg.hidden_size,
                                     self.experts.inter, x.device)
        return self.ws

    def tensors(self):
        ts = [self.gate] + ([self.gate_bias] if self.gate_bias is not None else [])
        if self.experts is not None:
            ts += [t for t in (self.experts.w13, self.experts.w2, self.experts.s13, self.experts.s2) if t is not None]
        if self.shared is not None:
            ts += self.shared.tensors()
        if self.shared_gate is not None:
            ts.append(self.shared_gate)
        return ts
