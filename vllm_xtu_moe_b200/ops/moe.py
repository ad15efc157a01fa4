"""GPU MoE layer: route -> permute -> grouped gate/up GEMM (+SwiGLU) -> grouped
down GEMM (x top-k weight, scattered to the pair's slot) -> per-token combine.

Replaces the reference's streamed-layer kernels (vllm_xiaotu_moe/gpu_prefill.py:
2566 ``gpu_moe_layer``; gpu_prefill_fp8.py:458 ``gpu_moe_layer_fp8``) with one
graph-capturable pipeline whose buffers are sized once (``MoEWorkspace``).

Tier split: only pairs whose expert id falls in ``[lo, hi)`` are computed here;
others (experts of another EP rank, or of the CPU tier) are skipped by the
permute and contribute through ``extra`` in the combine.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _native as N
from . import gemm as G
from .quant import dequant_fp8_block, dequant_mxfp4, dequant_nvfp4


@dataclass
class ExpertWeights:
    """Routed-expert weights of one layer in GPU-kernel layout.

    fmt: "bf16" or "fp8" (e4m3 + 128x128 fp32 block scales).
    w13: [E, 2I, H]; when ``interleaved``, rows are arranged in 256-row blocks of
    (128 gate rows, 128 up rows) so the gate/up GEMM can fuse SwiGLU.
    w2:  [E, H, I].
    """
    fmt: str
    w13: torch.Tensor
    w2: torch.Tensor
    s13: torch.Tensor | None = None
    s2: torch.Tensor | None = None
    interleaved: bool = False
    gs13: torch.Tensor | None = None  # nvfp4 per-expert global scales
    gs2: torch.Tensor | None = None

    @property
    def num_experts(self) -> int:
        return self.w13.shape[0]

    @property
    def hidden(self) -> int:
        return self.w13.shape[2] if self.fmt in ("bf16", "fp8") else self.w13.shape[2] * 2

    @property
    def inter(self) -> int:
        return self.w13.shape[1] // 2

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.w13, self.w2, self.s13, self.s2) if t is not None)

    def dequant(self, e: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense fp32 (w13 [2I,H] in gate-then-up order, w2 [H,I]) of expert e."""
        if self.fmt == "bf16":
            w13, w2 = self.w13[e].float(), self.w2[e].float()
            s13 = None
        elif self.fmt == "fp8":
            w13 = dequant_fp8_block(self.w13[e], self.s13[e])
            w2 = dequant_fp8_block(self.w2[e], self.s2[e])
        elif self.fmt == "mxfp4":
            w13 = dequant_mxfp4(self.w13[e], self.s13[e])
            w2 = dequant_mxfp4(self.w2[e], self.s2[e])
        elif self.fmt == "nvfp4":
            w13 = dequant_nvfp4(self.w13[e], self.s13[e], self.gs13[e])
            w2 = dequant_nvfp4(self.w2[e], self.s2[e], self.gs2[e])
        else:
            raise ValueError(self.fmt)
        if self.interleaved:
            I = w13.shape[0] // 2
            b = w13.reshape(I // 128, 2, 128, -1)
            w13 = torch.cat([b[:, 0].reshape(I, -1), b[:, 1].reshape(I, -1)], dim=0)
        return w13, w2


@dataclass
class MoEWorkspace:
    """Static buffers for one MoE layer call of up to ``max_tokens`` tokens."""
    max_tokens: int
    top_k: int
    num_experts: int
    hidden: int
    inter: int
    device: torch.device
    bufs: dict = field(default_factory=dict)

    def __post_init__(self):
        n = self.max_tokens * self.top_k
        E, H, I, d = self.num_experts, self.hidden, self.inter, self.device
        self.counts = torch.zeros(E, dtype=torch.int32, device=d)
        self.seg = torch.zeros(E + 1, dtype=torch.int32, device=d)
        self.cursor = torch.zeros(E, dtype=torch.int32, device=d)
        self.perm_slot = torch.zeros(n, dtype=torch.int32, device=d)
        self.perm_w = torch.zeros(n, dtype=torch.float32, device=d)
        # pair rows, then (decode verification steps) the token rows of a fused shared expert
        self.xp = torch.empty(n + self.max_tokens, H, dtype=torch.bfloat16, device=d)
        # pair rows, then one row per token for a shared expert fused into the decode GEMV
        self.h = torch.empty(n + self.max_tokens, I, dtype=torch.bfloat16, device=d)
        self.h13 = None  # unfused gate/up output, allocated on demand
        self.slots = torch.empty(n + self.max_tokens, H, dtype=torch.bfloat16, device=d)
        self.mx = G.max_mtiles(n, E)
        self.tiles = torch.empty(self.mx * 4, dtype=torch.int32, device=d)
        self.active = torch.zeros(E + 1, dtype=torch.int32, device=d)   # decode GEMV: experts with rows
        self.tokrow = torch.zeros(min(E, n) * 16, dtype=torch.int32, device=d)   # decode: (expert, token) -> row
        self.route_logits = None                                                 # fused decode router scratch
        self.route_counter = torch.zeros(1, dtype=torch.int32, device=d)
        self.ntiles = torch.zeros(1, dtype=torch.int32, device=d)
        self.xq = self.xs = self.hq = self.hs = None                              # native fp8 path

    def fp8_buffers(self):
        """(x e4m3 [n, H], x scales [n, H/128], h e4m3 [n, I], h scales [n, I/128]) of the
        native fp8 expert GEMMs, allocated on first use."""
        if self.xq is None:
            n = self.max_tokens * self.top_k
            d = self.device
            self.xq = torch.empty(n, self.hidden, dtype=torch.float8_e4m3fn, device=d)
            self.xs = torch.empty(n, self.hidden // 128, dtype=torch.float32, device=d)
            self.hq = torch.empty(n, self.inter, dtype=torch.float8_e4m3fn, device=d)
            self.hs = torch.empty(n, self.inter // 128, dtype=torch.float32, device=d)
        return self.xq, self.xs, self.hq, self.hs

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in vars(self).values() if isinstance(t, torch.Tensor))


def moe_ref(x, ids, weights, experts: ExpertWeights, lo=0, hi=None, act_limit=0.0, act_alpha=1.0, act_beta=0.0):
    """fp32 reference: sum_k w_k * down(SwiGLU(gate_up(x))) over local pairs (bf16 intermediates)."""
    T, H = x.shape
    hi = experts.num_experts + lo if hi is None else hi
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for e in torch.unique(ids).tolist():
        if e < lo or e >= hi:
            continue
        w13, w2 = experts.dequant(e - lo)
        w13 = w13.to(torch.bfloat16).float()
        w2 = w2.to(torch.bfloat16).float()
        I = w13.shape[0] // 2
        tok, kk = (ids == e).nonzero(as_tuple=True)
        y = x[tok].float() @ w13.t()
        h = G.silu_and_mul_clamped(y[:, :I], y[:, I:], act_limit, act_alpha, act_beta).to(torch.bfloat16).float()
        o = (h @ w2.t()) * weights[tok, kk].float()[:, None]
        out.index_add_(0, tok, o.to(torch.bfloat16).float())
    return out


# rows per pass of the gathered grouped GEMV on verification steps (8 or 16): an expert
# rarely holds more than a few of a 20-row step's pairs, and 8-row activation boxes leave
# more of each CTA's ring to weights (GLM-4.5-Air, C = 4, MTP k = 4: decode step 21.31 ->
# 19.52 ms against 16-row passes); XTU_MOE_VERIFY_ROWS overrides
import os as _os
_VERIFY_PASS_ROWS = int(_os.environ.get("XTU_MOE_VERIFY_ROWS", "8"))
# steps of at most this many tokens take the token-direct form (every active expert
# multiplies all of the step's tokens); larger ones gather each expert's rows (C = 2,
# MTP k = 4, 10 rows: decode step 14.31 -> 13.33 ms against the token-direct form)
_DIRECT_MAX_ROWS = int(_os.environ.get("XTU_MOE_DIRECT_ROWS", "8"))


def moe_experts_partial(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, experts: ExpertWeights,
                        ws: MoEWorkspace, *, lo: int = 0, act_limit: float = 0.0, act_alpha: float = 1.0,
                        act_beta: float = 0.0, shared_mlp=None, permuted: bool = False) -> torch.Tensor | None:
    """Expert GEMMs for the pairs whose id is in [lo, lo + E): each such pair's weighted
    output row lands in ws.slots[pair].  Other pairs are untouched (other tiles / tiers).

    ``shared_mlp`` (a DenseMLP in the experts' layout): on the decode GEMV path it runs in
    the same launches as one more expert over every token, and its output rows are
    returned (ws.slots[T*K : T*K + T]); otherwise None is returned and the caller runs it.
    ``permuted``: :func:`route_decode` has already filled the decode permutation."""
    T, H = x.shape
    K = ids.shape[1]
    E = experts.num_experts
    if ws.num_experts < E or ws.max_tokens < T:
        raise ValueError(f"workspace for {ws.num_experts} experts x {ws.max_tokens} tokens; call needs {E} x {T}")
    s = N.stream_ptr(x.device)
    n = T * K
    fp8 = experts.fmt == "fp8"
    I = experts.inter
    # decode: weight-streaming grouped GEMV (gate/up + SwiGLU, down + weight + scatter); with
    # fp8 experts it reads the gathered rows as f16 x 2^-8, which the permute writes
    # up to GEMV_MAX_M_MOE rows (speculative verification batches) the grouped GEMV streams
    # each active expert's weights once per 16 of its rows; up to 16 rows in all it reads the
    # step's tokens directly (token-direct form), above that the permute gathers them
    gemv_path = (T <= G.GEMV_MAX_M_MOE and experts.interleaved and experts.fmt not in G.FP4_FMTS
                 and H % 128 == 0 and I % 128 == 0)   # whole 128-byte chunks per weight row
    if gemv_path and T <= min(G.GEMV_MAX_M, _DIRECT_MAX_ROWS) and E <= 1024:
        # one-CTA permute (no row gather): the gate/up GEMV reads the T tokens directly
        # and keeps each expert's own columns through ws.tokrow
        xt = G.tma_rows(x)
        x16 = getattr(x, "xtu_f16s", None)   # f16 x 2^-8 rows from the producing RMSNorm
        use16 = fp8 and x16 is not None and x16.shape == x.shape and x16.is_contiguous()
        if not permuted:
            N.call("xtu_moe_permute_decode", ids.data_ptr(), weights.data_ptr(), T, K, lo, lo + E, ws.seg.data_ptr(),
                   ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), ws.active.data_ptr(), ws.tokrow.data_ptr(), s)
        N.call("xtu_moe_gemv", experts.w13.data_ptr(), N.ptr(experts.s13 if fp8 else None),
               experts.w2.data_ptr(), N.ptr(experts.s2 if fp8 else None), int(fp8), E, H, I,
               x16.data_ptr() if use16 else xt.data_ptr(), int(use16), H if use16 else xt.stride(0),
               ws.tokrow.data_ptr(), T, ws.seg.data_ptr(), ws.perm_slot.data_ptr(),
               ws.perm_w.data_ptr(), ws.h.data_ptr(), ws.slots.data_ptr(), T, min(E, T * K), n,
               ws.active.data_ptr(), 1, float(act_limit), float(act_alpha), float(act_beta),
               *_shared_ptrs(shared_mlp), n, _gv_ws(x.device), N.status_buffer(x.device).data_ptr(), s)
        return ws.slots[n:n + T] if shared_mlp is not None else None
    if (T <= G.GEMV_MAX_M and experts.interleaved and experts.fmt in G.FP4_FMTS and H % 256 == 0 and I % 256 == 0
            and E <= 1024):
        # packed-4-bit experts at decode: the same token-direct grouped GEMV with e2m1 weights
        # decoded on chip (xtu_moe_gemv4)
        xt = G.tma_rows(x)
        if not permuted:
            N.call("xtu_moe_permute_decode", ids.data_ptr(), weights.data_ptr(), T, K, lo, lo + E, ws.seg.data_ptr(),
                   ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), ws.active.data_ptr(), ws.tokrow.data_ptr(), s)
        nv = experts.fmt == "nvfp4"
        N.call("xtu_moe_gemv4", experts.w13.data_ptr(), experts.s13.data_ptr(), N.ptr(experts.gs13 if nv else None),
               experts.w2.data_ptr(), experts.s2.data_ptr(), N.ptr(experts.gs2 if nv else None),
               G.FP4_FMTS[experts.fmt], E, H, I, xt.data_ptr(), xt.stride(0), ws.tokrow.data_ptr(), T,
               ws.seg.data_ptr(), ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), ws.h.data_ptr(), ws.slots.data_ptr(),
               T, min(E, T * K), n, ws.active.data_ptr(), 1, float(act_limit), float(act_alpha), float(act_beta),
               N.status_buffer(x.device).data_ptr(), s)
        return None
    if permuted:
        # a verification step of more tokens than the token-direct form takes: route_decode
        # has built the permutation; gather its rows (and the token rows of a fused shared
        # expert) and run the grouped GEMV on them
        if not gemv_path or T > G.DECODE_MAX_M:
            raise ValueError("a decode-permuted workspace needs the decode GEMV path")
        f16s = int(fp8)
        nsh = T if shared_mlp is not None else 0
        xt = G.tma_rows(x)
        N.call("xtu_moe_gather_rows", xt.data_ptr(), xt.stride(0), K, H, ws.perm_slot.data_ptr(),
               ws.seg[E:].data_ptr(), n, nsh, ws.xp.data_ptr(), f16s, s)
        N.call("xtu_moe_gemv", experts.w13.data_ptr(), N.ptr(experts.s13 if fp8 else None),
               experts.w2.data_ptr(), N.ptr(experts.s2 if fp8 else None), int(fp8), E, H, I, ws.xp.data_ptr(), f16s,
               H, None, T, ws.seg.data_ptr(), ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), ws.h.data_ptr(),
               ws.slots.data_ptr(), min(T, _VERIFY_PASS_ROWS), min(E, n), n, ws.active.data_ptr(), 1,
               float(act_limit), float(act_alpha), float(act_beta), *_shared_ptrs(shared_mlp), n,
               _gv_ws(x.device), N.status_buffer(x.device).data_ptr(), s)
        return ws.slots[n:n + T] if shared_mlp is not None else None
    f16s = int(gemv_path and fp8)
    N.call("xtu_moe_permute", ids.data_ptr(), weights.data_ptr(), T, K, lo, lo + E, ws.counts.data_ptr(),
           ws.seg.data_ptr(), ws.cursor.data_ptr(), ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), x.data_ptr(), H,
           x.stride(0), ws.xp.data_ptr(), f16s, s)
    if experts.fmt in G.FP4_FMTS:
        _experts_fp4(experts, ws, n, act_limit, act_alpha, act_beta)
        return None
    if gemv_path:
        N.call("xtu_moe_gemv", experts.w13.data_ptr(), N.ptr(experts.s13 if fp8 else None),
               experts.w2.data_ptr(), N.ptr(experts.s2 if fp8 else None), int(fp8), E, H, I, ws.xp.data_ptr(), f16s,
               H, None, 0, ws.seg.data_ptr(), ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), ws.h.data_ptr(),
               ws.slots.data_ptr(), min(T, G.GEMV_MAX_M), min(E, T * K), n, ws.active.data_ptr(), 0,
               float(act_limit), float(act_alpha),
               float(act_beta), None, None, None, None, 0, _gv_ws(x.device), N.status_buffer(x.device).data_ptr(), s)
        return None
    # the segment table of this call has E + 1 entries (the workspace may serve more experts)
    tiles = G.build_mtiles(ws.seg[: E + 1], n, ws.tiles, ws.ntiles)
    xp = ws.xp[:n]
    if fp8 and experts.interleaved and G.fp8_native_ok(n, 2 * I, H, swiglu=True) and I % 128 == 0:
        # native fp8 tensor cores: rows quantized per 128 columns, gate/up + SwiGLU written
        # straight back as e4m3 (+ scales), which the down GEMM reads as its A operand
        xq, xs, hq, hs = ws.fp8_buffers()
        G.quant_fp8_rows(xp, xq[:n], xs[:n])
        G.gemm_fp8_native(xq[:n], xs[:n], experts.w13, experts.s13, tiles=tiles, epilogue=G.EPI_SWIGLU_Q8,
                          out=hq[:n], out_scale=hs[:n], act_limit=act_limit, act_alpha=act_alpha, act_beta=act_beta)
        G.gemm_fp8_native(hq[:n], hs[:n], experts.w2, experts.s2, tiles=tiles, epilogue=G.EPI_BF16,
                          out=ws.slots, row_scale=ws.perm_w, row_dest=ws.perm_slot, out_rows=ws.slots.shape[0])
        return None
    sc13 = experts.s13 if fp8 else None
    sc2 = experts.s2 if fp8 else None
    if experts.interleaved:
        G.grouped_gemm(xp, experts.w13, ws.seg, w_scale=sc13, epilogue=G.EPI_SWIGLU, out=ws.h[:n],
                       act_limit=act_limit, act_alpha=act_alpha, act_beta=act_beta, tiles=tiles)
    else:
        if ws.h13 is None or ws.h13.shape[0] < n:
            ws.h13 = torch.empty(ws.max_tokens * K, 2 * I, dtype=torch.bfloat16, device=x.device)
        G.grouped_gemm(xp, experts.w13, ws.seg, w_scale=sc13, epilogue=G.EPI_BF16, out=ws.h13[:n], tiles=tiles)
        N.call("xtu_silu_mul", ws.h13.data_ptr(), n, I, float(act_limit), float(act_alpha), float(act_beta),
               ws.h.data_ptr(), s)
    G.grouped_gemm(ws.h[:n], experts.w2, ws.seg, w_scale=sc2, epilogue=G.EPI_BF16, out=ws.slots[:n],
                   row_scale=ws.perm_w, row_dest=ws.perm_slot, tiles=tiles)
    return None


def _experts_fp4(experts: ExpertWeights, ws: MoEWorkspace, n: int, act_limit, act_alpha, act_beta) -> None:
    """MXFP4 / NVFP4 experts (gate/up rows interleaved): grouped GEMMs with on-chip widening."""
    tiles = G.build_mtiles(ws.seg[: experts.num_experts + 1], n, ws.tiles, ws.ntiles)
    seg = ws.seg[: experts.num_experts + 1]
    G.grouped_gemm(ws.xp[:n], experts.w13, seg, w_scale=experts.s13, w_fmt=experts.fmt, w_gs=experts.gs13,
                   epilogue=G.EPI_SWIGLU, out=ws.h[:n], act_limit=act_limit, act_alpha=act_alpha,
                   act_beta=act_beta, tiles=tiles)
    G.grouped_gemm(ws.h[:n], experts.w2, seg, w_scale=experts.s2, w_fmt=experts.fmt, w_gs=experts.gs2,
                   epilogue=G.EPI_BF16, out=ws.slots[:n], row_scale=ws.perm_w, row_dest=ws.perm_slot, tiles=tiles)


def moe_combine(ws: MoEWorkspace, ids: torch.Tensor, lo: int, hi: int, *, shared: torch.Tensor | None = None,
                extra: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum of the slot rows of t's pairs with id in [lo, hi) (+ shared + extra fp32)."""
    T, K = ids.shape
    H = ws.hidden
    y = out if out is not None else torch.empty(T, H, dtype=torch.bfloat16, device=ids.device)
    N.call("xtu_moe_combine", ws.slots.data_ptr(), ids.data_ptr(), T, K, H, lo, hi, N.ptr(shared), N.ptr(extra),
           y.data_ptr(), None, N.stream_ptr(ids.device))
    return y


def fused_moe(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, experts: ExpertWeights,
              ws: MoEWorkspace | None = None, *, lo: int = 0, shared: torch.Tensor | None = None,
              extra: torch.Tensor | None = None, act_limit: float = 0.0, act_alpha: float = 1.0,
              act_beta: float = 0.0, out: torch.Tensor | None = None, shared_mlp=None,
              permuted: bool = False) -> torch.Tensor:
    """Routed-expert MoE over the local experts [lo, lo+E).

    x [T, H] bf16, ids/weights [T, K]; shared [T, H] (shared-expert output) and
    extra [T, H] fp32 (e.g. the CPU tier's partial) are added in the combine.
    """
    T, H = x.shape
    K = ids.shape[1]
    E = experts.num_experts
    if not x.is_cuda:
        o = moe_ref(x, ids, weights, experts, lo, lo + E, act_limit, act_alpha, act_beta)
        if shared is not None:
            o = o + shared.float()
        if extra is not None:
            o = o + extra.float()
        return o.to(x.dtype) if out is None else out.copy_(o)
    if experts.fmt in G.FP4_FMTS and not experts.interleaved:
        raise NotImplementedError(f"GPU {experts.fmt} experts need I % 128 == 0 (gate/up interleave)")
    if ws is None or ws.max_tokens < T:
        ws = MoEWorkspace(T, K, E, H, experts.inter, x.device)
    assert x.is_contiguous() and ids.is_contiguous() and weights.is_contiguous()
    fused_sh = moe_experts_partial(x, ids, weights, experts, ws, lo=lo, act_limit=act_limit, act_alpha=act_alpha,
                                   act_beta=act_beta, shared_mlp=shared_mlp, permuted=permuted)
    if shared_mlp is not None and fused_sh is None:   # not the decode GEMV path: run it on its own
        fused_sh = shared_mlp(x)
    if fused_sh is not None:
        shared = fused_sh if shared is None else shared + fused_sh
    return moe_combine(ws, ids, lo, lo + E, shared=shared, extra=extra, out=out)


def route_split(ids: torch.Tensor, slotmap: torch.Tensor, lo: int, gpu_ids: torch.Tensor, cpu_ids: torch.Tensor,
                hits: torch.Tensor | None = None) -> None:
    """Pairs -> pool slot id (or -1) and CPU expert id (or -1); counts hits per expert."""
    n = ids.numel()
    N.call("xtu_route_split", ids.data_ptr(), n, lo, slotmap.numel(), slotmap.data_ptr(), gpu_ids.data_ptr(),
           cpu_ids.data_ptr(), N.ptr(hits), N.stream_ptr(ids.device))


def decode_route_ok(x: torch.Tensor, gate: torch.Tensor, experts: ExpertWeights | None, top_k: int,
                    n_group: int) -> bool:
    """Whether :func:`route_decode` (router + permute in one launch) serves this step."""
    if experts is None or not x.is_cuda or x.shape[0] > G.DECODE_MAX_M or x.dtype != torch.bfloat16:
        return False
    H = x.shape[1]
    return (gate.dtype == torch.bfloat16 and gate.is_contiguous() and gate.shape[0] <= 1024 and H % 128 == 0
            and experts.num_experts <= 1024 and experts.interleaved and experts.fmt in ("fp8", "bf16")
            and experts.inter % 128 == 0 and top_k <= 32 and n_group <= 64)


def route_decode(x: torch.Tensor, gate: torch.Tensor, bias: torch.Tensor | None, top_k: int, scoring: str,
                 n_group: int, topk_group: int, renorm: bool, scale: float, ws: MoEWorkspace, lo: int,
                 num_local: int):
    """Decode router and permute in one launch: logits = x gate^T (fp32), scoring + bias +
    grouped top-k + renorm + scale per token, then the decode permutation of the pairs whose
    expert is in [lo, lo + num_local) into ``ws``.  Returns (ids int32 [T, K], weights fp32)."""
    from .router import SCORING
    T, H = x.shape
    E = gate.shape[0]
    xt = G.tma_rows(x)
    if ws.route_logits is None or ws.route_logits.numel() < G.DECODE_MAX_M * E:
        ws.route_logits = torch.empty(G.DECODE_MAX_M * E, dtype=torch.float32, device=x.device)
    ids = torch.empty(T, top_k, dtype=torch.int32, device=x.device)
    w = torch.empty(T, top_k, dtype=torch.float32, device=x.device)
    N.call("xtu_moe_route_decode", xt.data_ptr(), xt.stride(0), T, gate.data_ptr(), E, H, N.ptr(bias), top_k,
           SCORING[scoring], n_group, topk_group, int(renorm), float(scale), ws.route_logits.data_ptr(),
           ws.route_counter.data_ptr(), ids.data_ptr(), w.data_ptr(), lo, lo + num_local, ws.seg.data_ptr(),
           ws.perm_slot.data_ptr(), ws.perm_w.data_ptr(), ws.active.data_ptr(),
           ws.tokrow.data_ptr() if T <= G.GEMV_MAX_M else None, N.stream_ptr(x.device))
    return ids, w


def shared_fusable(shared_mlp, experts: ExpertWeights, act_limit: float = 0.0, act_alpha: float = 1.0,
                   act_beta: float = 0.0) -> bool:
    """Whether a DenseMLP shared expert can ride in the routed decode GEMV launches: same
    weight format, width and activation as the experts, gate/up interleaved in 128-row blocks."""
    if act_alpha != 1.0 or act_beta != 0.0 or getattr(shared_mlp, "limit", None) != act_limit:
        return False
    if shared_mlp is None or experts is None or not getattr(shared_mlp, "interleaved", False):
        return False
    fp8 = experts.fmt == "fp8"
    if experts.fmt not in ("fp8", "bf16") or (shared_mlp.gate_up.scale is not None) != fp8:
        return False
    return (shared_mlp.gate_up.weight.dtype == experts.w13.dtype and shared_mlp.down.weight.shape[1] == experts.inter
            and shared_mlp.gate_up.weight.shape[0] == 2 * experts.inter)


def _shared_ptrs(shared_mlp):
    if shared_mlp is None:
        return None, None, None, None
    return (shared_mlp.gate_up.weight.data_ptr(), N.ptr(shared_mlp.gate_up.scale), shared_mlp.down.weight.data_ptr(),
            N.ptr(shared_mlp.down.scale))


def _gv_ws(device):
    return G._gemv_split_ws(device)[0].data_ptr()


def dense_swiglu_gemv(x: torch.Tensor, w13: torch.Tensor, s13, w2: torch.Tensor, s2, limit: float,
                      cache: dict) -> torch.Tensor:
    """Decode-size SwiGLU MLP (gate/up interleaved in 128-row blocks) as a one-expert grouped GEMV."""
    x16 = getattr(x, "xtu_f16s", None)
    x = G.tma_rows(x)
    if x16 is not None:
        x.xtu_f16s = x16
    T, H = x.shape
    I = w13.shape[0] // 2
    key = ("gemv", x.device, T, I)
    st = cache.get(key)
    if st is None:
        d = x.device
        st = dict(seg=torch.tensor([0, T], dtype=torch.int32, device=d),
                  slot=torch.arange(T, dtype=torch.int32, device=d),
                  w=torch.ones(T, dtype=torch.float32, device=d),
                  h=torch.empty(T, I, dtype=torch.bfloat16, device=d),
                  active=torch.tensor([1, 0], dtype=torch.int32, device=d))   # one expert, always active
        cache[key] = st
    y = torch.empty(T, w2.shape[0], dtype=torch.bfloat16, device=x.device)
    x16 = getattr(x, "xtu_f16s", None)   # f16 x 2^-8 rows from the producing RMSNorm
    use16 = s13 is not None and x16 is not None and x16.shape == x.shape and x16.is_contiguous()
    N.call("xtu_moe_gemv", w13.data_ptr(), N.ptr(s13), w2.data_ptr(), N.ptr(s2), int(s13 is not None), 1, H, I,
           x16.data_ptr() if use16 else x.data_ptr(), int(use16), H if use16 else x.stride(0), None, 0,
           st["seg"].data_ptr(), st["slot"].data_ptr(), st["w"].data_ptr(), st["h"].data_ptr(),
           y.data_ptr(), min(T, G.GEMV_MAX_M), 1, T, st["active"].data_ptr(), 1, float(limit), 1.0, 0.0, None, None,
           None, None, 0,
           _gv_ws(x.device),
           N.status_buffer(x.device).data_ptr(), N.stream_ptr(x.device))
    return y


def prepare_experts(fmt: str, w13: torch.Tensor, w2: torch.Tensor, s13=None, s2=None, gs13=None,
                    gs2=None) -> ExpertWeights:
    """Checkpoint layout (w13 [E, 2I, H] gate-then-up) -> kernel layout.

    Interleaves gate/up rows in 128-row blocks when I % 128 == 0 (fused SwiGLU).  "int4"
    (GPTQ rows kept at 4 bits for the CPU tier) is dequantized to bf16 for the GPU kernels.
    """
    if fmt == "int4":
        from .quant import dequant_int4_rows
        dq = lambda w, sz: torch.stack([dequant_int4_rows(w[e], sz[e]) for e in range(w.shape[0])]).to(torch.bfloat16)
        return prepare_experts("bf16", dq(w13, s13), dq(w2, s2))
    I = w13.shape[1] // 2
    inter = I % 128 == 0
    if inter:
        if fmt == "fp8":
            w13 = G.interleave_gate_up(w13.view(torch.uint8)).view(torch.float8_e4m3fn)
            s13 = G.interleave_gate_up_scale(s13)
        elif fmt in ("mxfp4", "nvfp4"):   # per-row scales follow their rows
            w13 = G.interleave_gate_up(w13)
            sdt = s13.dtype
            s13 = G.interleave_gate_up(s13.view(torch.uint8)).view(sdt)
        else:
            w13 = G.interleave_gate_up(w13)
    return ExpertWeights(fmt, w13.contiguous(), w2.contiguous(), s13, s2, inter, gs13, gs2)
