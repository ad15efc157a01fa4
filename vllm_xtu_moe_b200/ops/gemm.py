"""Tensor-core GEMMs (tcgen05, sm_100a): dense and grouped per-expert.

``linear(x, w)`` computes ``x @ w.T`` for bf16 weights or for e4m3 weights with
128x128 fp32 block scales (the HF ``weight`` + ``weight_scale_inv`` pair).  On a
GPU the hand-written kernels in ``csrc/cuda/gemm_tc.cu`` run; on a CPU the
PyTorch restatement below runs (it is also the numerics oracle of the tests).
"""
from __future__ import annotations

import torch

from . import _native as N
from .quant import dequant_fp8_block

MTILE_BYTES = 16
BM = 128


def _on_gpu(t: torch.Tensor) -> bool:
    return t.is_cuda


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16, row_scale: torch.Tensor | None = None) -> torch.Tensor:
    """out[M,N] = a[M,K] @ b[N,K]^T (bf16 in, fp32 accumulate)."""
    M, K = a.shape
    Nn = b.shape[0]
    if not _on_gpu(a):
        r = a.float() @ b.float().t()
        if row_scale is not None:
            r = r * row_scale.float()[:, None]
        return r.to(out_dtype) if out is None else out.copy_(r)
    assert a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and b.shape[1] == K
    assert a.is_contiguous() and b.is_contiguous() and K % 8 == 0
    if out is None:
        out = torch.empty(M, Nn, dtype=out_dtype, device=a.device)
    assert out.stride(1) == 1
    N.call("xtu_gemm_bf16", a.data_ptr(), b.data_ptr(), out.data_ptr(), M, Nn, K, out.stride(0),
           int(out.dtype == torch.float32), N.ptr(row_scale), N.status_buffer(a.device).data_ptr(),
           N.stream_ptr(a.device))
    return out


def gemm_fp8w(a: torch.Tensor, w8: torch.Tensor, w_scale: torch.Tensor, out: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """out = a @ dequant(w8, w_scale)^T with e4m3 w8 [N,K] and fp32 scales [ceil(N/128), ceil(K/128)]."""
    M, K = a.shape
    Nn = w8.shape[0]
    if not _on_gpu(a):
        w = dequant_fp8_block(w8, w_scale).to(torch.bfloat16)
        r = a.float() @ w.float().t()
        return r.to(out_dtype) if out is None else out.copy_(r)
    assert a.dtype == torch.bfloat16 and a.is_contiguous() and w8.is_contiguous() and K % 16 == 0
    if out is None:
        out = torch.empty(M, Nn, dtype=out_dtype, device=a.device)
    N.call("xtu_gemm_fp8w", a.data_ptr(), w8.data_ptr(), w_scale.data_ptr(), out.data_ptr(), M, Nn, K,
           out.stride(0), int(out.dtype == torch.float32), N.status_buffer(a.device).data_ptr(),
           N.stream_ptr(a.device))
    return out


GEMV_MAX_M = 16          # rows of the token-direct decode forms (MoE, fused TP, norms' f16 copies)
GEMV_MAX_M_DENSE = 32    # rows a plain dense GEMV call takes (speculative verification batches)
GEMV_MAX_M_MOE = 64      # rows the gathered grouped MoE GEMV takes (<= 16 per expert per pass)
DECODE_MAX_M = 32        # rows of a decode / verification step the decode forms serve (RMSNorm f16
                         # copies, fused router + permute, shared expert inside the routed GEMVs)


def gemv(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor | None = None, bias: torch.Tensor | None = None,
         out_dtype: torch.dtype = torch.bfloat16, out: torch.Tensor | None = None,
         x16: torch.Tensor | None = None) -> torch.Tensor:
    """Decode-size y[M<=32, N] = x W^T (+ bias) streaming W (bf16 or e4m3 + block scales).
    ``x16``: the same rows already as f16 x 2^-8 (fp8 weights then skip their conversion)."""
    x = tma_rows(x)
    M, K = x.shape
    flags = int(scale is not None)
    xp, xs = x.data_ptr(), x.stride(0)
    if x16 is not None and scale is not None and x16.shape == (M, K) and x16.is_contiguous():
        flags |= 4
        xp, xs = x16.data_ptr(), K
    Nn = weight.shape[0]
    y = out if out is not None else torch.empty(M, Nn, dtype=out_dtype, device=x.device)
    ws, cnt = _gemv_split_ws(x.device)
    N.call("xtu_gemv", weight.data_ptr(), N.ptr(scale), flags, Nn, K, xp, xs, M,
           N.ptr(bias), y.data_ptr(), y.stride(0), int(y.dtype == torch.float32), ws.data_ptr(), cnt.data_ptr(),
           N.status_buffer(x.device).data_ptr(), N.stream_ptr(x.device))
    return y


def tma_rows(x: torch.Tensor) -> torch.Tensor:
    """x itself when its rows can be read by TMA (unit inner stride, 16-byte aligned base and
    row pitch), else a packed copy."""
    if x.stride(-1) == 1 and x.data_ptr() % 16 == 0 and (x.stride(0) * x.element_size()) % 16 == 0:
        return x
    return x.clone(memory_format=torch.contiguous_format)


_GEMV_WS: dict = {}


def _gemv_split_ws(device):
    """Per-device scratch of the decode GEMVs: 4 MB of fp32 split-K partials (dense calls
    whose tiles do not fill the GPU) followed by 1 MB for the f16 activations of fp8-weight
    calls, and per-tile completion counters that start zeroed and that every launch leaves
    zeroed.  Allocated once, so captured graphs keep valid pointers; launches on one stream
    share it."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _GEMV_WS.get(key)
    if t is None:
        t = (torch.empty((1 << 20) + (1 << 18), dtype=torch.float32, device=device),
             torch.zeros(1024, dtype=torch.int32, device=device))
        _GEMV_WS[key] = t
    return t


def gemv_ws_reset(device) -> None:
    """Re-zero the GEMV tile counters (after a launch that reported an error, whose CTAs
    may have stopped between bumping a counter and clearing it)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _GEMV_WS.get(key)
    if t is not None:
        t[1].zero_()


def linear(x: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor | None = None,
           out_dtype: torch.dtype = torch.bfloat16, bias: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ W^T (+ bias) for 2-D or batched x; W bf16 or e4m3 (+ block scales).

    GPU dispatch: <= 16 rows -> weight-streaming GEMV (bias fused); more rows ->
    tcgen05 GEMM."""
    shp = x.shape
    x16 = getattr(x, "xtu_f16s", None)   # f16 x 2^-8 copy written by the producing RMSNorm
    x2 = x.reshape(-1, shp[-1])
    if x2.shape[0] == 0:
        return x.new_empty(*shp[:-1], weight.shape[0], dtype=out_dtype)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    K = x2.shape[1]
    if x2.is_cuda and x2.shape[0] <= GEMV_MAX_M_DENSE and K % 64 == 0 and x2.dtype == torch.bfloat16:
        y = gemv(x2, weight, scale, bias, out_dtype, x16=x16)
        return y.reshape(*shp[:-1], weight.shape[0])
    if scale is None:
        y = gemm_bf16(x2, weight, out_dtype=out_dtype)
    elif (x2.is_cuda and x2.dtype == torch.bfloat16 and fp8_native_ok(x2.shape[0], weight.shape[0], K)
          and out_dtype in (torch.bfloat16, torch.float32)):
        xq, xs = quant_fp8_rows(x2)
        y = gemm_fp8_native(xq, xs, weight, scale, epilogue=EPI_F32 if out_dtype == torch.float32 else EPI_BF16,
                            bias=bias if bias is not None and bias.dtype == torch.bfloat16 else None)
        if bias is not None and bias.dtype != torch.bfloat16:
            y.add_(bias)
        return y.reshape(*shp[:-1], weight.shape[0])
    else:
        y = gemm_fp8w(x2, weight, scale, out_dtype=out_dtype)
    if bias is not None:
        y.add_(bias)
    return y.reshape(*shp[:-1], weight.shape[0])


# ---------------------------------------------------------------------------
# native fp8 (kind::f8f6f4): activations quantized per (row, 128 columns)
# ---------------------------------------------------------------------------
import os as _os

# XTU_FP8_MMA=1 ("W8A8" mode): fp8-weight GEMMs of more than GEMV_MAX_M rows quantize their
# activations to e4m3 per (row, 128 columns) and run on the kind::f8f6f4 tensor cores.  Off by
# default: quantizing activations moves an MoE layer's output by ~4% (relative, measured on
# GLM-4.5-Air shapes) from the bf16-activation result, so the default keeps bf16 activations
# (weights widened to bf16 on chip) and the numerics of a bf16 compute path.
FP8_MMA = _os.environ.get("XTU_FP8_MMA", "0") == "1"
EPI_SWIGLU_Q8 = 3


def quant_fp8_rows(x: torch.Tensor, out: torch.Tensor | None = None, scale: torch.Tensor | None = None):
    """bf16 [M, K] -> (e4m3 [M, K], fp32 scales [M, K/128]): per (row, 128-column block)
    scale = amax / 448, value = x / scale rounded to nearest e4m3 (saturating)."""
    M, K = x.shape
    assert K % 128 == 0
    if out is None:
        out = torch.empty(M, K, dtype=torch.float8_e4m3fn, device=x.device)
    if scale is None:
        scale = torch.empty(M, K // 128, dtype=torch.float32, device=x.device)
    if not x.is_cuda:
        xb = x.float().view(M, K // 128, 128)
        am = xb.abs().amax(-1)
        sc = torch.where(am > 0, am / 448.0, torch.ones_like(am))
        inv = torch.where(am > 0, 448.0 / am, torch.zeros_like(am))
        q = (xb * inv[..., None]).clamp(-448, 448).to(torch.float8_e4m3fn).view(M, K)
        out.copy_(q)
        scale.copy_(sc)
        return out, scale
    assert x.dtype == torch.bfloat16 and x.stride(1) == 1 and x.stride(0) % 4 == 0
    N.call("xtu_quant_fp8_rows", x.data_ptr(), M, K, x.stride(0), out.data_ptr(), scale.data_ptr(),
           N.stream_ptr(x.device))
    return out, scale


def dequant_fp8_rows(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    M, K = q.shape
    return (q.float().view(M, K // 128, 128) * scale.float()[..., None]).view(M, K)


def fp8_native_ok(M: int, N_out: int, K: int, swiglu: bool = False) -> bool:
    return FP8_MMA and M > GEMV_MAX_M and K % 128 == 0 and (N_out % 256 == 0 if swiglu else N_out % 16 == 0)


def linear_takes_gemv(M: int) -> bool:
    """Whether G.linear serves an M-row call with the weight-streaming GEMV."""
    return M <= GEMV_MAX_M_DENSE


def gemm_fp8_native(aq: torch.Tensor, a_scale: torch.Tensor, w8: torch.Tensor, w_scale: torch.Tensor, *,
                    seg: torch.Tensor | None = None, tiles=None, epilogue: int = 0,
                    out: torch.Tensor | None = None, out_scale: torch.Tensor | None = None,
                    row_scale: torch.Tensor | None = None, row_dest: torch.Tensor | None = None,
                    out_rows: int | None = None, bias: torch.Tensor | None = None, act_limit: float = 0.0,
                    act_alpha: float = 1.0, act_beta: float = 0.0, peer_out=None, peer_rows: int = 0):
    """e4m3 activations (+ per-(row, 128) scales) x e4m3 weights (+ 128x128 block scales) on
    the kind::f8f6f4 tensor cores.  ``w8`` [N, K] (dense) or [E, N, K] with ``seg`` (grouped);
    epilogues as :func:`grouped_gemm`, plus EPI_SWIGLU_Q8: SwiGLU quantized to e4m3 into
    ``out`` [*, N/2] with scales ``out_scale`` [*, N/256]."""
    M, K = aq.shape
    grouped = w8.dim() == 3
    E, Nn = (w8.shape[0], w8.shape[1]) if grouped else (1, w8.shape[0])
    assert w8.shape[-1] == K and K % 128 == 0 and aq.is_cuda and aq.is_contiguous() and w8.is_contiguous()
    swi = epilogue in (EPI_SWIGLU, EPI_SWIGLU_Q8)
    out_cols = Nn // 2 if swi else Nn
    rows = out_rows if out_rows is not None else M
    if out is None:
        dt = {EPI_F32: torch.float32, EPI_SWIGLU_Q8: torch.float8_e4m3fn}.get(epilogue, torch.bfloat16)
        out = torch.empty(rows, out_cols, dtype=dt, device=aq.device)
    if epilogue == EPI_SWIGLU_Q8 and out_scale is None:
        out_scale = torch.empty(rows, Nn // 256, dtype=torch.float32, device=aq.device)
    if M == 0:
        return (out, out_scale) if epilogue == EPI_SWIGLU_Q8 else out
    t = cnt = None
    mx = 0
    if grouped:
        if tiles is None:
            tiles = build_mtiles(seg, M)
        t, cnt, mx = tiles
    N.call("xtu_gemm_fp8_native", aq.data_ptr(), a_scale.data_ptr(), w8.data_ptr(), w_scale.data_ptr(),
           out.data_ptr(), out.stride(0), N.ptr(out_scale), out_scale.stride(0) if out_scale is not None else 0,
           M, Nn, K, E, N.ptr(t), N.ptr(cnt), mx, epilogue, N.ptr(row_scale), N.ptr(row_dest), N.ptr(bias),
           float(act_limit), float(act_alpha), float(act_beta), peer_out, int(peer_rows),
           N.status_buffer(aq.device).data_ptr(), N.stream_ptr(aq.device))
    return (out, out_scale) if epilogue == EPI_SWIGLU_Q8 else out


# ---------------------------------------------------------------------------
# grouped (MoE) GEMM
# ---------------------------------------------------------------------------
def max_mtiles(num_rows: int, num_experts: int) -> int:
    return (num_rows + BM - 1) // BM + num_experts


def build_mtiles(seg: torch.Tensor, num_rows: int, tiles: torch.Tensor | None = None,
                 count: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor, int]:
    """Device list of 128-row tiles per expert segment (seg: int32 [E+1])."""
    E = seg.numel() - 1
    mx = max_mtiles(num_rows, E)
    if tiles is None:
        tiles = torch.empty(mx * 4, dtype=torch.int32, device=seg.device)
    if count is None:
        count = torch.empty(1, dtype=torch.int32, device=seg.device)
    N.call("xtu_build_mtiles", seg.data_ptr(), E, tiles.data_ptr(), count.data_ptr(), mx, N.stream_ptr(seg.device))
    return tiles, count, mx


EPI_BF16, EPI_F32, EPI_SWIGLU = 0, 1, 2


FP4_FMTS = {"mxfp4": 2, "nvfp4": 3}


def grouped_gemm(a: torch.Tensor, w: torch.Tensor, seg: torch.Tensor, *, w_scale: torch.Tensor | None = None,
                 epilogue: int = EPI_BF16, out: torch.Tensor | None = None, row_scale: torch.Tensor | None = None,
                 row_dest: torch.Tensor | None = None, out_rows: int | None = None,
                 act_limit: float = 0.0, act_alpha: float = 1.0, act_beta: float = 0.0,
                 tiles: tuple[torch.Tensor, torch.Tensor, int] | None = None, w_fmt: str | None = None,
                 w_gs: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped GEMM: rows a[seg[e]:seg[e+1]] are multiplied by w[e]^T.

    w is [E, N, K] bf16, or e4m3 with w_scale [E, ceil(N/128), ceil(K/128)].
    epilogue EPI_SWIGLU expects w rows arranged in 256-row blocks of
    (128 gate rows, 128 up rows) (see :func:`interleave_gate_up`) and writes
    [rows, N/2] bf16.  row_scale multiplies each output row; row_dest scatters
    row m to out[row_dest[m]] (rows with row_dest < 0 are dropped).
    """
    M, K = a.shape
    E, Nn, Kw = w.shape
    if w_fmt in FP4_FMTS:
        return _grouped_gemm_fp4(a, w, seg, w_scale, w_gs, FP4_FMTS[w_fmt], epilogue, out, row_scale, row_dest,
                                 out_rows, act_limit, act_alpha, act_beta, tiles)
    assert Kw == K
    out_cols = Nn // 2 if epilogue == EPI_SWIGLU else Nn
    rows = out_rows if out_rows is not None else M
    if out is None:
        dt = torch.float32 if epilogue == EPI_F32 else torch.bfloat16
        out = torch.zeros(rows, out_cols, dtype=dt, device=a.device)
    if M == 0:
        return out
    if not _on_gpu(a):
        return _grouped_gemm_torch(a, w, seg, w_scale, epilogue, out, row_scale, row_dest, act_limit,
                                   act_alpha, act_beta)
    assert a.dtype == torch.bfloat16 and a.is_contiguous() and w.is_contiguous()
    assert seg.dtype == torch.int32 and seg.is_cuda
    if tiles is None:
        tiles = build_mtiles(seg, M)
    t, cnt, mx = tiles
    bfmt = 1 if w_scale is not None else 0
    if bfmt:
        assert w.dtype in (torch.float8_e4m3fn, torch.uint8)
    else:
        assert w.dtype == torch.bfloat16
    N.call("xtu_grouped_gemm", a.data_ptr(), w.data_ptr(), N.ptr(w_scale), bfmt, out.data_ptr(), out.stride(0),
           M, Nn, K, E, t.data_ptr(), cnt.data_ptr(), mx, epilogue, N.ptr(row_scale), N.ptr(row_dest),
           float(act_limit), float(act_alpha), float(act_beta), N.status_buffer(a.device).data_ptr(),
           N.stream_ptr(a.device))
    return out


def silu_and_mul_clamped(g: torch.Tensor, u: torch.Tensor, limit: float = 0.0, alpha: float = 1.0,
                         beta: float = 0.0) -> torch.Tensor:
    """Clamped gated SiLU: clamp(g, max=limit) * sigmoid(alpha*g') * (clamp(u, +-limit) + beta)."""
    g = g.float()
    u = u.float()
    if limit > 0:
        g = g.clamp(max=limit)
        u = u.clamp(-limit, limit)
    return g * torch.sigmoid(alpha * g) * (u + beta)


def interleave_gate_up(w13: torch.Tensor, block: int = 128) -> torch.Tensor:
    """[.., 2I, K] (gate rows then up rows) -> rows in (gate block, up block) pairs of `block` rows."""
    *lead, two_i, K = w13.shape
    I = two_i // 2
    assert I % block == 0
    g = w13[..., :I, :].reshape(*lead, I // block, block, K)
    u = w13[..., I:, :].reshape(*lead, I // block, block, K)
    return torch.stack([g, u], dim=-3).reshape(*lead, two_i, K).contiguous()


def interleave_gate_up_scale(s13: torch.Tensor) -> torch.Tensor:
    """Matching reorder of [.., 2I/128, K/128] block scales (one scale row per 128 rows)."""
    *lead, nb, kb = s13.shape
    h = nb // 2
    g = s13[..., :h, :]
    u = s13[..., h:, :]
    return torch.stack([g, u], dim=-2).reshape(*lead, nb, kb).contiguous()


def _grouped_gemm_torch(a, w, seg, w_scale, epilogue, out, row_scale, row_dest, limit, alpha, beta):
    segl = seg.tolist()
    for e in range(w.shape[0]):
        s0, s1 = segl[e], segl[e + 1]
        if s1 <= s0:
            continue
        we = w[e]
        if w_scale is not None:
            we = dequant_fp8_block(we, w_scale[e]).to(torch.bfloat16)
        y = a[s0:s1].float() @ we.float().t()
        if epilogue == EPI_SWIGLU:
            n = y.shape[1]
            yb = y.reshape(y.shape[0], n // 256, 2, 128)
            y = silu_and_mul_clamped(yb[:, :, 0], yb[:, :, 1], limit, alpha, beta).reshape(y.shape[0], n // 2)
        if row_scale is not None:
            y = y * row_scale[s0:s1].float()[:, None]
        if row_dest is not None:
            d = row_dest[s0:s1].long()
            keep = d >= 0
            out[d[keep]] = y[keep].to(out.dtype)
        else:
            out[s0:s1] = y.to(out.dtype)
    return out


def _grouped_gemm_fp4(a, w, seg, w_scale, w_gs, bfmt, epilogue, out, row_scale, row_dest, out_rows, act_limit,
                      act_alpha, act_beta, tiles):
    """MXFP4 / NVFP4 expert weights: w [E, N, K/2] bytes + per-row scales, widened on chip."""
    M, K = a.shape
    E, Nn, Kh = w.shape
    assert Kh * 2 == K and w.dtype == torch.uint8 and w_scale is not None
    out_cols = Nn // 2 if epilogue == EPI_SWIGLU else Nn
    rows = out_rows if out_rows is not None else M
    if out is None:
        dt = torch.float32 if epilogue == EPI_F32 else torch.bfloat16
        out = torch.zeros(rows, out_cols, dtype=dt, device=a.device)
    if M == 0:
        return out
    assert a.is_cuda and a.dtype == torch.bfloat16 and a.is_contiguous() and w.is_contiguous()
    if tiles is None:
        tiles = build_mtiles(seg, M)
    t, cnt, mx = tiles
    gs = None
    if bfmt == 3:
        gs = w_gs.float().contiguous()
    N.call("xtu_grouped_gemm_ex", a.data_ptr(), w.data_ptr(), w_scale.contiguous().data_ptr(), N.ptr(gs), bfmt,
           out.data_ptr(), out.stride(0), M, Nn, K, E, t.data_ptr(), cnt.data_ptr(), mx, epilogue, N.ptr(row_scale),
           N.ptr(row_dest), float(act_limit), float(act_alpha), float(act_beta), None, 0,
           N.status_buffer(a.device).data_ptr(), N.stream_ptr(a.device))
    return out
