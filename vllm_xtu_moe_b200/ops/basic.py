"""Norm / RoPE / KV-cache write / embedding / sampling ops.

Each op runs the sm_100a kernel from ``csrc/cuda/elementwise.cu`` when its
inputs live on a GPU and the PyTorch restatement (``*_ref``) otherwise.  The
restatements are the numerics oracle of ``tests/test_ops.py``.
"""
from __future__ import annotations

import math

import torch

from . import _native as N


# ---------------------------------------------------------------------------
# RMSNorm (+ residual)
# ---------------------------------------------------------------------------
def rmsnorm_ref(x, w, eps, residual=None, add_one=False):
    if residual is not None:
        r = (x.float() + residual.float()).to(x.dtype)
    else:
        r = x
    rf = r.float()
    y = rf * torch.rsqrt(rf.pow(2).mean(-1, keepdim=True) + eps)
    ww = w.float() + (1.0 if add_one else 0.0)
    return (y * ww).to(x.dtype), r


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, residual: torch.Tensor | None = None,
            add_one: bool = False, out: torch.Tensor | None = None, f16s: bool = False):
    """y = RMSNorm(x [+ residual]) * w.  With a residual, returns (y, x + residual).

    ``f16s``: also produce y as f16 x 2^-8 (the input form of the fp8-weight decode GEMVs),
    attached to the returned y as ``y.xtu_f16s`` so those GEMVs skip their conversion."""
    if not x.is_cuda:
        y, r = rmsnorm_ref(x, w, eps, residual, add_one)
        return (y, r) if residual is not None else y
    H = x.shape[-1]
    x2 = x.reshape(-1, H)
    T = x2.shape[0]
    assert x2.stride(-1) == 1 and w.is_contiguous()
    y = out if out is not None else torch.empty(T, H, dtype=x.dtype, device=x.device)
    r_out = None
    if residual is not None:
        residual = residual.reshape(-1, H)
        assert residual.is_contiguous()
        r_out = torch.empty_like(residual)
    y16 = torch.empty(T, H, dtype=torch.float16, device=x.device) if f16s and H % 8 == 0 else None
    N.call("xtu_rmsnorm", x2.data_ptr(), N.ptr(residual), N.ptr(r_out), w.data_ptr(), y.data_ptr(), T, H,
           float(eps), int(add_one), x2.stride(0), y.stride(0), N.ptr(y16), N.stream_ptr(x.device))
    y = y.reshape(x.shape)
    if y16 is not None and y.dim() == 2 and y.stride(0) == H:
        y.xtu_f16s = y16
    if residual is not None:
        return y, r_out.reshape(x.shape)
    return y


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------
def rope_cache(rot_dim: int, max_pos: int, theta: float, device=None, scaling: dict | None = None) -> torch.Tensor:
    """[max_pos, rot_dim] fp32: cos in the first half, sin in the second.

    ``scaling`` supports {"type": "yarn", "factor", "original_max_position_embeddings",
    "beta_fast", "beta_slow", "mscale", "mscale_all_dim"} (DeepSeek-V3) and
    {"type": "linear", "factor"}.
    """
    inv = 1.0 / (theta ** (torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim))
    mscale = 1.0
    if scaling and scaling.get("type", scaling.get("rope_type")) == "yarn":
        f = float(scaling["factor"])
        orig = int(scaling.get("original_max_position_embeddings", 4096))
        bf, bs = float(scaling.get("beta_fast", 32)), float(scaling.get("beta_slow", 1))

        def corr_dim(nrot):
            return (rot_dim * math.log(orig / (nrot * 2 * math.pi))) / (2 * math.log(theta))

        lo = max(math.floor(corr_dim(bf)), 0)
        hi = min(math.ceil(corr_dim(bs)), rot_dim - 1)
        ramp = torch.clamp((torch.arange(rot_dim // 2, dtype=torch.float64) - lo) / max(hi - lo, 1e-3), 0, 1)
        inter = inv / f
        inv = inter * ramp + inv * (1 - ramp)

        def ms(scale, m):
            return 1.0 if scale <= 1 else 0.1 * m * math.log(scale) + 1.0

        mscale = ms(f, float(scaling.get("mscale", 1))) / ms(f, float(scaling.get("mscale_all_dim", 0) or 1e-9)) \
            if scaling.get("mscale_all_dim") else ms(f, float(scaling.get("mscale", 1)))
    elif scaling and scaling.get("type", scaling.get("rope_type")) == "linear":
        inv = inv / float(scaling["factor"])
    pos = torch.arange(max_pos, dtype=torch.float64)
    fr = torch.outer(pos, inv)
    cs = torch.cat([fr.cos() * mscale, fr.sin() * mscale], dim=-1).float()
    return cs.to(device) if device is not None else cs


def apply_rope_ref(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, rot: int, neox: bool):
    """x [T, H, D] -> rotated copy (first `rot` dims)."""
    cs = cos_sin[positions.long()]
    half = rot // 2
    c, s = cs[:, None, :half], cs[:, None, half:]
    xf = x.float()
    out = xf.clone()
    if neox:
        x0, x1 = xf[..., :half], xf[..., half:rot]
        out[..., :half] = x0 * c - x1 * s
        out[..., half:rot] = x1 * c + x0 * s
    else:
        x0, x1 = xf[..., 0:rot:2], xf[..., 1:rot:2]
        out[..., 0:rot:2] = x0 * c - x1 * s
        out[..., 1:rot:2] = x1 * c + x0 * s
    return out.to(x.dtype)


def rope_and_cache(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
                   cos_sin: torch.Tensor, rot: int, neox: bool = True, *, slot_mapping: torch.Tensor | None = None,
                   k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                   q_norm_w: torch.Tensor | None = None, k_norm_w: torch.Tensor | None = None,
                   norm_eps: float = 1e-6, norm_add_one: bool = False, k_scale: float = 1.0,
                   v_scale: float = 1.0):
    """In place: optional per-head RMSNorm of q/k, RoPE on the first `rot` dims,
    then write k, v into the paged cache ([blocks, Hk, block_size, D]).

    q [T, Hq, D], k [T, Hk, D], v [T, Hk, Dv] may be strided views of a fused QKV
    projection output (the head dimension must be contiguous).  An e4m3 cache (k_cache
    dtype float8_e4m3fn) stores k / k_scale and v / v_scale, saturated, with V transposed
    per block ([blocks, Hk, Dv, block_size]).
    """
    T, Hq, D = q.shape
    Hk = k.shape[1]
    Dv = v.shape[2]
    if not q.is_cuda:
        if q_norm_w is not None:
            q.copy_(rmsnorm_ref(q, q_norm_w, norm_eps, add_one=norm_add_one)[0])
        if k_norm_w is not None:
            k.copy_(rmsnorm_ref(k, k_norm_w, norm_eps, add_one=norm_add_one)[0])
        if rot > 0:
            q.copy_(apply_rope_ref(q, positions, cos_sin, rot, neox))
            k.copy_(apply_rope_ref(k, positions, cos_sin, rot, neox))
        if k_cache is not None:
            write_kv_ref(k, v, slot_mapping, k_cache, v_cache, k_scale, v_scale)
        return q, k
    assert q.stride(2) == 1 and k.stride(2) == 1 and v.stride(2) == 1
    assert q.stride(1) == D and k.stride(1) == D and v.stride(1) == Dv
    bs = k_cache.shape[2] if k_cache is not None else 1
    N.call("xtu_rope_kv", q.data_ptr(), k.data_ptr(), v.data_ptr(), positions.data_ptr(), cos_sin.data_ptr(), T,
           Hq, Hk, D, Dv, rot, int(neox), q.stride(0), k.stride(0), v.stride(0), N.ptr(q_norm_w), N.ptr(k_norm_w),
           float(norm_eps), int(norm_add_one), N.ptr(slot_mapping), N.ptr(k_cache), N.ptr(v_cache), bs,
           k_cache.shape[0] * bs if k_cache is not None else 0, N.status_buffer(q.device).data_ptr(),
           int(is_fp8_cache(k_cache)), 1.0 / k_scale, 1.0 / v_scale, N.stream_ptr(q.device))
    return q, k


FP8_MAX = 448.0


def is_fp8_cache(cache: torch.Tensor | None) -> bool:
    return cache is not None and cache.dtype == torch.float8_e4m3fn


def to_e4m3(x: torch.Tensor, inv_scale: float) -> torch.Tensor:
    """x / scale -> e4m3, saturating at +-448 (as the cache-write kernel does)."""
    return (x.float() * inv_scale).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)


def write_kv_ref(k, v, slot_mapping, k_cache, v_cache, k_scale: float = 1.0, v_scale: float = 1.0):
    bs = k_cache.shape[2]
    fp8 = is_fp8_cache(k_cache)
    for t in range(k.shape[0]):
        s = int(slot_mapping[t])
        if s < 0:
            continue
        if fp8:
            k_cache[s // bs, :, s % bs] = to_e4m3(k[t], 1.0 / k_scale)
            v_cache[s // bs, :, :, s % bs] = to_e4m3(v[t], 1.0 / v_scale)
        else:
            k_cache[s // bs, :, s % bs] = k[t]
            v_cache[s // bs, :, s % bs] = v[t]


def write_kv(k, v, slot_mapping, k_cache, v_cache):
    if not k.is_cuda:
        return write_kv_ref(k, v, slot_mapping, k_cache, v_cache)
    T, Hk, D = k.shape
    Dv = v.shape[2]
    N.call("xtu_kv_write", k.data_ptr(), v.data_ptr(), T, Hk, D, Dv, k.stride(0), v.stride(0),
           slot_mapping.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[2],
           k_cache.shape[0] * k_cache.shape[2], N.status_buffer(k.device).data_ptr(), N.stream_ptr(k.device))


def write_cache_rows(x, slot_mapping, cache):
    """cache[slot // bs, :, slot % bs] = x[t] for every token t with slot >= 0 (x [T, H, D]
    bf16, cache [blocks, H, bs, D]): one kernel, no host synchronisation, so it can be
    captured in a CUDA graph (the MLA latent cache, which has no separate V cache)."""
    if not x.is_cuda:
        bs = cache.shape[2]
        sm = slot_mapping.long()
        valid = sm >= 0
        cache[(sm // bs)[valid], :, (sm % bs)[valid]] = x[valid].to(cache.dtype)
        return
    T, H, D = x.shape
    assert x.stride(2) == 1 and x.stride(1) == D and x.dtype == cache.dtype == torch.bfloat16
    N.call("xtu_kv_write", x.data_ptr(), x.data_ptr(), T, H, D, 0, x.stride(0), x.stride(0),
           slot_mapping.data_ptr(), cache.data_ptr(), cache.data_ptr(), cache.shape[2],
           cache.shape[0] * cache.shape[2], N.status_buffer(x.device).data_ptr(), N.stream_ptr(x.device))


# ---------------------------------------------------------------------------
# embedding / argmax / silu
# ---------------------------------------------------------------------------
def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Rows of ``table`` for ``ids``.  With ids on a GPU the table may also be pinned host
    memory: the kernel then reads the rows over the host link (HBM holds no copy)."""
    if not ids.is_cuda:
        return table[ids.long()]
    T = ids.numel()
    H = table.shape[1]
    y = out if out is not None else torch.empty(T, H, dtype=table.dtype, device=ids.device)
    if table.is_cuda:
        N.call("xtu_embed", ids.data_ptr(), table.data_ptr(), T, H, table.shape[0], y.data_ptr(),
               N.status_buffer(ids.device).data_ptr(), N.stream_ptr(ids.device))
    else:
        if not table.is_pinned() or table.dtype != torch.bfloat16 or not table.is_contiguous():
            raise ValueError("a host-resident embedding table must be contiguous, bf16 and pinned")
        N.call("xtu_embed_host", ids.data_ptr(), table.data_ptr(), T, H, table.shape[0], y.data_ptr(),
               N.status_buffer(ids.device).data_ptr(), N.stream_ptr(ids.device))
    return y


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy token per row (ties -> lowest index), int32."""
    if not logits.is_cuda:
        return logits.float().argmax(-1).int()
    T, V = logits.shape
    assert logits.stride(1) == 1
    y = out if out is not None else torch.empty(T, dtype=torch.int32, device=logits.device)
    ws = torch.empty(T * 64 * 2, dtype=torch.float32, device=logits.device) if V > 8192 else None
    N.call("xtu_argmax", logits.data_ptr(), int(logits.dtype == torch.bfloat16), T, V, logits.stride(0),
           y.data_ptr(), None, N.ptr(ws), N.stream_ptr(logits.device))
    return y


def silu_mul(x: torch.Tensor, limit: float = 0.0, alpha: float = 1.0, beta: float = 0.0) -> torch.Tensor:
    """[T, 2I] (gate | up) -> [T, I]."""
    T, two_i = x.shape
    I = two_i // 2
    if not x.is_cuda:
        from .gemm import silu_and_mul_clamped
        return silu_and_mul_clamped(x[:, :I], x[:, I:], limit, alpha, beta).to(x.dtype)
    y = torch.empty(T, I, dtype=x.dtype, device=x.device)
    N.call("xtu_silu_mul", x.data_ptr(), T, I, float(limit), float(alpha), float(beta), y.data_ptr(),
           N.stream_ptr(x.device))
    return y


# ---------------------------------------------------------------------------
# sigmoid gates
# ---------------------------------------------------------------------------
def gate_mul_(y: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """In place: y [T, nh, D] *= sigmoid(g [T, nh, D]) (bf16; either may be a strided view
    with a contiguous last dim) -- the gated-GQA output gate."""
    if not y.is_cuda or y.dtype != torch.bfloat16 or g.dtype != torch.bfloat16:
        y.copy_((y.float() * torch.sigmoid(g.float())).to(y.dtype))
        return y
    T, nh, D = y.shape
    assert y.stride(2) == 1 and g.stride(2) == 1 and g.shape == y.shape
    N.call("xtu_gate_mul", y.data_ptr(), y.stride(0), y.stride(1), g.data_ptr(), g.stride(0), g.stride(1), T, nh, D,
           N.stream_ptr(y.device))
    return y


def shared_gate_(y: torch.Tensor, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """In place: y [T, H] *= sigmoid(x [T, H] . w) per token, w [1, H] or [H] (bf16) -- the
    shared-expert gate."""
    wv = w.reshape(-1)
    if not y.is_cuda or y.dtype != torch.bfloat16 or x.dtype != torch.bfloat16 or wv.dtype != torch.bfloat16:
        g = torch.sigmoid(x.float() @ wv.float())
        y.copy_((y.float() * g[:, None]).to(y.dtype))
        return y
    T, H = y.shape
    assert y.stride(1) == 1 and x.stride(1) == 1 and wv.is_contiguous() and x.shape == y.shape
    N.call("xtu_shared_gate", y.data_ptr(), y.stride(0), x.data_ptr(), x.stride(0), wv.data_ptr(), T, H,
           N.stream_ptr(y.device))
    return y
