"""Weight formats of the expert checkpoints and their PyTorch reference codecs.

Formats (the HF safetensors layouts the reference loads):

* **fp8 block-128** -- ``weight`` e4m3 ``[N, K]`` and ``weight_scale_inv`` fp32
  ``[ceil(N/128), ceil(K/128)]``; ``W[n,k] = e4m3[n,k] * scale[n//128, k//128]``
  (reference: xiaotu_moe/csrc/moe/moe_v2_fp8.hpp:1-20, mixed_experts.py:3326-3333).
* **MXFP4** -- e2m1 nibbles packed along K (low nibble = even k), ``[N, K/2]`` u8,
  and e8m0 scales ``[N, K/32]`` u8 with value ``2^(b-127)``
  (reference: vllm_xiaotu_moe/gpu_prefill.py:14-21).
* **NVFP4** -- e2m1 nibbles as above, e4m3 scales per 16 along K ``[N, K/16]`` and
  one fp32 ``weight_scale_2`` per tensor (reference: hybrid_model.py:477-530).

These functions are the numerics oracle for the GPU and CPU kernels, and the
random-init quantizers used by the synthetic-weight factory.
"""
from __future__ import annotations

import torch

FP8_MAX = 448.0
E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                            -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=torch.float32)


# ---------------------------------------------------------------------------
# fp8 e4m3 with 128x128 block scales
# ---------------------------------------------------------------------------
def _expand_blocks(s: torch.Tensor, n: int, k: int, bn: int = 128, bk: int = 128) -> torch.Tensor:
    return s.repeat_interleave(bn, dim=-2)[..., :n, :].repeat_interleave(bk, dim=-1)[..., :k]


def quant_fp8_block(w: torch.Tensor, block: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """w [..., N, K] float -> (e4m3 [..., N, K], fp32 scales [..., ceil(N/b), ceil(K/b)])."""
    *lead, n, k = w.shape
    nb, kb = (n + block - 1) // block, (k + block - 1) // block
    wp = torch.zeros(*lead, nb * block, kb * block, dtype=torch.float32, device=w.device)
    wp[..., :n, :k] = w.float()
    blocks = wp.reshape(*lead, nb, block, kb, block)
    amax = blocks.abs().amax(dim=(-3, -1)).clamp(min=1e-12)
    scale = amax / FP8_MAX
    q = (blocks / scale[..., :, None, :, None]).clamp(-FP8_MAX, FP8_MAX)
    q = q.reshape(*lead, nb * block, kb * block)[..., :n, :k].to(torch.float8_e4m3fn)
    return q.contiguous(), scale.contiguous()


def dequant_fp8_block(q: torch.Tensor, scale: torch.Tensor, block: int = 128) -> torch.Tensor:
    """e4m3 [..., N, K] (or its uint8 bit pattern) * block scales -> fp32."""
    if q.dtype == torch.uint8:
        q = q.view(torch.float8_e4m3fn)
    n, k = q.shape[-2], q.shape[-1]
    return q.float() * _expand_blocks(scale.float(), n, k, block, block)


# ---------------------------------------------------------------------------
# e2m1 (fp4) helpers
# ---------------------------------------------------------------------------
def _round_to_e2m1_codes(x: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest-even onto the e2m1 grid; returns 4-bit codes (sign in bit 3)."""
    mag = x.abs().clamp(max=6.0)
    grid = E2M1_VALUES[:8].to(x.device)
    # nearest grid point; ties go to the even mantissa (codes 0,2,4,6 are even)
    d = (mag[..., None] - grid).abs()
    best = d.min(dim=-1, keepdim=True).values
    cand = (d <= best + 1e-12)
    codes = torch.arange(8, device=x.device)
    # prefer even code among ties
    score = cand.float() * 2.0 + (codes % 2 == 0).float()
    code = score.argmax(dim=-1)
    sign = (x < 0) & (code > 0)
    return (code + sign.long() * 8).to(torch.uint8)


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] 4-bit codes -> [..., K/2] bytes, low nibble = even k."""
    lo = codes[..., 0::2]
    hi = codes[..., 1::2]
    return (lo | (hi << 4)).to(torch.uint8).contiguous()


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    lo = packed & 0x0F
    hi = packed >> 4
    return torch.stack([lo, hi], dim=-1).reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def e2m1_decode(codes: torch.Tensor) -> torch.Tensor:
    return E2M1_VALUES.to(codes.device)[codes.long()]


# ---------------------------------------------------------------------------
# MXFP4: e2m1 + e8m0 per 32 along K
# ---------------------------------------------------------------------------
def quant_mxfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """w [..., N, K] -> (packed [..., N, K/2] u8, e8m0 scales [..., N, K/32] u8)."""
    *lead, n, k = w.shape
    assert k % 32 == 0
    blocks = w.float().reshape(*lead, n, k // 32, 32)
    amax = blocks.abs().amax(dim=-1).clamp(min=2.0 ** -126)
    # smallest power of two s with amax / s <= 6
    e = torch.ceil(torch.log2(amax / 6.0)).clamp(-127, 127)
    scale = torch.pow(2.0, e)
    codes = _round_to_e2m1_codes(blocks / scale[..., None]).reshape(*lead, n, k)
    return pack_nibbles(codes), (e + 127).to(torch.uint8).contiguous()


def dequant_mxfp4(packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    codes = unpack_nibbles(packed)
    vals = e2m1_decode(codes)
    s = torch.pow(2.0, scales.float() - 127.0)
    *lead, n, k = vals.shape
    return (vals.reshape(*lead, n, k // 32, 32) * s[..., None]).reshape(*lead, n, k)


# ---------------------------------------------------------------------------
# NVFP4: e2m1 + e4m3 per 16 along K + fp32 per-tensor scale
# ---------------------------------------------------------------------------
def quant_nvfp4(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """w [..., N, K] -> (packed u8 [..., N, K/2], e4m3 scales [..., N, K/16], fp32 global scale [])."""
    *lead, n, k = w.shape
    assert k % 16 == 0
    blocks = w.float().reshape(*lead, n, k // 16, 16)
    amax = blocks.abs().amax(dim=-1)
    gscale = (amax.max() / (6.0 * FP8_MAX)).clamp(min=1e-12)
    s = (amax / 6.0 / gscale).clamp(max=FP8_MAX).to(torch.float8_e4m3fn)
    sf = s.float() * gscale
    sf = torch.where(sf > 0, sf, torch.ones_like(sf))
    codes = _round_to_e2m1_codes(blocks / sf[..., None]).reshape(*lead, n, k)
    return pack_nibbles(codes), s.contiguous(), gscale.reshape(()).float()


def dequant_nvfp4(packed: torch.Tensor, scales: torch.Tensor, gscale: torch.Tensor | float) -> torch.Tensor:
    codes = unpack_nibbles(packed)
    vals = e2m1_decode(codes)
    if scales.dtype == torch.uint8:
        scales = scales.view(torch.float8_e4m3fn)
    s = scales.float() * float(gscale)
    *lead, n, k = vals.shape
    return (vals.reshape(*lead, n, k // 16, 16) * s[..., None]).reshape(*lead, n, k)


def dequant_gptq(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor | None = None,
                 g_idx: torch.Tensor | None = None, bits: int = 4, zero_offset: int = 1) -> torch.Tensor:
    """GPTQ-packed linear weight -> dense fp32 [out, in] (the HF Linear layout).

    The AutoGPTQ "gptq" checkpoint format: ``qweight`` int32 [in * bits / 32, out] packs
    32 / bits consecutive input rows per word (lowest bits first); ``scales`` [groups, out];
    ``qzeros`` int32 [groups, out * bits / 32] packs the zero points along the output,
    stored minus one (``zero_offset`` 1; the "gptq_v2" format stores them as they are:
    ``zero_offset`` 0; absent: symmetric, zero point 2^(bits-1)); ``g_idx`` [in] gives each
    input row's group (absent: row // (in / groups)).  w[k, n] = (q[k, n] - z[g(k), n]) *
    scales[g(k), n].  ``bits`` 2, 4 or 8 (widths that divide the 32-bit word)."""
    if bits not in (2, 4, 8):
        raise ValueError(f"GPTQ with {bits}-bit weights is not supported (2, 4 or 8)")
    per = 32 // bits
    mask = (1 << bits) - 1
    qw = qweight.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, dtype=torch.int64) * bits
    q = ((qw[:, None, :] >> shifts[None, :, None]) & mask).reshape(qw.shape[0] * per, qw.shape[1])  # [in, out]
    K, N = q.shape
    G = scales.shape[0]
    grp = g_idx.to(torch.int64) if g_idx is not None else torch.arange(K) // (K // G)
    if qzeros is not None:
        qz = qzeros.to(torch.int64) & 0xFFFFFFFF
        z = ((qz[:, :, None] >> shifts[None, None, :]) & mask).reshape(G, -1)[:, :N] + zero_offset
    else:
        z = torch.full((G, N), 1 << (bits - 1), dtype=torch.int64)
    w = (q - z[grp]).float() * scales.float()[grp]
    return w.t().contiguous()


def gptq_to_int4_rows(qweight: torch.Tensor, scales: torch.Tensor, qzeros: torch.Tensor | None = None,
                      g_idx: torch.Tensor | None = None, zero_offset: int = 1, group: int = 128):
    """A 4-bit GPTQ linear weight kept at 4 bits, in the row layout of the CPU engine's INT4
    format: (packed uint8 [out, in / 2], low nibble = even input index; scale / zero fp32
    [out, in / group, 2]) with w[n, k] = (q - zero) * scale.  Returns None when the weight
    is not in that form (group size other than ``group``, or act-order: g_idx not in input
    order) -- the caller then dequantizes."""
    K = qweight.shape[0] * 8
    N = qweight.shape[1]
    G = scales.shape[0]
    if K % group or K // group != G:
        return None
    if g_idx is not None and not torch.equal(g_idx.to(torch.int64), torch.arange(K) // group):
        return None
    qw = qweight.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(8, dtype=torch.int64) * 4
    q = ((qw[:, None, :] >> shifts[None, :, None]) & 0xF).reshape(K, N).t().contiguous()   # [out, in]
    packed = (q[:, 0::2] | (q[:, 1::2] << 4)).to(torch.uint8)
    if qzeros is not None:
        qz = qzeros.to(torch.int64) & 0xFFFFFFFF
        z = ((qz[:, :, None] >> shifts[None, None, :]) & 0xF).reshape(G, -1)[:, :N] + zero_offset
    else:
        z = torch.full((G, N), 8, dtype=torch.int64)
    sz = torch.stack([scales.float().t(), z.float().t()], dim=-1).contiguous()          # [out, G, 2]
    return packed, sz


def dequant_int4_rows(packed: torch.Tensor, sz: torch.Tensor) -> torch.Tensor:
    """INT4 rows (``gptq_to_int4_rows``; leading dims allowed) -> fp32 [..., out, in]."""
    lo = (packed & 0xF).to(torch.float32)
    hi = (packed >> 4).to(torch.float32)
    q = torch.stack([lo, hi], dim=-1).flatten(-2)                                   # [..., out, in]
    group = q.shape[-1] // sz.shape[-2]
    s = sz[..., 0].repeat_interleave(group, dim=-1)
    z = sz[..., 1].repeat_interleave(group, dim=-1)
    return (q - z) * s
