"""Paged attention (GQA / MHA / MLA) for prefill (varlen, causal) and decode.

KV-cache layout per layer: ``k_cache [num_blocks, Hkv, block_size, D]`` and
``v_cache [num_blocks, Hkv, block_size, Dv]`` bf16 (MLA: one latent "head" of
kv_lora + rope dims, ``v_cache`` None).  A step's sequences are described by
:class:`AttnMetadata`: query rows of sequence b are ``q[q_start[b]:q_start[b+1]]``
at absolute positions ``kv_len[b] - q_len_b + i``, attending causally to keys
``[0, pos]`` found through ``block_table[b]`` -- or, with a sliding ``window``, to
``(pos - window, pos]``.  Optional per-head ``sinks`` (learned logits on the scale of the
scaled scores) join each row's softmax denominator and take no value.

On a GPU, ``paged_attention`` runs the tcgen05 flash-attention kernel in
``csrc/cuda/attention_tc.cu`` (query rows of a GQA group packed into one
128-row MMA tile, split-KV for decode); ``paged_attention_ref`` is the
PyTorch restatement used on CPU and as the test oracle.

An fp8 KV cache (GQA, ``float8_e4m3fn``): ``k_cache [num_blocks, Hkv, block_size, D]``
holds k / k_scale and ``v_cache [num_blocks, Hkv, Dv, block_size]`` holds v / v_scale,
transposed per block (the decode kernel reads 4 consecutive keys of one value column per
fragment).  Decode-shaped steps read it directly (``csrc/cuda/attention_decode.cu``);
other steps dequantise the step's blocks into bf16 scratch blocks first.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass

import torch

from . import _native as N


@dataclass
class AttnMetadata:
    num_seqs: int
    q_start: torch.Tensor        # int32 [B+1] (device)
    kv_len: torch.Tensor         # int32 [B]
    block_table: torch.Tensor    # int32 [B, max_blocks]
    slot_mapping: torch.Tensor   # int32 [T]
    positions: torch.Tensor      # int32 [T]
    max_q_len: int
    max_kv_len: int
    is_decode: bool
    # host copies (for CPU reference paths / planning); optional
    q_start_host: list | None = None
    kv_len_host: list | None = None
    seq_slots: torch.Tensor | None = None   # int32 [B] request slot (recurrent-state index)
    seq_fresh: torch.Tensor | None = None   # int32 [B] 1 if the sequence starts at position 0 this step
    num_splits: int = 1
    # sliding-window layers with a bounded pool: their own block table and KV-write slots
    swa_block_table: torch.Tensor | None = None
    swa_slot_mapping: torch.Tensor | None = None
    # > 0: a speculative verification step (rows per sequence); recurrent layers keep the
    # state after every row for the rollback of rejected drafts
    spec_rows: int = 0

    @property
    def num_tokens(self) -> int:
        return self.slot_mapping.shape[0]


def _gather_kv(cache: torch.Tensor, block_table_row: torch.Tensor, n: int) -> torch.Tensor:
    """[num_blocks, H, bs, D] -> [n, H, D] for the first n tokens of one sequence."""
    bs = cache.shape[2]
    nb = (n + bs - 1) // bs
    blocks = cache[block_table_row[:nb].long()]            # [nb, H, bs, D]
    return blocks.permute(0, 2, 1, 3).reshape(nb * bs, cache.shape[1], cache.shape[3])[:n]


def dequant_fp8_cache(k_cache: torch.Tensor, v_cache: torch.Tensor, k_scale: float = 1.0, v_scale: float = 1.0):
    """fp8 GQA cache -> bf16 caches in the plain layout (K and V [blocks, Hkv, bs, D])."""
    k = (k_cache.float() * k_scale).to(torch.bfloat16)
    v = (v_cache.float() * v_scale).transpose(2, 3).contiguous().to(torch.bfloat16)
    return k, v


def paged_attention_ref(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor | None, meta: AttnMetadata,
                        scale: float, v_dim: int | None = None, out: torch.Tensor | None = None, window: int = 0,
                        sinks: torch.Tensor | None = None, k_scale: float = 1.0,
                        v_scale: float = 1.0) -> torch.Tensor:
    """q [T, Hq, Dqk] -> o [T, Hq, Dv] (fp32 math)."""
    if k_cache.dtype == torch.float8_e4m3fn:
        k_cache, v_cache = dequant_fp8_cache(k_cache, v_cache, k_scale, v_scale)
    T, Hq, D = q.shape
    qs = meta.q_start_host if meta.q_start_host is not None else meta.q_start.tolist()
    kl = meta.kv_len_host if meta.kv_len_host is not None else meta.kv_len.tolist()
    Dv = v_dim if v_dim is not None else (v_cache.shape[3] if v_cache is not None else D)
    o = out if out is not None else torch.zeros(T, Hq, Dv, dtype=q.dtype, device=q.device)
    for b in range(meta.num_seqs):
        s0, s1 = qs[b], qs[b + 1]
        ql = s1 - s0
        if ql == 0:
            continue
        n = kl[b]
        k = _gather_kv(k_cache, meta.block_table[b], n).float()          # [n, Hk, D]
        v = _gather_kv(v_cache, meta.block_table[b], n).float() if v_cache is not None else k[..., :Dv]
        Hk = k.shape[1]
        G = Hq // Hk
        qq = q[s0:s1].float()                                              # [ql, Hq, D]
        kk = k.repeat_interleave(G, dim=1)
        vv = v.repeat_interleave(G, dim=1)
        s = torch.einsum("qhd,khd->hqk", qq, kk) * scale
        pos = torch.arange(n - ql, n, device=q.device)
        keys = torch.arange(n, device=q.device)[None, :]
        mask = keys > pos[:, None]
        if window > 0:
            mask |= keys <= pos[:, None] - window
        s = s.masked_fill(mask[None], float("-inf"))
        if sinks is not None:   # one more logit per row that takes no value
            sk = sinks.float().to(q.device)[:, None, None].expand(Hq, ql, 1)
            p = torch.softmax(torch.cat([s, sk], dim=-1), dim=-1)[..., :-1]
        else:
            p = torch.softmax(s, dim=-1)
        o[s0:s1] = torch.einsum("hqk,khd->qhd", p, vv).to(o.dtype)
    return o


KV_BLOCK = 64   # tokens per KV-cache block read by the GPU kernel
_SPLIT_COUNTERS: dict = {}
_MAX_SPLIT_GROUPS = 1 << 16


def _split_counters(device) -> torch.Tensor:
    """Per-device zeroed ints, one per (sequence, kv head): the decode kernel's last
    split CTA of a group merges the partials and re-zeroes its counter.  Allocated once
    (captured graphs keep the pointer)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _SPLIT_COUNTERS.get(key)
    if t is None:
        t = torch.zeros(_MAX_SPLIT_GROUPS, dtype=torch.int32, device=device)
        _SPLIT_COUNTERS[key] = t
    return t


def split_counters_reset(device) -> None:
    """Re-zero the split counters (after a launch that reported an error)."""
    key = device.index if device.index is not None else torch.cuda.current_device()
    t = _SPLIT_COUNTERS.get(key)
    if t is not None:
        t.zero_()


def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor | None, meta: AttnMetadata,
                    scale: float | None = None, v_dim: int | None = None, out: torch.Tensor | None = None,
                    workspace: torch.Tensor | None = None, window: int = 0,
                    sinks: torch.Tensor | None = None, k_scale: float = 1.0, v_scale: float = 1.0) -> torch.Tensor:
    T, Hq, D = q.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if not q.is_cuda or not N.has_symbol("xtu_paged_attention"):
        if q.is_cuda and N.native_required():
            raise N.NativeLibraryMissing("xtu_paged_attention missing from the CUDA library")
        return paged_attention_ref(q, k_cache, v_cache, meta, scale, v_dim, out, window, sinks, k_scale, v_scale)
    if k_cache.dtype == torch.float8_e4m3fn:
        return _paged_attention_fp8(q, k_cache, v_cache, meta, scale, out, workspace, window, sinks, k_scale, v_scale)
    Hk = k_cache.shape[1]
    if sinks is not None:
        assert sinks.dtype == torch.float32 and sinks.is_contiguous() and sinks.numel() == Hq
    if k_cache.shape[2] != KV_BLOCK:
        raise ValueError(f"the GPU paged-attention kernel reads KV blocks of {KV_BLOCK} tokens, "
                         f"not {k_cache.shape[2]} (set RunnerConfig.block_size={KV_BLOCK})")
    Dv = v_dim if v_dim is not None else (v_cache.shape[3] if v_cache is not None else D)
    o = out if out is not None else torch.empty(T, Hq, Dv, dtype=q.dtype, device=q.device)
    assert q.stride(2) == 1 and q.stride(1) == D and o.is_contiguous()
    splits = meta.num_splits
    ws = workspace
    need = num_split_workspace(T, Hq, Dv, splits) if splits > 1 else 0
    if need and (ws is None or ws.numel() < need):
        ws = torch.empty(need, dtype=torch.float32, device=q.device)
    vc = v_cache if v_cache is not None else k_cache
    cnt = _split_counters(q.device) if splits > 1 and meta.num_seqs * Hk <= _MAX_SPLIT_GROUPS else None
    N.call("xtu_paged_attention", q.data_ptr(), q.stride(0), k_cache.data_ptr(), vc.data_ptr(),
           int(v_cache is None), o.data_ptr(), o.stride(0), meta.q_start.data_ptr(), meta.kv_len.data_ptr(),
           meta.block_table.data_ptr(), meta.block_table.stride(0), meta.num_seqs, meta.max_q_len,
           meta.max_kv_len, T, Hq, Hk, D, Dv, k_cache.shape[2], k_cache.shape[0], float(scale), splits,
           N.ptr(ws) if splits > 1 else None, N.ptr(cnt), int(window),
           N.ptr(sinks), N.status_buffer(q.device).data_ptr(),
           N.stream_ptr(q.device))
    return o


def _paged_attention_fp8(q, k_cache, v_cache, meta: AttnMetadata, scale, out, workspace, window, sinks, k_scale,
                         v_scale) -> torch.Tensor:
    T, Hq, D = q.shape
    nb, Hk, bs, _ = k_cache.shape
    Dv = v_cache.shape[2]
    assert v_cache.shape == (nb, Hk, Dv, bs) and bs == KV_BLOCK, "fp8 V cache is [blocks, Hkv, Dv, 64]"
    o = out if out is not None else torch.empty(T, Hq, Dv, dtype=q.dtype, device=q.device)
    assert q.stride(2) == 1 and q.stride(1) == D and o.is_contiguous()
    if D == Dv and meta.max_q_len * (Hq // Hk) <= 64 and D in (64, 128):
        splits = meta.num_splits
        ws = workspace
        need = num_split_workspace(T, Hq, Dv, splits) if splits > 1 else 0
        if need and (ws is None or ws.numel() < need):
            ws = torch.empty(need, dtype=torch.float32, device=q.device)
        cnt = _split_counters(q.device) if splits > 1 and meta.num_seqs * Hk <= _MAX_SPLIT_GROUPS else None
        if splits == 1 or cnt is not None:
            r = N.call("xtu_paged_attention_fp8", q.data_ptr(), q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(),
                       o.data_ptr(), o.stride(0), meta.q_start.data_ptr(), meta.kv_len.data_ptr(),
                       meta.block_table.data_ptr(), meta.block_table.stride(0), meta.num_seqs, meta.max_q_len, T, Hq,
                       Hk, D, nb, float(scale), float(k_scale), float(v_scale), splits,
                       N.ptr(ws) if splits > 1 else None, N.ptr(cnt), int(window), N.ptr(sinks),
                       N.status_buffer(q.device).data_ptr(), N.stream_ptr(q.device))
            if r == 1:
                return o
    # other shapes (prefill chunks, long verification steps): the step's blocks as bf16
    if torch.cuda.is_current_stream_capturing():
        raise RuntimeError("fp8 KV: this attention shape needs a dequantised copy, which cannot be captured")
    kl = meta.kv_len_host if meta.kv_len_host is not None else meta.kv_len.tolist()
    nblk = [(int(n) + bs - 1) // bs for n in kl]
    start = [0]
    for n in nblk:
        start.append(start[-1] + n)
    total, mx = start[-1], max(nblk) if nblk else 0
    kb = torch.empty(max(1, total), Hk, bs, D, dtype=torch.bfloat16, device=q.device)
    vb = torch.empty(max(1, total), Hk, bs, Dv, dtype=torch.bfloat16, device=q.device)
    bt = torch.zeros(meta.num_seqs, max(1, mx), dtype=torch.int32, device=q.device)
    st = torch.tensor(start, dtype=torch.int32).to(q.device, non_blocking=True)
    N.call("xtu_kv_dequant_gather", k_cache.data_ptr(), v_cache.data_ptr(), meta.block_table.data_ptr(),
           meta.block_table.stride(0), st.data_ptr(), meta.kv_len.data_ptr(), meta.num_seqs, mx, Hk, D, Dv,
           float(k_scale), float(v_scale), kb.data_ptr(), vb.data_ptr(), bt.data_ptr(), bt.stride(0), nb,
           N.status_buffer(q.device).data_ptr(), N.stream_ptr(q.device))
    m2 = dataclasses.replace(meta, block_table=bt)
    return paged_attention(q, kb, vb, m2, scale, Dv, o, workspace, window, sinks)


def num_split_workspace(T: int, Hq: int, Dv: int, splits: int) -> int:
    """fp32 elements of split-KV partials: O [splits, T, Hq, Dv] + (m, l) [splits, T, Hq, 2]."""
    return splits * T * Hq * (Dv + 2)


def choose_splits(num_seqs: int, num_kv_heads: int, max_kv_len: int, rows_per_tile_tiles: int = 1,
                  num_sms: int = 148, ctas_per_sm: int = 1) -> int:
    """Split-KV factor for decode: the largest split count whose CTAs (seqs x kv heads x
    splits, `ctas_per_sm` resident per SM) still fit in one wave, so no SM runs a lone
    second-wave CTA."""
    slots = num_sms * ctas_per_sm
    ctas = max(1, num_seqs * num_kv_heads * rows_per_tile_tiles)
    if ctas >= slots:
        return 1
    per_split_min = 512  # keys
    max_split = max(1, max_kv_len // per_split_min)
    return int(max(1, min(max_split, slots // ctas, 64)))


def decode_ctas_per_sm(cfg, q_len: int = 1) -> int:
    """CTAs per SM the split count of a decode step of ``q_len`` query positions per
    sequence is sized for: the warp-level GQA decode kernel (head_dim 64 or 128, 96 KB ring)
    runs two per SM up to 32 query rows per KV head; with more rows (MTP verification steps
    of a large GQA group: four m-tiles per CTA) one CTA keeps an SM's tensor pipe busy and
    a second one only slows both (measured: 4 x 15K-token sequences, 60 rows per KV head,
    94 us at 4 splits against 121 us at 9).  The tcgen05 kernel (MLA, other head sizes)
    runs one per SM."""
    if cfg.is_mla or cfg.head_dim not in (64, 128):
        return 1
    G = cfg.num_heads // max(1, cfg.num_kv_heads)
    return 2 if q_len * G <= 32 else 1
