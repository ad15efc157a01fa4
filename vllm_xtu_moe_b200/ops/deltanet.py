"""Gated DeltaNet and Kimi Delta Attention on the GPU (``csrc/cuda/deltanet.cu``): conv +
L2 norm, conv-state update and the gated delta-rule recurrence (scalar decay per head, or
channel-wise decay per key dim) over a step's sequences."""
from __future__ import annotations

import torch

from . import _native as N


def deltanet_fwd(qkvz: torch.Tensor, conv_w32: torch.Tensor, g: torch.Tensor, beta: torch.Tensor, meta, state,
                 nk: int, nv: int, dk: int, dv: int, blocked: bool = False) -> torch.Tensor:
    """qkvz [T, W] bf16 (in_proj output: per key head [q | k | v | z], or ``blocked``
    [Q | K | V] for KDA), conv_w32 fp32 [ch, kw], g fp32 [T, nv] or [T, nv, dk] (channel-wise
    decay), beta fp32 [T, nv] -> o fp32 [T, nv, dv].

    Updates ``state.conv`` and ``state.ssm`` of the step's sequence slots in place."""
    T = qkvz.shape[0]
    d = qkvz.device
    qs = torch.empty(T, nk, dk, dtype=torch.float32, device=d)
    ks = torch.empty(T, nk, dk, dtype=torch.float32, device=d)
    vs = torch.empty(T, nv, dv, dtype=torch.float32, device=d)
    out = torch.empty(T, nv, dv, dtype=torch.float32, device=d)
    g = g.float().contiguous()
    beta = beta.float().contiguous()
    N.call("xtu_deltanet_fwd", qkvz.data_ptr(), qkvz.stride(0), T, meta.num_seqs, meta.q_start.data_ptr(),
           meta.seq_slots.data_ptr(), N.ptr(meta.seq_fresh), nk, nv, dk, dv, conv_w32.shape[1],
           conv_w32.data_ptr(), state.conv.data_ptr(), state.ssm.data_ptr(), g.data_ptr(), beta.data_ptr(),
           qs.data_ptr(), ks.data_ptr(), vs.data_ptr(), out.data_ptr(), int(blocked), int(g.dim() == 3),
           N.stream_ptr(d))
    return out
