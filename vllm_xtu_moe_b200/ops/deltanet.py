"""Gated DeltaNet and Kimi Delta Attention on the GPU (``csrc/cuda/deltanet.cu``): conv +
L2 norm, conv-state update and the gated delta-rule recurrence (scalar decay per head, or
channel-wise decay per key dim) over a step's sequences."""
from __future__ import annotations

import os

import torch

from . import _native as N


# the chunked tensor-core form serves prefill steps whose longest sequence chunk reaches
# this many tokens (scalar decay, dv = 128); shorter steps run the token-serial kernel
CHUNK_MIN_TOKENS = int(os.environ.get("XTU_GDN_CHUNK_MIN", "64"))


def deltanet_fwd(qkvz: torch.Tensor, conv_w32: torch.Tensor, g: torch.Tensor | None, beta: torch.Tensor | None,
                 meta, state, nk: int, nv: int, dk: int, dv: int, blocked: bool = False,
                 chunked: bool | None = None, ba: torch.Tensor | None = None, A_log32: torch.Tensor | None = None,
                 dt_bias32: torch.Tensor | None = None, norm_w32: torch.Tensor | None = None, eps: float = 1e-6,
                 gate: torch.Tensor | None = None) -> torch.Tensor:
    """qkvz [T, W] bf16 (in_proj output: per key head [q | k | v | z], or ``blocked``
    [Q | K | V] for KDA), conv_w32 fp32 [ch, kw], g fp32 [T, nv] or [T, nv, dk] (channel-wise
    decay), beta fp32 [T, nv] -> o fp32 [T, nv, dv].

    ``ba`` (the in_proj_ba output [T, 2 nv] bf16, with ``A_log32`` / ``dt_bias32`` fp32 [nv])
    in place of g and beta: the conv kernel forms beta = sigmoid(b) and
    g = -exp(A_log) softplus(a + dt_bias) itself.  ``norm_w32`` fp32 [dv]: the result is the
    gated RMSNorm y = rmsnorm(o) * w * act(gate) as bf16 [T, nv * dv], act = silu of the z
    part of ``qkvz`` (``gate`` None) or sigmoid of ``gate`` [T, nv * dv] bf16.

    Updates ``state.conv`` and ``state.ssm`` of the step's sequence slots in place."""
    T = qkvz.shape[0]
    d = qkvz.device
    qs = torch.empty(T, nk, dk, dtype=torch.float32, device=d)
    ks = torch.empty(T, nk, dk, dtype=torch.float32, device=d)
    vs = torch.empty(T, nv, dv, dtype=torch.float32, device=d)
    out = torch.empty(T, nv, dv, dtype=torch.float32, device=d)
    if ba is not None:
        assert ba.stride(1) == 1 and A_log32 is not None and dt_bias32 is not None and not blocked
        g = torch.empty(T, nv, dtype=torch.float32, device=d)
        beta = torch.empty(T, nv, dtype=torch.float32, device=d)
    else:
        g = g.float().contiguous()
        beta = beta.float().contiguous()
    # speculative verification: the states after every token are kept for the rollback
    spec_n = meta.max_q_len if getattr(meta, "spec_rows", 0) > 0 and state.spec_ssm is not None else 0
    if spec_n and spec_n > state.spec_ssm.shape[1]:
        raise ValueError(f"verification step of {spec_n} tokens per sequence > {state.spec_ssm.shape[1]} spec states")
    spec_ssm = state.spec_ssm if spec_n else None
    spec_conv = state.spec_conv if spec_n else None
    if chunked is None:
        chunked = not meta.is_decode and meta.max_q_len >= CHUNK_MIN_TOKENS
    chunked = bool(chunked) and g.dim() == 2 and dk == 128 and dv == 128
    # W [T, nv, 128], P [T, nv, 64] and the in-chunk cumulative decay [T, nv] of the chunked form
    ws = torch.empty(T * nv * (128 + 64 + 1), dtype=torch.float32, device=d) if chunked else None
    y = None
    if norm_w32 is not None:
        y = torch.empty(T, nv * dv, dtype=torch.bfloat16, device=d)
        if gate is None:
            assert not blocked
            gate_t, gate_mode = qkvz, 0
        else:
            assert gate.stride(1) == 1
            gate_t, gate_mode = gate, 1
    N.call("xtu_deltanet_fwd", qkvz.data_ptr(), qkvz.stride(0), T, meta.num_seqs, meta.q_start.data_ptr(),
           meta.seq_slots.data_ptr(), N.ptr(meta.seq_fresh), nk, nv, dk, dv, conv_w32.shape[1],
           conv_w32.data_ptr(), state.conv.data_ptr(), state.ssm.data_ptr(), g.data_ptr(), beta.data_ptr(),
           qs.data_ptr(), ks.data_ptr(), vs.data_ptr(), out.data_ptr(), int(blocked), int(g.dim() == 3),
           int(chunked), N.ptr(ws), N.ptr(ba), ba.stride(0) if ba is not None else 0, N.ptr(A_log32),
           N.ptr(dt_bias32), N.ptr(gate_t) if y is not None else None, gate_t.stride(0) if y is not None else 0,
           gate_mode if y is not None else 0, N.ptr(norm_w32), float(eps), N.ptr(y),
           N.ptr(spec_ssm), N.ptr(spec_conv), spec_n, N.stream_ptr(d))
    return out if y is None else y
