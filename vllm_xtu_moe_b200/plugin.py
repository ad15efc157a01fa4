"""vLLM general-plugin entry point (``vllm.general_plugins`` -> ``vllm_xtu_moe_b200:register``).

The reference registers itself into vLLM as a plugin and swaps vLLM's expert
backend for its own (vllm_xiaotu_moe/__init__.py:162-194, mixed_experts.py:3486).
This framework owns its executor instead, so ``register`` does what still applies
inside a stock vLLM process:

* fills the environment from ``XIAOTU_ENV_FILE`` and loads the typed config once
  (the same ``XIAOTU_*`` / ``VLLM_EXPERTS_LOAD_DEVICE`` knobs);
* registers the library's kernels as PyTorch custom ops under the ``xtu`` namespace
  (``torch.ops.xtu.fused_moe``, ``rmsnorm``, ``argmax``), so model code running in
  any PyTorch program, vLLM's included, can call the sm_100a MoE / norm / sampling
  kernels without importing this package's model stack.

Serving itself goes through ``python -m vllm_xtu_moe_b200.serve`` (OpenAI-compatible).
"""
from __future__ import annotations

import torch

from .config import get_engine_config

_REGISTERED = False


def _define_ops() -> None:
    from .ops import basic as B
    from .ops import moe as M

    lib = torch.library.Library("xtu", "DEF")
    lib.define("fused_moe(Tensor x, Tensor ids, Tensor weights, Tensor w13, Tensor w2, Tensor? s13, Tensor? s2, "
               "bool interleaved, float act_limit) -> Tensor")
    lib.define("rmsnorm(Tensor x, Tensor w, float eps) -> Tensor")
    lib.define("argmax(Tensor logits) -> Tensor")

    def fused_moe(x, ids, weights, w13, w2, s13, s2, interleaved, act_limit):
        fmt = "fp8" if s13 is not None else "bf16"
        ex = M.ExpertWeights(fmt, w13, w2, s13, s2, interleaved)
        return M.fused_moe(x.contiguous(), ids.to(torch.int32).contiguous(), weights.float().contiguous(), ex,
                           act_limit=act_limit)

    def rmsnorm(x, w, eps):
        return B.rmsnorm(x, w, eps)

    def argmax(logits):
        return B.argmax(logits)

    for dev in ("CUDA", "CPU"):
        lib.impl("fused_moe", fused_moe, dev)
        lib.impl("rmsnorm", rmsnorm, dev)
        lib.impl("argmax", argmax, dev)
    globals()["_LIB"] = lib


def register():
    """Idempotent; returns the effective engine config."""
    global _REGISTERED
    cfg = get_engine_config()
    if not _REGISTERED:
        _define_ops()
        _REGISTERED = True
    return cfg
