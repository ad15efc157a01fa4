"""vllm_xtu_moe_b200: a B200-native tiered MoE inference framework.

Packages:
  models/    model configs, layers (GQA, MLA, gated DeltaNet, MoE), synthetic weights, HF loading
  ops/       sm_100a kernels (ctypes) with PyTorch restatements used on CPU and in tests
  engine/    scheduler, paged KV blocks, model runner (CUDA graphs), MTP speculative decoding, LLM API
  tiering/   expert placement: GPU-resident pool, streamed prefill ring, CPU engine bridge, planner
  parallel/  process groups, symmetric memory, fused EP dispatch/combine and TP GEMM+collective
  utils/     logging, timing, tracing, safetensors IO
"""
__version__ = "0.1.0"

from .config import EngineConfig, get_engine_config  # noqa: F401
from .utils.diagnostics import install_death_debug as _install_death_debug

_install_death_debug()       # XIAOTU_DEATH_DEBUG=1: signal stack dumps + heartbeat


def register():
    """vLLM general-plugin entry point (``vllm.general_plugins``)."""
    from .plugin import register as _register
    return _register()
