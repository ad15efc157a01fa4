"""Typed configuration registry with the reference's public environment names.

One dataclass holds every runtime knob; each field lists the environment
variables it reads (first match wins), so the reference's public surface keeps
working unchanged:

* ``VLLM_EXPERTS_LOAD_DEVICE=cpu``  -> hybrid mode (routed experts on the host
  tier; reference: mainline_shims.py:44-56)
* ``XIAOTU_PIN`` (+ ``_TABLE/_WINDOW/_HYST/_MAXSWAP/_MAX_PER_LAYER/_STATIC/_MIN_QLEN``)
  -> GPU hot-expert pool with route-driven swap-in (expert_pool.py:19-26)
* ``XIAOTU_GPF_STAGE_TILE_E`` / ``XIAOTU_GPF_STAGE_NSLOTS`` -> streamed prefill
  ring geometry (gpu_prefill.py:1673-1704; default 48 experts per tile, >=2 slots)
* ``XIAOTU_MOE_INT8`` (+ ``_VNNI_MIN_TOKENS``) -> INT8-activation x MXFP4 path
  (mixed_experts.py:1457-1490; default on for MXFP4 at M >= 160)
* ``XIAOTU_MOE_GPU_RESIDENT_LAYERS`` ("0-4,10" syntax), ``XIAOTU_MOE_RESIDENT_BUDGET_GB``

Values are read once per process (``get_engine_config``) and printed once when
``XTU_PRINT_CONFIG=1``.  An env file (``XIAOTU_ENV_FILE``) fills missing keys, so
settings survive process spawns that drop the environment (the reference's
``__init__.py:19-74`` bridge).
"""
from __future__ import annotations

import dataclasses
import os
import sys
from dataclasses import dataclass, field


def _env_file_bridge() -> None:
    path = os.environ.get("XIAOTU_ENV_FILE")
    if not path or not os.path.isfile(path):
        return
    try:
        for line in open(path):
            line = line.strip()
            if not line or line.startswith("#") or "=" not in line:
                continue
            k, v = line.split("=", 1)
            k = k.strip().removeprefix("export ").strip()
            os.environ.setdefault(k, v.strip().strip('"').strip("'"))
    except OSError:
        pass


def parse_layer_list(s: str) -> set[int]:
    """'0-4,10' -> {0,1,2,3,4,10}."""
    out: set[int] = set()
    for part in (s or "").split(","):
        part = part.strip()
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-", 1)
            out.update(range(int(a), int(b) + 1))
        else:
            out.add(int(part))
    return out


def _f(default, *envs, kind=None):
    return field(default=default, metadata={"env": envs, "kind": kind})


@dataclass
class EngineConfig:
    # tiering / placement
    experts_load_device: str = _f("auto", "VLLM_EXPERTS_LOAD_DEVICE", "XTU_EXPERTS_LOAD_DEVICE")
    resident_layers: str = _f("", "XIAOTU_MOE_GPU_RESIDENT_LAYERS")
    resident_budget_gb: float = _f(0.0, "XIAOTU_MOE_RESIDENT_BUDGET_GB")
    # hot-expert pool
    pin: bool = _f(False, "XIAOTU_PIN")
    pin_table: str = _f("", "XIAOTU_PIN_TABLE")
    pin_gib: float = _f(0.0, "XIAOTU_PIN_GIB")
    pin_window: int = _f(0, "XIAOTU_PIN_WINDOW")
    pin_hyst: float = _f(0.25, "XIAOTU_PIN_HYST")
    pin_maxswap: int = _f(0, "XIAOTU_PIN_MAXSWAP")
    pin_max_per_layer: int = _f(0, "XIAOTU_PIN_MAX_PER_LAYER")
    pin_static: bool = _f(False, "XIAOTU_PIN_STATIC")
    pin_min_qlen: int = _f(0, "XIAOTU_PIN_MIN_QLEN")
    # streamed prefill ring
    stage_tile_e: int = _f(48, "XIAOTU_GPF_STAGE_TILE_E")
    stage_nslots: int = _f(2, "XIAOTU_GPF_STAGE_NSLOTS")
    gpu_prefill_min_tokens: int = _f(256, "VLLM_XIAOTU_GPU_PREFILL_MIN_TOKENS")
    # CPU engine
    moe_threads: int = _f(0, "XIAOTU_MOE_THREADS")
    moe_int8: str = _f("auto", "XIAOTU_MOE_INT8")
    moe_int8_min_tokens: int = _f(160, "XIAOTU_MOE_INT8_VNNI_MIN_TOKENS")
    pool_deadline_ms: int = _f(300000, "XIAOTU_MOE_POOL_DEADLINE_MS")
    moe_async: bool = _f(False, "XIAOTU_MOE_ASYNC")
    moe_async_timeout_ms: int = _f(20000, "XIAOTU_MOE_ASYNC_TIMEOUT_MS")
    moe_spin_idle_us: int = _f(50, "XIAOTU_MOE_SPIN_IDLE_US")
    moe_defer: bool = _f(False, "XIAOTU_MOE_DEFER")
    moe_defer_maxq: int = _f(16, "XIAOTU_MOE_DEFER_MAXQ")
    moe_defer_maxlayer: int = _f(-1, "XIAOTU_MOE_DEFER_MAXLAYER")
    # expert parallel
    moe_ep: str = _f("auto", "XIAOTU_MOE_EP")
    # formats
    nvfp4: bool = _f(False, "XIAOTU_NVFP4")
    # observability
    nvtx: bool = _f(False, "XIAOTU_NVTX")
    layer_timing: bool = _f(False, "XIAOTU_LAYER_TIMING")
    torch_profile: str = _f("", "XIAOTU_TORCH_PROFILE")
    routing_dump: str = _f("", "XIAOTU_ROUTING_DUMP")
    print_config: bool = _f(False, "XTU_PRINT_CONFIG")
    # debug / fault injection on the host only
    fake_cpu: bool = _f(False, "XIAOTU_MOE_FAKE_CPU")
    skip_moe: bool = _f(False, "XIAOTU_MOE_SKIP")

    @classmethod
    def from_env(cls, env: dict | None = None) -> "EngineConfig":
        env = os.environ if env is None else env
        kw = {}
        for f in dataclasses.fields(cls):
            for name in f.metadata.get("env", ()):
                if name in env and env[name] != "":
                    kw[f.name] = _coerce(env[name], f.type, f.default)
                    break
        return cls(**kw)

    def hybrid(self) -> bool:
        return self.experts_load_device.lower() == "cpu"

    def resident_layer_set(self) -> set[int]:
        return parse_layer_list(self.resident_layers)

    def int8_mode(self, fmt: str, tokens: int) -> bool:
        m = self.moe_int8.lower()
        if m in ("0", "off", "false"):
            return False
        if m in ("1", "on", "true"):
            return True
        return fmt == "mxfp4" and tokens >= self.moe_int8_min_tokens

    def describe(self) -> str:
        parts = []
        for f in dataclasses.fields(self):
            v = getattr(self, f.name)
            if v != f.default:
                parts.append(f"{f.name}={v!r}")
        return "[xtu-config] " + (", ".join(parts) if parts else "defaults")


def _coerce(raw: str, typ, default):
    t = typ if isinstance(typ, type) else type(default)
    if t is bool or isinstance(default, bool):
        return raw.strip().lower() in ("1", "true", "yes", "on")
    if t is int or isinstance(default, int):
        try:
            v = int(raw.strip())
        except ValueError:
            return default
        return max(v, 0) if default >= 0 else v
    if t is float or isinstance(default, float):
        try:
            return float(raw.strip())
        except ValueError:
            return default
    return raw


_CFG: EngineConfig | None = None


def get_engine_config(refresh: bool = False) -> EngineConfig:
    global _CFG
    if _CFG is None or refresh:
        _env_file_bridge()
        _CFG = EngineConfig.from_env()
        if _CFG.print_config:
            print(_CFG.describe(), file=sys.stderr, flush=True)
    return _CFG
