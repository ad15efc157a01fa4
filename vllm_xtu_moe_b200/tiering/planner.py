"""VRAM priority planner: how one GPU's memory is split between the KV cache, the
prefill staging ring, the MTP drafter, GPU-resident expert layers and hot-expert
pools (the reference's ``vram_policy.plan``/``emit_env``, vllm_xiaotu_moe/
vram_policy.py:167,363, sized here for 180 GB parts).

Fixed priority, each step taking what it needs from what is left:
  1. non-expert weights (attention, dense/shared MLPs, embeddings, routers) -- always GPU;
  2. KV cache for ``max_model_len`` x ``max_seqs`` tokens (plus the CUDA-graph pool);
  3. the streamed-prefill ring (``staging_bytes``), so long prompts never fall back to CPU;
  4. the MTP drafter layers, GPU-resident so speculation stays on the device;
  5. whole resident expert layers, middle layers first (``order``);
  6. the rest, divided evenly across host-tier layers, as hot-expert pool slots
     (capped by ``pin_max_per_layer``).

The result can be emitted as the ``XIAOTU_*`` environment that configures
:class:`~vllm_xtu_moe_b200.tiering.executor.TieredExperts`.
"""
from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass, field

from ..models.config import ModelConfig, get_preset
from .ring import staging_bytes

GiB = 1 << 30


def expert_bytes(cfg: ModelConfig, fmt: str | None = None) -> int:
    """Bytes of one routed expert (gate, up, down) including block scales."""
    fmt = fmt or cfg.expert_fmt
    H, I = cfg.hidden_size, cfg.moe_intermediate
    n = 3 * H * I
    if fmt == "bf16":
        return 2 * n
    if fmt == "fp8":
        return n + 4 * (((2 * I + 127) // 128) * ((H + 127) // 128) + ((H + 127) // 128) * ((I + 127) // 128))
    if fmt == "mxfp4":
        return n // 2 + n // 32
    if fmt == "nvfp4":
        return n // 2 + n // 16 + 8
    raise ValueError(fmt)


def kv_bytes_per_token(cfg: ModelConfig, kv_dtype_bytes: int = 2, layer_type: str = "full") -> int:
    """Paged-KV bytes per token over the layers of one attention type ("full": they grow
    with the context; "swa": they hold one window per sequence)."""
    attn = [i for i in range(cfg.num_layers) if cfg.layer_type(i) == layer_type]
    if cfg.is_mla:
        return len(attn) * (cfg.kv_lora_rank + cfg.qk_rope_head_dim) * kv_dtype_bytes
    return sum(cfg.kv_heads(i) * (cfg.head_dim + cfg.gqa_v_dim) for i in attn) * kv_dtype_bytes


def kv_bytes(cfg: ModelConfig, max_model_len: int, max_seqs: int, max_batched_tokens: int = 16384,
             block_size: int = 64) -> int:
    """KV-cache bytes the runner allocates: the full-context layers for every sequence at
    max_model_len, plus the sliding-window layers' bounded pool."""
    from ..engine.block_manager import swa_pool_blocks
    n = kv_bytes_per_token(cfg) * max_model_len * max_seqs
    if cfg.sliding_window > 0:
        blocks = swa_pool_blocks(max_seqs, cfg.sliding_window, block_size, max_batched_tokens)
        n += kv_bytes_per_token(cfg, layer_type="swa") * blocks * block_size
    return n


def non_expert_bytes(cfg: ModelConfig) -> int:
    total = cfg.param_count(active=False)
    moe_layers = sum(1 for i in range(cfg.num_layers) if cfg.is_moe_layer(i))
    routed = moe_layers * cfg.num_experts * 3 * cfg.hidden_size * cfg.moe_intermediate
    dense_b = 1 if cfg.dense_fmt == "fp8" else 2
    return max(0, total - routed) * dense_b


@dataclass
class Placement:
    gpu_bytes: int
    non_expert: int
    kv: int
    staging: int
    drafter: int
    resident_layers: list[int] = field(default_factory=list)
    pool_per_layer: int = 0
    pool_layers: list[int] = field(default_factory=list)
    free: int = 0
    notes: list[str] = field(default_factory=list)

    def to_env(self, tile_e: int, nslots: int) -> dict[str, str]:
        env = {"XIAOTU_GPF_STAGE_TILE_E": str(tile_e), "XIAOTU_GPF_STAGE_NSLOTS": str(nslots)}
        if self.resident_layers:
            env["XIAOTU_MOE_GPU_RESIDENT_LAYERS"] = _ranges(self.resident_layers)
        if self.pool_per_layer:
            env["XIAOTU_PIN"] = "1"
            env["XIAOTU_PIN_MAX_PER_LAYER"] = str(self.pool_per_layer)
        return env

    def summary(self) -> dict:
        d = asdict(self)
        for k in ("gpu_bytes", "non_expert", "kv", "staging", "drafter", "free"):
            d[k + "_gib"] = round(d.pop(k) / GiB, 2)
        return d


def _ranges(xs: list[int]) -> str:
    xs = sorted(xs)
    out, i = [], 0
    while i < len(xs):
        j = i
        while j + 1 < len(xs) and xs[j + 1] == xs[j] + 1:
            j += 1
        out.append(str(xs[i]) if i == j else f"{xs[i]}-{xs[j]}")
        i = j + 1
    return ",".join(out)


def middle_first(layers: list[int]) -> list[int]:
    """Resident-layer order: the middle of the stack first, alternating outwards."""
    if not layers:
        return []
    mid = (len(layers) - 1) / 2
    return sorted(layers, key=lambda l: (abs(layers.index(l) - mid), l))


def plan(cfg: ModelConfig, gpu_gib: float = 178.0, *, max_model_len: int = 16384, max_seqs: int = 4,
         tile_e: int = 48, nslots: int = 2, drafter_layers: int | None = None, graph_pool_gib: float = 2.0,
         reserve_gib: float = 4.0, pin_max_per_layer: int = 0, order: list[int] | None = None) -> Placement:
    gpu = int(gpu_gib * GiB)
    ne = non_expert_bytes(cfg)
    kv = kv_bytes(cfg, max_model_len, max_seqs) + int(graph_pool_gib * GiB)
    eb = expert_bytes(cfg)
    layer_b = eb * cfg.num_experts
    gfmt = cfg.expert_fmt in ("bf16", "fp8", "mxfp4", "nvfp4")
    te = max(1, min(tile_e, cfg.num_experts))
    stage = staging_bytes(cfg.expert_fmt, cfg.hidden_size, cfg.moe_intermediate, te, nslots) if gfmt else 0
    nd = cfg.num_mtp_layers if drafter_layers is None else drafter_layers
    drafter = nd * layer_b
    p = Placement(gpu, ne, kv, stage, drafter)
    left = gpu - int(reserve_gib * GiB) - ne - kv
    if left < 0:
        p.notes.append("non-expert weights + KV exceed the GPU; lower max_model_len or max_seqs")
        p.free = left
        return p
    if stage > left:
        p.notes.append("no room for the prefill ring; long prefill runs on the CPU tier")
        p.staging = stage = 0
    left -= stage
    if drafter > left:
        p.notes.append("drafter layers stay on the CPU tier")
        p.drafter = drafter = 0
    left -= drafter
    moe = [i for i in range(cfg.num_layers) if cfg.is_moe_layer(i)]
    for l in (order or middle_first(moe)):
        if layer_b <= left:
            p.resident_layers.append(l)
            left -= layer_b
    host_layers = [l for l in moe if l not in p.resident_layers]
    if host_layers and gfmt:
        per = left // (eb * len(host_layers))
        if pin_max_per_layer:
            per = min(per, pin_max_per_layer)
        per = int(min(per, cfg.num_experts - 1))
        if per > 0:
            p.pool_per_layer = per
            p.pool_layers = host_layers
            left -= per * eb * len(host_layers)
    p.resident_layers.sort()
    p.free = left
    return p


def main(argv=None):
    ap = argparse.ArgumentParser(description="VRAM placement plan for one GPU")
    ap.add_argument("--model", default="glm-4.5-air")
    ap.add_argument("--gpu-gib", type=float, default=178.0)
    ap.add_argument("--max-model-len", type=int, default=16384)
    ap.add_argument("--max-seqs", type=int, default=4)
    ap.add_argument("--tile-e", type=int, default=48)
    ap.add_argument("--nslots", type=int, default=2)
    ap.add_argument("--pin-max-per-layer", type=int, default=0)
    ap.add_argument("--env", action="store_true", help="print shell exports instead of JSON")
    a = ap.parse_args(argv)
    cfg = get_preset(a.model)
    p = plan(cfg, a.gpu_gib, max_model_len=a.max_model_len, max_seqs=a.max_seqs, tile_e=a.tile_e, nslots=a.nslots,
             pin_max_per_layer=a.pin_max_per_layer)
    if a.env:
        for k, v in p.to_env(a.tile_e, a.nslots).items():
            print(f"export {k}={v}")
    else:
        print(json.dumps(p.summary(), indent=1))


if __name__ == "__main__":
    main()
