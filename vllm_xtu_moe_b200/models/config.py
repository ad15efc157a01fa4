"""Model architecture configs and the presets of the benchmarked families.

One dataclass describes every family the framework serves: Mixtral-style
(GQA + softmax top-k MoE), GLM-4.5-style (GQA with partial RoPE and qkv bias,
sigmoid router with correction bias, shared expert, leading dense layers, MTP
layer), Qwen3-Next-style (3 gated-DeltaNet : 1 gated-GQA, 512 experts, shared
expert with a sigmoid gate, zero-centred norms), DeepSeek-V3-style (MLA,
group-limited sigmoid router, shared expert, leading dense layers), MiMo-V2-style
(hybrid global / sliding-window GQA with their own KV-head counts, 192-wide q/k and
128-wide v heads, learned attention sinks on the sliding-window layers) and
Kimi-Linear-style (3 Kimi Delta Attention : 1 MLA without RoPE).
``from_hf_config`` maps a HF ``config.json`` onto it.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class ModelConfig:
    name: str
    arch: str                      # "mixtral" | "glm4_moe" | "qwen3_next" | "deepseek_v3" | "mimo_v2" | "kimi_linear"
    vocab_size: int
    hidden_size: int
    num_layers: int
    # attention (GQA)
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float = 10000.0
    rotary_dim: int | None = None  # partial RoPE (GLM: head_dim/2, Qwen3-Next: head_dim/4)
    rope_neox: bool = True
    rope_scaling: dict | None = None
    qkv_bias: bool = False
    qk_norm: bool = False
    attn_output_gate: bool = False  # Qwen3-Next gated attention
    # MLA (DeepSeek-V3)
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_nope_head_dim: int = 0
    qk_rope_head_dim: int = 0
    v_head_dim: int = 0            # MLA value width; for GQA a value width other than head_dim
    # sliding-window attention (MiMo-V2): layers of type "swa"
    sliding_window: int = 0
    swa_num_kv_heads: int = 0      # KV heads of the "swa" layers (0: num_kv_heads)
    attn_sinks: str = ""           # learned per-head sink logits on "swa" | "full" | "all" layers
    # gated DeltaNet linear attention (Qwen3-Next)
    layer_types: list[str] | None = None   # per layer: "full" | "linear" | "swa"
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel: int = 4
    linear_kind: str = "gdn"       # "gdn" (Qwen3-Next gated DeltaNet) | "kda" (Kimi Delta Attention)
    mla_rope: bool = True          # False: MLA without rotary embedding (Kimi-Linear's NoPE MLA)
    # DeepSeek sparse attention (DeepSeek-V3.2-style MLA): a lightning indexer scores every
    # context token per query and attention runs over the index_topk best (0 = dense MLA)
    index_topk: int = 0
    index_n_heads: int = 64
    index_head_dim: int = 128
    # MLP / MoE
    num_dense_layers: int = 0      # leading dense-MLP layers
    dense_intermediate: int = 0
    num_experts: int = 0
    top_k: int = 0
    moe_intermediate: int = 0
    num_shared_experts: int = 0
    shared_intermediate: int = 0
    shared_expert_gate: bool = False  # Qwen3-Next: sigmoid(x W_g) * shared(x)
    scoring: str = "softmax"
    router_bias: bool = False        # e_score_correction_bias
    n_group: int = 1
    topk_group: int = 1
    routed_scale: float = 1.0
    norm_topk_prob: bool = True
    swiglu_limit: float = 0.0
    # formats
    expert_fmt: str = "bf16"         # bf16 | fp8 | mxfp4 | nvfp4
    dense_fmt: str = "bf16"          # bf16 | fp8 (attention / dense / shared / lm_head excluded)
    # misc
    num_mtp_layers: int = 0
    norm_eps: float = 1e-6
    norm_add_one: bool = False
    tie_embeddings: bool = False
    max_position: int = 131072
    extra: dict = field(default_factory=dict)

    # ----------------------------------------------------------------------
    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def rot_dim(self) -> int:
        if self.is_mla:
            return self.qk_rope_head_dim
        return self.rotary_dim if self.rotary_dim is not None else self.head_dim

    def layer_type(self, i: int) -> str:
        if self.layer_types is None:
            return "full"
        return self.layer_types[i]

    def kv_heads(self, i: int) -> int:
        """KV heads of GQA layer i."""
        if self.layer_type(i) == "swa" and self.swa_num_kv_heads:
            return self.swa_num_kv_heads
        return self.num_kv_heads

    @property
    def gqa_v_dim(self) -> int:
        return self.v_head_dim if (self.v_head_dim and not self.is_mla) else self.head_dim

    def window(self, i: int) -> int:
        return self.sliding_window if self.layer_type(i) == "swa" else 0

    def has_sinks(self, i: int) -> bool:
        k = self.layer_type(i)
        return self.attn_sinks == "all" or (self.attn_sinks == k and k in ("swa", "full"))

    def is_moe_layer(self, i: int) -> bool:
        return self.num_experts > 0 and i >= self.num_dense_layers

    def param_count(self, active: bool = False) -> int:
        """Approximate parameter count (all or active per token)."""
        H = self.hidden_size
        tot = self.vocab_size * H * (1 if self.tie_embeddings else 2)
        for i in range(self.num_layers + self.num_mtp_layers):
            li = min(i, self.num_layers - 1)
            if self.layer_type(li) == "linear" and self.linear_kind == "kda":
                kd = self.linear_num_key_heads * self.linear_key_head_dim
                vd = self.linear_num_value_heads * self.linear_value_head_dim
                dk = self.linear_key_head_dim
                tot += H * (2 * kd + vd + self.linear_num_value_heads) + vd * H
                tot += 2 * H * dk + dk * (self.linear_num_value_heads * dk + vd)
            elif self.layer_type(li) == "linear":
                kd = self.linear_num_key_heads * self.linear_key_head_dim
                vd = self.linear_num_value_heads * self.linear_value_head_dim
                tot += H * (2 * kd + 2 * vd + 2 * self.linear_num_value_heads) + vd * H
            elif self.is_mla:
                qd = self.num_heads * (self.qk_nope_head_dim + self.qk_rope_head_dim)
                tot += H * self.q_lora_rank + self.q_lora_rank * qd
                tot += H * (self.kv_lora_rank + self.qk_rope_head_dim)
                tot += self.kv_lora_rank * self.num_heads * (self.qk_nope_head_dim + self.v_head_dim)
                tot += self.num_heads * self.v_head_dim * H
            else:
                q = self.num_heads * self.head_dim * (2 if self.attn_output_gate else 1)
                kv = self.kv_heads(li) * (self.head_dim + self.gqa_v_dim)
                tot += H * (q + kv) + self.num_heads * self.gqa_v_dim * H
            if self.is_moe_layer(li):
                ne = self.top_k if active else self.num_experts
                tot += ne * 3 * H * self.moe_intermediate + H * self.num_experts
                tot += self.num_shared_experts * 3 * H * self.shared_intermediate
            else:
                tot += 3 * H * self.dense_intermediate
        return tot

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


# ---------------------------------------------------------------------------
# presets (the benchmarked configurations 1-5, plus the MiMo-V2 and Kimi-Linear families)
# ---------------------------------------------------------------------------
def tiny_mixtral() -> ModelConfig:
    """Config 1: 2 layers, hidden 256, 4 heads / 2 KV heads x 64, 8 experts top-2, I=512, vocab 1024."""
    return ModelConfig(name="tiny-mixtral", arch="mixtral", vocab_size=1024, hidden_size=256, num_layers=2,
                       num_heads=4, num_kv_heads=2, head_dim=64, rope_theta=1e4, num_experts=8, top_k=2,
                       moe_intermediate=512, scoring="softmax", norm_topk_prob=True, norm_eps=1e-5,
                       expert_fmt="bf16", max_position=4096)


def deepseek_v3_moe_layer() -> ModelConfig:
    """Config 2: one MoE layer, hidden 7168, 256 routed experts top-8 + 1 shared, I=2048, fp8-128."""
    return ModelConfig(name="dsv3-moe-layer", arch="deepseek_v3", vocab_size=129280, hidden_size=7168,
                       num_layers=1, num_heads=128, num_kv_heads=128, head_dim=128, num_experts=256, top_k=8,
                       moe_intermediate=2048, num_shared_experts=1, shared_intermediate=2048, scoring="sigmoid",
                       router_bias=True, n_group=8, topk_group=4, routed_scale=2.5, expert_fmt="fp8",
                       dense_fmt="fp8")


def qwen3_next_80b() -> ModelConfig:
    """Config 3: Qwen3-Next-style 80B-A3B: 48 layers, hidden 2048, 3 gated-DeltaNet : 1 gated GQA
    (16 q / 2 kv heads x 256), 512 experts top-10 + 1 shared, I=512, MXFP4 experts."""
    types = ["linear", "linear", "linear", "full"] * 12
    return ModelConfig(name="qwen3-next-80b-a3b", arch="qwen3_next", vocab_size=151936, hidden_size=2048,
                       num_layers=48, num_heads=16, num_kv_heads=2, head_dim=256, rope_theta=1e7,
                       rotary_dim=64, qk_norm=True, attn_output_gate=True, layer_types=types,
                       linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128,
                       linear_value_head_dim=128, linear_conv_kernel=4, num_experts=512, top_k=10,
                       moe_intermediate=512, num_shared_experts=1, shared_intermediate=512, shared_expert_gate=True,
                       scoring="softmax", norm_topk_prob=True, expert_fmt="mxfp4", dense_fmt="bf16",
                       norm_add_one=True, norm_eps=1e-6, max_position=262144, num_mtp_layers=1)


def glm45_air() -> ModelConfig:
    """Config 4: GLM-4.5-Air-style 106B-A12B: 46 layers, hidden 4096, GQA 96 q / 8 kv x 128, partial RoPE,
    128 experts top-8 + 1 shared, I=1408, first layer dense (I=10944), fp8-128, 1 MTP layer."""
    return ModelConfig(name="glm-4.5-air", arch="glm4_moe", vocab_size=151552, hidden_size=4096, num_layers=46,
                       num_heads=96, num_kv_heads=8, head_dim=128, rope_theta=1e6, rotary_dim=64, rope_neox=True,
                       qkv_bias=True, num_dense_layers=1, dense_intermediate=10944, num_experts=128, top_k=8,
                       moe_intermediate=1408, num_shared_experts=1, shared_intermediate=1408, scoring="sigmoid",
                       router_bias=True, n_group=1, topk_group=1, routed_scale=1.0, norm_topk_prob=True,
                       expert_fmt="fp8", dense_fmt="fp8", num_mtp_layers=1, norm_eps=1e-5, max_position=131072)


def deepseek_v3() -> ModelConfig:
    """Config 5: DeepSeek-V3 shape 671B-A37B: 61 layers (3 dense), hidden 7168, MLA 128 heads
    (q_lora 1536, kv_lora 512, rope 64), 256 experts top-8 + 1 shared, I=2048, fp8-128."""
    return ModelConfig(name="deepseek-v3", arch="deepseek_v3", vocab_size=129280, hidden_size=7168, num_layers=61,
                       num_heads=128, num_kv_heads=128, head_dim=192, rope_theta=10000.0,
                       rope_scaling={"type": "yarn", "factor": 40, "original_max_position_embeddings": 4096,
                                     "beta_fast": 32, "beta_slow": 1, "mscale": 1.0, "mscale_all_dim": 1.0},
                       rope_neox=False, q_lora_rank=1536, kv_lora_rank=512, qk_nope_head_dim=128,
                       qk_rope_head_dim=64, v_head_dim=128, num_dense_layers=3, dense_intermediate=18432,
                       num_experts=256, top_k=8, moe_intermediate=2048, num_shared_experts=1,
                       shared_intermediate=2048, scoring="sigmoid", router_bias=True, n_group=8, topk_group=4,
                       routed_scale=2.5, norm_topk_prob=True, expert_fmt="fp8", dense_fmt="fp8",
                       num_mtp_layers=1, max_position=163840)


def deepseek_v32() -> ModelConfig:
    """DeepSeek-V3.2-style sparse attention on the DeepSeek-V3 shape: the same MLA plus a
    lightning indexer (64 heads x 128, ReLU-gated, weighted over heads) that keeps the 2048
    best-scored context tokens of every query."""
    return deepseek_v3().replace(name="deepseek-v3.2", index_topk=2048, index_n_heads=64,
                                 index_head_dim=128)


def mimo_v2_flash() -> ModelConfig:
    """MiMo-V2-style hybrid-attention MoE (the shape the reference's MiMo guide lists): 48
    layers (1 dense + 47 MoE), hidden 4096, 9 global-attention layers (64 q / 4 kv heads) and
    39 sliding-window layers (window 128, 64 q / 8 kv heads, learned sinks), q/k heads 192
    wide with 64 rotary dims, v heads 128 wide; 256 experts top-8, I=2048, sigmoid router
    with correction bias, plain SwiGLU, MXFP4 experts, 3 MTP layers."""
    types = ["full" if (i == 0 or i % 6 == 5) else "swa" for i in range(48)]
    return ModelConfig(name="mimo-v2-flash", arch="mimo_v2", vocab_size=152576, hidden_size=4096, num_layers=48,
                       num_heads=64, num_kv_heads=4, head_dim=192, v_head_dim=128, rotary_dim=64,
                       rope_theta=5e6, layer_types=types, sliding_window=128, swa_num_kv_heads=8,
                       attn_sinks="swa", num_dense_layers=1, dense_intermediate=16384, num_experts=256, top_k=8,
                       moe_intermediate=2048, scoring="sigmoid", router_bias=True, n_group=1, topk_group=1,
                       norm_topk_prob=True, expert_fmt="mxfp4", dense_fmt="fp8", num_mtp_layers=3,
                       norm_eps=1e-5, max_position=262144)


def kimi_linear_48b() -> ModelConfig:
    """Kimi-Linear-style 48B-A3B hybrid: 27 layers, hidden 2304; Kimi Delta Attention layers
    (32 heads x 128, short conv 4, decay per key dim) with an MLA layer (32 heads, kv_lora 512,
    nope 128 + rope 64 dims used without rotary, v 128) at every fourth layer and the last;
    256 experts top-8 + 1 shared, I=1024, first layer dense (I=9216), sigmoid router with
    correction bias, bf16 weights."""
    types = ["full" if (i % 4 == 3 or i == 26) else "linear" for i in range(27)]
    return ModelConfig(name="kimi-linear-48b-a3b", arch="kimi_linear", vocab_size=163840, hidden_size=2304,
                       num_layers=27, num_heads=32, num_kv_heads=32, head_dim=192, q_lora_rank=0, kv_lora_rank=512,
                       qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128, mla_rope=False, rope_neox=False,
                       layer_types=types, linear_kind="kda", linear_num_key_heads=32, linear_num_value_heads=32,
                       linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel=4,
                       num_dense_layers=1, dense_intermediate=9216, num_experts=256, top_k=8, moe_intermediate=1024,
                       num_shared_experts=1, shared_intermediate=1024, scoring="sigmoid", router_bias=True,
                       n_group=1, topk_group=1, routed_scale=2.446, norm_topk_prob=True, expert_fmt="bf16",
                       dense_fmt="bf16", norm_eps=1e-5, max_position=1048576)


PRESETS = {
    "tiny-mixtral": tiny_mixtral,
    "dsv3-moe-layer": deepseek_v3_moe_layer,
    "qwen3-next-80b-a3b": qwen3_next_80b,
    "glm-4.5-air": glm45_air,
    "deepseek-v3": deepseek_v3,
    "deepseek-v3.2": deepseek_v32,
    "mimo-v2-flash": mimo_v2_flash,
    "kimi-linear-48b-a3b": kimi_linear_48b,
}


def get_preset(name: str, **overrides) -> ModelConfig:
    cfg = PRESETS[name]()
    return cfg.replace(**overrides) if overrides else cfg


def scaled_down(cfg: ModelConfig, layers: int = 2, hidden: int | None = None, experts: int | None = None,
                vocab: int = 512) -> ModelConfig:
    """A small member of the same family (tests): same structure, fewer/smaller pieces."""
    kw = dict(name=cfg.name + "-mini", num_layers=layers, vocab_size=vocab, max_position=4096,
              num_mtp_layers=min(cfg.num_mtp_layers, 1))
    if hidden is not None:
        kw["hidden_size"] = hidden
    if experts is not None:
        kw["num_experts"] = experts
        kw["top_k"] = min(cfg.top_k, experts)
        if cfg.n_group > 1:
            kw["n_group"] = min(cfg.n_group, experts // 2)
            kw["topk_group"] = max(1, min(cfg.topk_group, kw["n_group"] // 2))
            # the kept groups must hold at least top_k experts
            per_group = experts // kw["n_group"]
            kw["topk_group"] = min(kw["n_group"], max(kw["topk_group"], -(-kw["top_k"] // per_group)))
    if cfg.layer_types is not None:
        pat = cfg.layer_types[:4]
        kw["layer_types"] = (pat * ((layers + 3) // 4))[:layers]
    if cfg.num_dense_layers:
        kw["num_dense_layers"] = min(cfg.num_dense_layers, 1)
    return cfg.replace(**kw)


def from_hf_config(path_or_dict) -> ModelConfig:
    """Map a HF config.json (Mixtral / Glm4Moe / Qwen3Next / DeepseekV3 / MiMoV2 / KimiLinear) onto ModelConfig."""
    if isinstance(path_or_dict, (str, Path)):
        p = Path(path_or_dict)
        if p.is_dir():
            p = p / "config.json"
        hf = json.loads(p.read_text())
    else:
        hf = dict(path_or_dict)
    archs = hf.get("architectures", [""])[0]
    H = hf["hidden_size"]
    nh = hf["num_attention_heads"]
    base = dict(vocab_size=hf["vocab_size"], hidden_size=H, num_layers=hf["num_hidden_layers"], num_heads=nh,
                num_kv_heads=hf.get("num_key_value_heads", nh), head_dim=hf.get("head_dim", H // nh),
                rope_theta=float(hf.get("rope_theta", 10000.0)), rope_scaling=hf.get("rope_scaling"),
                norm_eps=hf.get("rms_norm_eps", 1e-6), tie_embeddings=hf.get("tie_word_embeddings", False),
                max_position=hf.get("max_position_embeddings", 131072))
    qc = hf.get("quantization_config") or {}
    fmt = "bf16"
    if qc.get("quant_method") == "fp8" or qc.get("fmt") == "e4m3":
        fmt = "fp8"
    elif qc.get("quant_method") in ("mxfp4",):
        fmt = "mxfp4"
    elif "nvfp4" in str(qc).lower():
        fmt = "nvfp4"
    if archs.startswith("Mixtral"):
        return ModelConfig(name="mixtral", arch="mixtral", num_experts=hf["num_local_experts"],
                           top_k=hf["num_experts_per_tok"], moe_intermediate=hf["intermediate_size"],
                           expert_fmt=fmt, **base)
    if archs.startswith("Glm4Moe"):
        return ModelConfig(name="glm4_moe", arch="glm4_moe",
                           rotary_dim=int(base["head_dim"] * hf.get("partial_rotary_factor", 0.5)),
                           qkv_bias=hf.get("attention_bias", True), qk_norm=hf.get("use_qk_norm", False),
                           num_dense_layers=hf.get("first_k_dense_replace", 1),
                           dense_intermediate=hf["intermediate_size"], num_experts=hf["n_routed_experts"],
                           top_k=hf["num_experts_per_tok"], moe_intermediate=hf["moe_intermediate_size"],
                           num_shared_experts=hf.get("n_shared_experts", 1),
                           shared_intermediate=hf["moe_intermediate_size"], scoring="sigmoid", router_bias=True,
                           n_group=hf.get("n_group", 1), topk_group=hf.get("topk_group", 1),
                           routed_scale=hf.get("routed_scaling_factor", 1.0),
                           norm_topk_prob=hf.get("norm_topk_prob", True), expert_fmt=fmt, dense_fmt=fmt,
                           num_mtp_layers=hf.get("num_nextn_predict_layers", 0), **base)
    if archs.startswith("Qwen3Next"):
        n = base["num_layers"]
        interval = hf.get("full_attention_interval", 4)
        types = ["full" if (i + 1) % interval == 0 else "linear" for i in range(n)]
        return ModelConfig(name="qwen3_next", arch="qwen3_next",
                           rotary_dim=int(base["head_dim"] * hf.get("partial_rotary_factor", 0.25)), qk_norm=True,
                           attn_output_gate=True, layer_types=types,
                           linear_num_key_heads=hf["linear_num_key_heads"],
                           linear_num_value_heads=hf["linear_num_value_heads"],
                           linear_key_head_dim=hf["linear_key_head_dim"],
                           linear_value_head_dim=hf["linear_value_head_dim"],
                           linear_conv_kernel=hf.get("linear_conv_kernel_dim", 4), num_experts=hf["num_experts"],
                           top_k=hf["num_experts_per_tok"], moe_intermediate=hf["moe_intermediate_size"],
                           num_shared_experts=1, shared_intermediate=hf["shared_expert_intermediate_size"],
                           shared_expert_gate=True, scoring="softmax", norm_topk_prob=hf.get("norm_topk_prob", True),
                           expert_fmt=fmt, norm_add_one=True,
                           num_mtp_layers=min(1, hf.get("mtp_num_hidden_layers", hf.get("num_nextn_predict_layers", 0))),
                           **base)
    if archs.startswith("MiMoV2"):
        # keys read: hybrid_layer_pattern (per layer, 1 = sliding window), sliding_window,
        # swa_num_key_value_heads, v_head_dim, partial_rotary_factor,
        # add_swa_attention_sink_bias / add_full_attention_sink_bias, n_routed_experts,
        # moe_intermediate_size, first_k_dense_replace, num_nextn_predict_layers
        n = base["num_layers"]
        pat = hf.get("hybrid_layer_pattern") or [0] * n
        types = ["swa" if int(pat[i]) == 1 else "full" for i in range(n)]
        sw, fl = hf.get("add_swa_attention_sink_bias", False), hf.get("add_full_attention_sink_bias", False)
        sinks = "all" if (sw and fl) else "swa" if sw else "full" if fl else ""
        return ModelConfig(name="mimo_v2", arch="mimo_v2", layer_types=types,
                           rotary_dim=int(base["head_dim"] * hf.get("partial_rotary_factor", 1.0)),
                           v_head_dim=hf.get("v_head_dim", base["head_dim"]),
                           sliding_window=hf.get("sliding_window", 0) or 0,
                           swa_num_kv_heads=hf.get("swa_num_key_value_heads", base["num_kv_heads"]),
                           attn_sinks=sinks, num_dense_layers=hf.get("first_k_dense_replace", 1),
                           dense_intermediate=hf["intermediate_size"], num_experts=hf["n_routed_experts"],
                           top_k=hf["num_experts_per_tok"], moe_intermediate=hf["moe_intermediate_size"],
                           scoring=hf.get("scoring_func", "sigmoid"), router_bias=True,
                           n_group=hf.get("n_group", 1), topk_group=hf.get("topk_group", 1),
                           routed_scale=hf.get("routed_scaling_factor", 1.0) or 1.0,
                           norm_topk_prob=hf.get("norm_topk_prob", True), expert_fmt=fmt, dense_fmt=fmt,
                           num_mtp_layers=hf.get("num_nextn_predict_layers", 0), **base)
    if archs.startswith("KimiLinear"):
        # keys read: linear_attn_config {full_attn_layers (1-based), num_heads, head_dim,
        # short_conv_kernel_size}, mla_use_nope, q_lora_rank, kv_lora_rank, qk_nope_head_dim,
        # qk_rope_head_dim, v_head_dim, num_experts, num_experts_per_token,
        # num_shared_experts, moe_intermediate_size, first_k_dense_replace, routed_scaling_factor
        n = base["num_layers"]
        la = hf.get("linear_attn_config") or {}
        full = {int(i) - 1 for i in la.get("full_attn_layers", [])}
        types = ["full" if i in full else "linear" for i in range(n)]
        nh_l, hd_l = la.get("num_heads", nh), la.get("head_dim", 128)
        base["head_dim"] = hf["qk_nope_head_dim"] + hf["qk_rope_head_dim"]
        return ModelConfig(name="kimi_linear", arch="kimi_linear", rope_neox=False,
                           q_lora_rank=hf.get("q_lora_rank") or 0, kv_lora_rank=hf["kv_lora_rank"],
                           qk_nope_head_dim=hf["qk_nope_head_dim"], qk_rope_head_dim=hf["qk_rope_head_dim"],
                           v_head_dim=hf["v_head_dim"], mla_rope=not hf.get("mla_use_nope", False),
                           layer_types=types, linear_kind="kda", linear_num_key_heads=nh_l,
                           linear_num_value_heads=nh_l, linear_key_head_dim=hd_l, linear_value_head_dim=hd_l,
                           linear_conv_kernel=la.get("short_conv_kernel_size", 4),
                           num_dense_layers=hf.get("first_k_dense_replace", 1),
                           dense_intermediate=hf["intermediate_size"],
                           num_experts=hf.get("num_experts", hf.get("n_routed_experts", 0)),
                           top_k=hf.get("num_experts_per_token", hf.get("num_experts_per_tok", 8)),
                           moe_intermediate=hf["moe_intermediate_size"],
                           num_shared_experts=hf.get("num_shared_experts", 1),
                           shared_intermediate=hf["moe_intermediate_size"], scoring="sigmoid", router_bias=True,
                           n_group=hf.get("num_expert_group", 1) or 1, topk_group=hf.get("topk_group", 1) or 1,
                           routed_scale=hf.get("routed_scaling_factor", 1.0) or 1.0,
                           norm_topk_prob=hf.get("moe_renormalize", True), expert_fmt=fmt, dense_fmt=fmt, **base)
    if archs.startswith("DeepseekV3"):
        base["head_dim"] = hf["qk_nope_head_dim"] + hf["qk_rope_head_dim"]
        return ModelConfig(name="deepseek_v3", arch="deepseek_v3", rope_neox=False, q_lora_rank=hf["q_lora_rank"],
                           kv_lora_rank=hf["kv_lora_rank"], qk_nope_head_dim=hf["qk_nope_head_dim"],
                           qk_rope_head_dim=hf["qk_rope_head_dim"], v_head_dim=hf["v_head_dim"],
                           num_dense_layers=hf.get("first_k_dense_replace", 3),
                           dense_intermediate=hf["intermediate_size"], num_experts=hf["n_routed_experts"],
                           top_k=hf["num_experts_per_tok"], moe_intermediate=hf["moe_intermediate_size"],
                           num_shared_experts=hf.get("n_shared_experts", 1),
                           shared_intermediate=hf["moe_intermediate_size"] * hf.get("n_shared_experts", 1),
                           scoring=hf.get("scoring_func", "sigmoid"), router_bias=True,
                           n_group=hf.get("n_group", 8), topk_group=hf.get("topk_group", 4),
                           routed_scale=hf.get("routed_scaling_factor", 2.5),
                           norm_topk_prob=hf.get("norm_topk_prob", True), expert_fmt=fmt, dense_fmt=fmt,
                           num_mtp_layers=hf.get("num_nextn_predict_layers", 0),
                           # DeepseekV32: the lightning indexer's width and how many tokens it keeps
                           index_topk=hf.get("index_topk", 0) or 0, index_n_heads=hf.get("index_n_heads", 64),
                           index_head_dim=hf.get("index_head_dim", 128), **base)
    raise ValueError(f"unsupported architecture {archs}")
