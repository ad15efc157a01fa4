"""Generic MoE decoder covering the Mixtral / GLM-4.5 / Qwen3-Next / DeepSeek-V3 families,
plus the seeded synthetic-weight factory used by the benchmarks and tests.

Forward contract (one engine step): token ids [T] and an :class:`AttnMetadata`
for the step's sequences -> final hidden states [T, H] (normed) ; ``logits``
maps selected rows to vocabulary scores.  KV caches / recurrent states are owned
by the engine and passed in per layer.
"""
from __future__ import annotations

import math

import torch

from ..ops import basic as B
from ..ops import gemm as G
from ..ops import moe as M
from ..ops.attention import AttnMetadata
from .config import ModelConfig
from .deltanet import DeltaNetState, GatedDeltaNet, KimiDeltaAttention
from .layers import DenseMLP, GQAAttention, Linear, MoEBlock, RMSNorm
from .mla import MLAAttention


class DecoderLayer:
    def __init__(self, idx: int, attn_norm: RMSNorm, attn, mlp_norm: RMSNorm, mlp, kind: str):
        self.idx, self.attn_norm, self.attn, self.mlp_norm, self.mlp, self.kind = idx, attn_norm, attn, mlp_norm, mlp, kind
        self.reduce = None      # tensor parallel: sums the ranks' partial outputs (parallel.tp)

    def __call__(self, x, residual, meta, kv, rope):
        if residual is None:
            h = self.attn_norm(x)
            residual = x
        else:
            h, residual = self.attn_norm(x, residual)
        h = self.attn(h, meta, kv, rope)
        if hasattr(h, "finish"):   # tensor parallel, fused: the partials are summed inside the norm
            h, residual = h.finish(residual, self.mlp_norm)
        else:
            if self.reduce is not None:
                h = self.reduce(h)
            h, residual = self.mlp_norm(h, residual)
        h = self.mlp(h)
        if self.reduce is not None:
            h = self.reduce(h)
        return h, residual

    def tensors(self):
        return self.attn_norm.tensors() + self.attn.tensors() + self.mlp_norm.tensors() + self.mlp.tensors()


class MTPLayer:
    """Multi-token-prediction module (GLM-4.5 / DeepSeek-V3 "nextn" layer):
    h' = Layer(eh_proj([enorm(embed(tok_{t+1})); hnorm(h_t)])) -> shared head."""

    def __init__(self, enorm: RMSNorm, hnorm: RMSNorm, eh_proj: Linear, layer: DecoderLayer, head_norm: RMSNorm):
        self.enorm, self.hnorm, self.eh_proj, self.layer, self.head_norm = enorm, hnorm, eh_proj, layer, head_norm

    def __call__(self, tok_emb, hidden, meta, kv, rope):
        e = self.enorm(tok_emb)
        h = self.hnorm(hidden)
        x = self.eh_proj(torch.cat([e, h], dim=-1))
        y, res = self.layer(x, None, meta, kv, rope)
        y, _ = self.head_norm(y, res)
        return y

    def tensors(self):
        return (self.enorm.tensors() + self.hnorm.tensors() + self.eh_proj.tensors() + self.layer.tensors() +
                self.head_norm.tensors())


class MoETransformer:
    def __init__(self, cfg: ModelConfig, embed: torch.Tensor, layers: list[DecoderLayer], norm: RMSNorm,
                 lm_head: torch.Tensor, mtp: list[MTPLayer] | None = None):
        self.cfg = cfg
        self.embed_tokens = embed
        self.layers = layers
        self.norm = norm
        self.lm_head = lm_head
        self.mtp = mtp or []
        self.device = lm_head.device
        self.act_dtype = torch.bfloat16   # fp32 allowed on CPU (exact-reference runs)
        self.tracer = None
        self.rope = B.rope_cache(cfg.rot_dim, min(cfg.max_position, 1 << 18), cfg.rope_theta, self.device,
                                 cfg.rope_scaling)
        self.wire_activation_forms()

    def wire_activation_forms(self) -> None:
        """Let each RMSNorm whose consumers are fp8-weight decode GEMVs also write their
        f16 x 2^-8 input rows (the GEMVs then skip their conversion pre-pass)."""
        def fp8_linear(lin) -> bool:
            return lin is not None and getattr(lin, "scale", None) is not None

        for l in list(self.layers) + [m.layer for m in self.mtp]:
            l.attn_norm.emit_f16s = fp8_linear(getattr(l.attn, "qkv", None))
            mlp = l.mlp
            if isinstance(mlp, MoEBlock):
                l.mlp_norm.emit_f16s = mlp.experts is not None and mlp.experts.fmt == "fp8"
            else:
                l.mlp_norm.emit_f16s = fp8_linear(getattr(mlp, "gate_up", None))

    def offload_embedding(self) -> int:
        """Keep the token-embedding table in pinned host memory instead of HBM (the rows a
        step needs are read over the host link by the lookup kernel), as the reference does
        for its large per-layer-embedding table (vllm_xiaotu_moe/ple_offload.py:176-267).
        Returns the device bytes freed.  Not for tied embeddings (the LM head reads it)."""
        if self.cfg.tie_embeddings or self.lm_head is self.embed_tokens:
            raise ValueError("tied embeddings are read by the LM head; keep them on the device")
        t = self.embed_tokens
        if not t.is_cuda:
            return 0
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        host.copy_(t)
        self.embed_tokens = host
        return t.numel() * t.element_size()

    # ------------------------------------------------------------------
    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        x = B.embed(ids, self.embed_tokens)
        return x if x.dtype == self.act_dtype else x.to(self.act_dtype)

    def forward(self, ids: torch.Tensor, meta: AttnMetadata, caches: list, return_prenorm: bool = False):
        x = self.embed(ids)
        residual = None
        tr = self.tracer
        for layer, kv in zip(self.layers, caches):
            if tr is None:
                x, residual = layer(x, residual, meta, kv, self.rope)
            else:
                with tr.layer(layer.idx):
                    x, residual = layer(x, residual, meta, kv, self.rope)
        h, pre = self.norm(x, residual)
        return (h, pre) if return_prenorm else h

    def attach_tracer(self, tracer) -> None:
        """Enable the observability hooks of ``utils.trace`` (routing dump, NVTX, timing)."""
        self.tracer = tracer
        for i, l in enumerate(self.layers):
            if isinstance(l.mlp, MoEBlock):
                l.mlp.tracer, l.mlp.trace_idx = tracer, i
        for j, m in enumerate(self.mtp):
            if isinstance(m.layer.mlp, MoEBlock):
                m.layer.mlp.tracer, m.layer.mlp.trace_idx = tracer, len(self.layers) + j

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        return G.linear(h, self.lm_head, out_dtype=torch.float32)

    def moe_blocks(self) -> list[MoEBlock]:
        return [l.mlp for l in self.layers if isinstance(l.mlp, MoEBlock)]

    def tensors(self):
        ts = [self.embed_tokens, self.lm_head] + self.norm.tensors()
        for l in self.layers:
            ts += l.tensors()
        for m in self.mtp:
            ts += m.tensors()
        seen, out = set(), []
        for t in ts:
            if t is not None and id(t) not in seen:
                seen.add(id(t))
                out.append(t)
        return out

    def to(self, device) -> "MoETransformer":
        """Copy every weight to `device` (returns a new model sharing nothing with self)."""
        import copy
        dev = torch.device(device)
        memo: dict[int, object] = {}

        def mv(o):
            if isinstance(o, torch.Tensor):
                if id(o) not in memo:
                    memo[id(o)] = o.to(dev)
                return memo[id(o)]
            if isinstance(o, (list, tuple)):
                return type(o)(mv(x) for x in o)
            if isinstance(o, dict):
                return {k: mv(v) for k, v in o.items()}
            if hasattr(o, "__dict__") and not isinstance(o, (type, torch.device)):
                if id(o) in memo:
                    return memo[id(o)]
                c = copy.copy(o)
                memo[id(o)] = c
                for k, v in vars(o).items():
                    setattr(c, k, mv(v))
                return c
            return o

        m = mv(self)
        m.device = dev
        for blk in m.moe_blocks():
            blk.ws = None
        for l in m.layers:
            if hasattr(l.mlp, "_seg"):
                l.mlp._seg = {}
            if hasattr(l.mlp, "shared") and l.mlp.shared is not None:
                l.mlp.shared._seg = {}
        return m

    def nbytes(self, device_only: bool = True) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors() if (t.is_cuda or not device_only))

    # KV cache / state allocation ---------------------------------------
    def kv_bytes_per_token(self, layers: range | None = None, skip_swa: bool = False, kv_dtype: str = "bf16") -> int:
        """KV bytes per token of context (skip_swa: leave out sliding-window layers, whose
        bounded pool does not grow with the context; kv_dtype "fp8": one byte per GQA value)."""
        c = self.cfg
        n = 0
        gqa_b = 1 if kv_dtype == "fp8" else 2
        for i in layers if layers is not None else range(c.num_layers):
            if c.layer_type(i) == "linear" or (skip_swa and c.layer_type(i) == "swa"):
                continue
            if c.is_mla:
                n += (c.kv_lora_rank + c.qk_rope_head_dim) * gqa_b + (c.index_head_dim * 2 if c.index_topk else 0)
            else:
                n += c.kv_heads(i) * (c.head_dim + c.gqa_v_dim) * gqa_b
        return n

    def _attn_cache(self, i: int, num_blocks: int, block_size: int, dtype, device, kv_dtype: str = "bf16"):
        """Paged KV cache of attention layer i: (K, V), or (latent, None) for MLA.  kv_dtype
        "fp8": e4m3 K [blocks, Hkv, bs, D] and V transposed per block [blocks, Hkv, Dv, bs]
        (GQA layers), e4m3 latent rows [blocks, 1, bs, kv_lora + rope] (MLA layers without
        sparse attention)."""
        c = self.cfg
        if kv_dtype not in ("bf16", "auto", "fp8"):
            raise ValueError(f"kv_cache_dtype {kv_dtype!r}: expected 'bf16' or 'fp8'")
        if c.is_mla:
            if kv_dtype == "fp8" and c.index_topk:
                raise NotImplementedError("fp8 latent cache with DeepSeek sparse attention")
            # DSA layers: the indexer's key cache rides in the second slot
            idx = (torch.zeros(num_blocks, 1, block_size, c.index_head_dim, dtype=torch.bfloat16, device=device)
                   if c.index_topk else None)
            ldt = torch.float8_e4m3fn if kv_dtype == "fp8" else torch.bfloat16
            return (torch.zeros(num_blocks, 1, block_size, c.kv_lora_rank + c.qk_rope_head_dim,
                                dtype=ldt, device=device), idx)
        nkv = c.kv_heads(i)
        if kv_dtype == "fp8":
            f8 = torch.float8_e4m3fn
            return (torch.zeros(num_blocks, nkv, block_size, c.head_dim, dtype=f8, device=device),
                    torch.zeros(num_blocks, nkv, c.gqa_v_dim, block_size, dtype=f8, device=device))
        if kv_dtype not in ("bf16", "auto"):
            raise ValueError(f"kv_cache_dtype {kv_dtype!r}: expected 'bf16' or 'fp8'")
        return (torch.zeros(num_blocks, nkv, block_size, c.head_dim, dtype=dtype, device=device),
                torch.zeros(num_blocks, nkv, block_size, c.gqa_v_dim, dtype=dtype, device=device))

    def allocate_caches(self, num_blocks: int, block_size: int, max_seqs: int, device=None,
                        layers: range | None = None, swa_blocks: int = 0, kv_dtype: str = "bf16") -> list:
        """Per layer: recurrent state, or a paged KV cache of num_blocks blocks
        (sliding-window layers: swa_blocks blocks when a bounded pool is used)."""
        c = self.cfg
        device = device or self.device
        caches = []
        for i in layers if layers is not None else range(c.num_layers):
            if c.layer_type(i) == "linear":
                caches.append(DeltaNetState(c, max_seqs, device))
            else:
                nb = swa_blocks if (swa_blocks > 0 and c.layer_type(i) == "swa") else num_blocks
                caches.append(self._attn_cache(i, nb, block_size, self.act_dtype, device, kv_dtype))
        return caches

    def allocate_mtp_caches(self, num_blocks: int, block_size: int, max_seqs: int, device=None,
                            kv_dtype: str = "bf16") -> list:
        device = device or self.device
        last = self.cfg.num_layers - 1      # an MTP layer has the last decoder layer's attention type
        return [self._attn_cache(last, num_blocks, block_size, torch.bfloat16, device, kv_dtype) for _ in self.mtp]

    def prepare_workspaces(self, max_tokens: int):
        """Allocate one MoE workspace shared by every MoE layer (they run one at a time)."""
        blocks = [b for b in self.moe_blocks() if b.experts is not None or b.executor is not None]
        if not blocks or not self.device.type == "cuda":
            return
        c = self.cfg
        ws = M.MoEWorkspace(max_tokens, c.top_k, c.num_experts, c.hidden_size, c.moe_intermediate, self.device)
        for b in self.moe_blocks():
            b.ws = ws
        return ws


# ===========================================================================
# synthetic weights
# ===========================================================================
class WeightFactory:
    """Seeded random-init weights, generated on the target device in the
    target format.  Each tensor's seed derives from (seed, name), so any tier
    (GPU, host, CPU engine) regenerates identical bytes independently."""

    def __init__(self, seed: int = 0, device="cpu", std: float = 0.02):
        self.seed, self.device, self.std = seed, torch.device(device), std

    def _gen(self, name: str):
        h = (hash_str(name) ^ (self.seed * 0x9E3779B97F4A7C15)) & 0x7FFFFFFFFFFFFFFF
        g = torch.Generator(device=self.device)
        g.manual_seed(h)
        return g

    def normal(self, name, shape, std=None, dtype=torch.bfloat16):
        g = self._gen(name)
        t = torch.randn(*shape, generator=g, device=self.device, dtype=torch.float32 if self.device.type == "cpu" else dtype)
        return (t * (std if std is not None else self.std)).to(dtype)

    def ones(self, shape, dtype=torch.bfloat16, name: str | None = None):
        return torch.ones(*shape, dtype=dtype, device=self.device)

    def zeros(self, shape, dtype=torch.bfloat16, name: str | None = None):
        return torch.zeros(*shape, dtype=dtype, device=self.device)

    def param(self, name: str, make, n: int):
        """A length-n tensor with a fixed synthetic value (``make(n)``); checkpoint sources load it by name."""
        return make(n)

    def linear(self, name, n, k, fmt="bf16", bias=False, std=None) -> Linear:
        std = std if std is not None else self.std
        if fmt == "bf16":
            w = self.normal(name, (n, k), std)
            return Linear(w, None, self.normal(name + ".bias", (n,), std) if bias else None)
        if fmt == "fp8":
            q, s = self.fp8(name, (n, k), std)
            return Linear(q, s, self.normal(name + ".bias", (n,), std) if bias else None)
        raise ValueError(fmt)

    def fp8(self, name, shape, std=None):
        """e4m3 codes ~ N(0, 8^2) with block scales std/8 (dequantised values ~ N(0, std^2))."""
        std = std if std is not None else self.std
        *lead, n, k = shape
        g = self._gen(name)
        dt = torch.float32 if self.device.type == "cpu" else torch.bfloat16
        q = (torch.randn(*shape, generator=g, device=self.device, dtype=dt) * 8.0).clamp(-448, 448)
        q = q.to(torch.float8_e4m3fn)
        s = torch.full((*lead, (n + 127) // 128, (k + 127) // 128), std / 8.0, dtype=torch.float32,
                       device=self.device)
        return q, s

    def experts(self, name, E, H, I, fmt) -> dict:
        """Checkpoint-layout routed experts: w13 [E, 2I, H] (gate rows then up rows), w2 [E, H, I]."""
        std = self.std
        if fmt == "bf16":
            return {"fmt": fmt, "w13": self.normal(name + ".w13", (E, 2 * I, H), std),
                    "w2": self.normal(name + ".w2", (E, H, I), std)}
        if fmt == "fp8":
            q13, s13 = self.fp8(name + ".w13", (E, 2 * I, H), std)
            q2, s2 = self.fp8(name + ".w2", (E, H, I), std)
            return {"fmt": fmt, "w13": q13, "s13": s13, "w2": q2, "s2": s2}
        if fmt == "mxfp4":
            return {"fmt": fmt, **self._fp4(name + ".w13", (E, 2 * I, H), 32, std, "13"),
                    **self._fp4(name + ".w2", (E, H, I), 32, std, "2")}
        if fmt == "nvfp4":
            return {"fmt": fmt, **self._fp4(name + ".w13", (E, 2 * I, H), 16, std, "13"),
                    **self._fp4(name + ".w2", (E, H, I), 16, std, "2")}
        raise ValueError(fmt)

    def _fp4(self, name, shape, group, std, suffix):
        """Random e2m1 codes with per-group scales giving values of roughly N(0, std^2)."""
        *lead, n, k = shape
        g = self._gen(name)
        packed = torch.randint(0, 256, (*lead, n, k // 2), generator=g, device=self.device, dtype=torch.uint8)
        if group == 32:  # e8m0: 2^(b-127); e2m1 magnitudes average ~2.5 -> scale ~ std / 2.5
            e = round(math.log2(std / 2.5)) + 127
            scales = torch.full((*lead, n, k // 32), e, dtype=torch.uint8, device=self.device)
            return {"w" + suffix: packed, "s" + suffix: scales}
        sc = torch.full((*lead, n, k // 16), 1.0, device=self.device).to(torch.float8_e4m3fn)
        gs = torch.full((lead[0] if lead else 1,), std / 2.5, dtype=torch.float32, device=self.device)
        return {"w" + suffix: packed, "s" + suffix: sc, "gs" + suffix: gs}


def hash_str(s: str) -> int:
    h = 1469598103934665603
    for ch in s.encode():
        h = ((h ^ ch) * 1099511628211) & 0xFFFFFFFFFFFFFFFF
    return h


def _norm(f: WeightFactory, cfg, shape, name: str, add_one=None):
    add = cfg.norm_add_one if add_one is None else add_one
    w = f.zeros(shape, name=name) if add else f.ones(shape, name=name)
    return RMSNorm(w, cfg.norm_eps, add)


def _dense_mlp(f: WeightFactory, name, H, I, fmt, limit=0.0) -> DenseMLP:
    inter = I % 128 == 0
    gu = f.linear(name + ".gate_up", 2 * I, H, fmt)
    if inter:
        if gu.scale is not None:
            gu = Linear(G.interleave_gate_up(gu.weight.view(torch.uint8)).view(torch.float8_e4m3fn),
                        G.interleave_gate_up_scale(gu.scale))
        else:
            gu = Linear(G.interleave_gate_up(gu.weight))
    return DenseMLP(gu, f.linear(name + ".down", H, I, fmt), inter, limit)


def _dsa_indexer(f, cfg: ModelConfig, name: str, H: int, dfmt: str):
    """The lightning indexer of a DSA (DeepSeek-V3.2-style) MLA layer, or None."""
    if not cfg.index_topk:
        return None
    if not cfg.q_lora_rank:
        raise ValueError("DSA needs the q latent (q_lora_rank > 0) for its index queries")
    from .mla import DSAIndexer
    ni, di = cfg.index_n_heads, cfg.index_head_dim
    return DSAIndexer(cfg, f.linear(name + ".idx_wq_b", ni * di, cfg.q_lora_rank, dfmt),
                      f.linear(name + ".idx_wk", di, H, dfmt), f.ones((di,), name=name + ".idx_k_norm_w"),
                      f.zeros((di,), name=name + ".idx_k_norm_b"), f.linear(name + ".idx_w", ni, H, "bf16"))


def build_layer(f: WeightFactory, cfg: ModelConfig, i: int, expert_sink=None, name_prefix="model.layers") -> DecoderLayer:
    H = cfg.hidden_size
    name = f"{name_prefix}.{i}"
    kind = cfg.layer_type(min(i, cfg.num_layers - 1))
    dfmt = cfg.dense_fmt
    if kind == "linear" and cfg.linear_kind == "kda":
        nk, nv, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        ch = 2 * nk * dk + nv * dv
        attn = KimiDeltaAttention(
            cfg, f.linear(name + ".kda_qkv", ch, H, dfmt), f.linear(name + ".kda_b", nv, H, "bf16"),
            f.linear(name + ".kda_f_a", dk, H, "bf16"), f.linear(name + ".kda_f_b", nv * dk, dk, "bf16"),
            f.linear(name + ".kda_g_a", dk, H, "bf16"), f.linear(name + ".kda_g_b", nv * dv, dk, "bf16"),
            f.normal(name + ".conv", (ch, cfg.linear_conv_kernel), 0.3),
            f.param(name + ".A_log", lambda n: torch.log(torch.linspace(1.0, 16.0, n, device=f.device)).float(), nv),
            f.param(name + ".dt_bias", lambda n: torch.zeros(n, device=f.device).float(), nv * dk),
            f.ones((dv,), name=name + ".gdn_norm"), f.linear(name + ".out", H, nv * dv, dfmt))
    elif kind == "linear":
        nk, nv, dk, dv = cfg.linear_num_key_heads, cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim
        ch = 2 * nk * dk + nv * dv
        attn = GatedDeltaNet(cfg, f.linear(name + ".qkvz", 2 * nk * dk + 2 * nv * dv, H, dfmt),
                             f.linear(name + ".ba", 2 * nv, H, "bf16"),
                             f.normal(name + ".conv", (ch, cfg.linear_conv_kernel), 0.3),
                             f.param(name + ".A_log", lambda n: torch.log(torch.linspace(1.0, 16.0, n,
                                                                                        device=f.device)).float(), nv),
                             f.param(name + ".dt_bias", lambda n: torch.zeros(n, device=f.device).float(), nv),
                             f.ones((dv,), name=name + ".gdn_norm"), f.linear(name + ".out", H, nv * dv, dfmt))
    elif cfg.is_mla:
        nh = cfg.num_heads
        q_a = f.linear(name + ".q_a", cfg.q_lora_rank, H, dfmt) if cfg.q_lora_rank else None
        attn = MLAAttention(cfg, q_a, f.ones((cfg.q_lora_rank,), name=name + ".q_a_norm") if q_a else None,
                            f.linear(name + ".q_b", nh * (cfg.qk_nope_head_dim + cfg.qk_rope_head_dim),
                                     cfg.q_lora_rank or H, dfmt),
                            f.linear(name + ".kv_a", cfg.kv_lora_rank + cfg.qk_rope_head_dim, H, dfmt),
                            f.ones((cfg.kv_lora_rank,), name=name + ".kv_a_norm"),
                            f.linear(name + ".kv_b", nh * (cfg.qk_nope_head_dim + cfg.v_head_dim), cfg.kv_lora_rank,
                                     dfmt),
                            f.linear(name + ".o", H, nh * cfg.v_head_dim, dfmt), _dsa_indexer(f, cfg, name, H, dfmt))
    else:
        li = min(i, cfg.num_layers - 1)
        nh, nkv, hd, vd = cfg.num_heads, cfg.kv_heads(li), cfg.head_dim, cfg.gqa_v_dim
        qdim = nh * hd * (2 if cfg.attn_output_gate else 1)
        qkn = (f.zeros if cfg.norm_add_one else f.ones) if cfg.qk_norm else None
        sinks = (f.param(name + ".sinks", lambda n: torch.linspace(-1.0, 1.0, n, device=f.device).float(), nh)
                 if cfg.has_sinks(li) else None)
        attn = GQAAttention(cfg, f.linear(name + ".qkv", qdim + nkv * (hd + vd), H, dfmt, bias=cfg.qkv_bias),
                            f.linear(name + ".o", H, nh * vd, dfmt),
                            qkn((hd,), name=name + ".q_norm") if qkn else None,
                            qkn((hd,), name=name + ".k_norm") if qkn else None,
                            num_kv_heads=nkv, window=cfg.window(li), sinks=sinks)
    if cfg.is_moe_layer(min(i, cfg.num_layers - 1)):
        E, I = cfg.num_experts, cfg.moe_intermediate
        gate = f.normal(name + ".router", (E, H), 0.02)
        bias = (f.normal(name + ".router_bias", (E,), 0.01, torch.float32)) if cfg.router_bias else None
        raw = f.experts(name + ".experts", E, H, I, cfg.expert_fmt)
        if expert_sink is not None:
            experts = expert_sink(i, raw)
        else:
            experts = M.prepare_experts(raw["fmt"], raw["w13"], raw["w2"], raw.get("s13"), raw.get("s2"),
                                        raw.get("gs13"), raw.get("gs2"))
        shared = None
        sgate = None
        if cfg.num_shared_experts:
            shared = _dense_mlp(f, name + ".shared", H, cfg.shared_intermediate * cfg.num_shared_experts, dfmt,
                                cfg.swiglu_limit)
            if cfg.shared_expert_gate:
                sgate = f.normal(name + ".shared_gate", (1, H), 0.02)
        mlp = MoEBlock(cfg, i, gate, bias, experts, shared, sgate)
    else:
        mlp = _dense_mlp(f, name + ".mlp", H, cfg.dense_intermediate, dfmt, cfg.swiglu_limit)
    return DecoderLayer(i, _norm(f, cfg, (H,), name + ".attn_norm"), attn, _norm(f, cfg, (H,), name + ".mlp_norm"),
                        mlp, kind)


def build_model(cfg: ModelConfig, device="cpu", seed: int = 0, expert_sink=None, std: float = 0.02,
                num_layers: int | None = None, source=None) -> MoETransformer:
    """Model in kernel layout, from seeded random init (default) or from ``source``
    (a checkpoint source with the factory's interface, see ``models.loader``).
    ``expert_sink(layer, raw)`` may take the routed experts elsewhere (CPU engine /
    host tier) and return what the MoE block should hold (None when no expert stays
    GPU-resident)."""
    f = source if source is not None else WeightFactory(seed, device, std)
    H = cfg.hidden_size
    n = cfg.num_layers if num_layers is None else num_layers
    embed = f.normal("model.embed", (cfg.vocab_size, H), 1.0)
    layers = [build_layer(f, cfg, i, expert_sink) for i in range(n)]
    lm_head = embed if cfg.tie_embeddings else f.normal("lm_head", (cfg.vocab_size, H), 0.02)
    mtp = []
    for j in range(cfg.num_mtp_layers):
        layer = build_layer(f, cfg, cfg.num_layers - 1, expert_sink, name_prefix=f"model.mtp{j}")
        mtp.append(MTPLayer(_norm(f, cfg, (H,), f"model.mtp{j}.enorm"), _norm(f, cfg, (H,), f"model.mtp{j}.hnorm"),
                            f.linear(f"mtp{j}.eh", H, 2 * H, cfg.dense_fmt), layer,
                            _norm(f, cfg, (H,), f"model.mtp{j}.head_norm")))
    return MoETransformer(cfg, embed, layers, _norm(f, cfg, (H,), "model.norm"), lm_head, mtp)
