"""HF safetensors checkpoints -> this framework's model (Mixtral, GLM-4.5, Qwen3-Next,
DeepSeek-V3 naming).

``CheckpointSource`` has the interface of the synthetic ``WeightFactory``
(``linear / normal / ones / zeros / param / experts``), so ``build_model(cfg,
source=...)`` builds the same model from real weights.  Internal tensor names
(``model.layers.{i}.qkv``, ``.router``, ``.experts`` ...) are translated to the HF
names of the model family; fused internal tensors are concatenations of HF tensors
(q|k|v -> qkv, gate|up -> gate_up, per-expert gate|up -> w13 [E, 2I, H]).

Formats, per HF linear prefix ``p``:
  * bf16 / fp16 / fp32: ``p.weight``;
  * fp8 e4m3 with 128x128 block scales: ``p.weight`` + ``p.weight_scale_inv`` (fp32);
  * MXFP4: ``p.weight`` (u8, two e2m1 per byte, low nibble = even k) + ``p.weight_scale``
    (u8 e8m0 per 32);
  * NVFP4: ``p.weight`` (u8) + ``p.weight_scale`` (e4m3 per 16) + ``p.weight_scale_2``
    (fp32 global).  1-byte scale tensors are taken bit for bit (never value-converted;
    the reference's loader makes the same point, hybrid_model.py:699-709).
Tensors come from the mmap'd files as zero-copy views; experts are stacked one layer
at a time and handed to the expert sink (CPU engine shards / GPU) right away.
"""
from __future__ import annotations

import re

import torch

from ..ops import gemm as G
from ..ops.quant import dequant_fp8_block, dequant_gptq, gptq_to_int4_rows, quant_fp8_block
from ..utils.safetensors import CheckpointDir
from .config import ModelConfig, from_hf_config
from .layers import Linear


def _family_names(cfg: ModelConfig) -> dict:
    a = cfg.arch
    if a == "mixtral":
        return dict(moe="block_sparse_moe", router="block_sparse_moe.gate", gate="w1", up="w3", down="w2",
                    experts="block_sparse_moe.experts", shared=None)
    if a == "qwen3_next":
        return dict(moe="mlp", router="mlp.gate", gate="gate_proj", up="up_proj", down="down_proj",
                    experts="mlp.experts", shared="mlp.shared_expert", shared_gate="mlp.shared_expert_gate")
    return dict(moe="mlp", router="mlp.gate", gate="gate_proj", up="up_proj", down="down_proj",
                experts="mlp.experts", shared="mlp.shared_experts", shared_gate=None)


class CheckpointSource:
    def __init__(self, path, cfg: ModelConfig | None = None, device="cpu"):
        self.ckpt = CheckpointDir(path)
        self.cfg = cfg or from_hf_config(path)
        self.device = torch.device(device)
        self.fam = _family_names(self.cfg)
        self.used: set[str] = set()
        self.gptq_bits, self.gptq_zero_offset = self._gptq_format(path)

    @staticmethod
    def _gptq_format(path) -> tuple[int, int]:
        """(bits, zero-point offset) from config.json's quantization_config (GPTQ defaults:
        4 bits, "gptq" format whose packed zero points are stored minus one)."""
        import json
        import os
        qc = {}
        cj = os.path.join(str(path), "config.json")
        if os.path.isfile(cj):
            with open(cj) as fh:
                qc = json.load(fh).get("quantization_config") or {}
        method = qc.get("quant_method", "gptq")
        if method not in ("gptq", "fp8", "mxfp4", "modelopt", "compressed-tensors", None):
            raise ValueError(f"quantization method {method!r} is not supported")
        bits = int(qc.get("bits", 4)) if method == "gptq" else 4
        fmt = qc.get("checkpoint_format", "gptq") if method == "gptq" else "gptq"
        if fmt not in ("gptq", "gptq_v2"):
            raise ValueError(f"GPTQ checkpoint format {fmt!r} is not supported (gptq, gptq_v2)")
        if bits not in (2, 4, 8):
            raise ValueError(f"GPTQ with {bits}-bit weights is not supported (2, 4 or 8)")
        return bits, (1 if fmt == "gptq" else 0)

    # ------------------------------------------------------------------ name mapping
    def _layer_prefix(self, name: str) -> tuple[str, str]:
        """internal 'model.layers.{i}.rest' / 'model.mtp{j}.{i}.rest' -> ('model.layers.{k}', 'rest')."""
        m = re.match(r"model\.layers\.(\d+)\.(.+)$", name)
        if m:
            return f"model.layers.{m.group(1)}", m.group(2)
        # MTP layers: GLM / DeepSeek number them after the decoder layers; Qwen3-Next keeps
        # them under "mtp.layers.{j}"
        qn = self.cfg.arch == "qwen3_next"
        m = re.match(r"model\.mtp(\d+)\.(\d+)\.(.+)$", name)
        if m:
            j = int(m.group(1))
            return (f"mtp.layers.{j}" if qn else f"model.layers.{self.cfg.num_layers + j}"), m.group(3)
        m = re.match(r"model\.mtp(\d+)\.(.+)$", name)
        if m:
            j = int(m.group(1))
            return (f"mtp.layers.{j}" if qn else f"model.layers.{self.cfg.num_layers + j}"), m.group(2)
        raise KeyError(name)

    def _hf(self, name: str) -> list[str]:
        """HF prefixes (or full tensor names) whose concatenation is the internal tensor."""
        c, f = self.cfg, self.fam
        fixed = {"model.embed": ["model.embed_tokens.weight"], "lm_head": ["lm_head.weight"],
                 "model.norm": ["model.norm.weight"]}
        if name in fixed:
            return fixed[name]
        m = re.match(r"mtp(\d+)\.eh$", name)
        if m:
            return ["mtp.fc"] if c.arch == "qwen3_next" else [f"model.layers.{c.num_layers + int(m.group(1))}.eh_proj"]
        if c.arch == "qwen3_next":      # the MTP module's own norms (one MTP layer)
            m = re.match(r"model\.mtp\d+\.(enorm|hnorm|head_norm)$", name)
            if m:
                return [{"enorm": "mtp.pre_fc_norm_embedding.weight", "hnorm": "mtp.pre_fc_norm_hidden.weight",
                         "head_norm": "mtp.norm.weight"}[m.group(1)]]
        pre, rest = self._layer_prefix(name)
        sa = "self_attn"
        table = {
            "attn_norm": [f"{pre}.input_layernorm.weight"], "mlp_norm": [f"{pre}.post_attention_layernorm.weight"],
            "enorm": [f"{pre}.enorm.weight"], "hnorm": [f"{pre}.hnorm.weight"],
            "head_norm": [f"{pre}.shared_head.norm.weight"],
            "qkv": [f"{pre}.{sa}.q_proj", f"{pre}.{sa}.k_proj", f"{pre}.{sa}.v_proj"],
            "o": [f"{pre}.{sa}.o_proj"], "q_norm": [f"{pre}.{sa}.q_norm.weight"],
            "k_norm": [f"{pre}.{sa}.k_norm.weight"], "sinks": [f"{pre}.{sa}.attention_sink_bias"],
            "q_a": [f"{pre}.{sa}.q_a_proj"], "q_a_norm": [f"{pre}.{sa}.q_a_layernorm.weight"],
            "q_b": [f"{pre}.{sa}.q_b_proj" if c.q_lora_rank else f"{pre}.{sa}.q_proj"],
            "kv_a": [f"{pre}.{sa}.kv_a_proj_with_mqa"], "kv_a_norm": [f"{pre}.{sa}.kv_a_layernorm.weight"],
            "kv_b": [f"{pre}.{sa}.kv_b_proj"],
            "qkvz": [f"{pre}.linear_attn.in_proj_qkvz"], "ba": [f"{pre}.linear_attn.in_proj_ba"],
            "conv": [f"{pre}.linear_attn.conv1d.weight"], "A_log": [f"{pre}.linear_attn.A_log"],
            "dt_bias": [f"{pre}.linear_attn.dt_bias"], "gdn_norm": [f"{pre}.linear_attn.norm.weight"],
            "out": [f"{pre}.linear_attn.out_proj"],
            "router": [f"{pre}.{f['router']}.weight"],
            "router_bias": [f"{pre}.{f['router']}.e_score_correction_bias"],
            "mlp.gate_up": [f"{pre}.mlp.gate_proj", f"{pre}.mlp.up_proj"], "mlp.down": [f"{pre}.mlp.down_proj"],
        }
        if c.linear_kind == "kda":
            # Kimi Delta Attention: separate q/k/v projections and convs, low-rank decay and gate
            table.update({
                "kda_qkv": [f"{pre}.{sa}.q_proj", f"{pre}.{sa}.k_proj", f"{pre}.{sa}.v_proj"],
                "kda_b": [f"{pre}.{sa}.b_proj"], "kda_f_a": [f"{pre}.{sa}.f_a_proj"],
                "kda_f_b": [f"{pre}.{sa}.f_b_proj"], "kda_g_a": [f"{pre}.{sa}.g_a_proj"],
                "kda_g_b": [f"{pre}.{sa}.g_b_proj"],
                "conv": [f"{pre}.{sa}.q_conv1d.weight", f"{pre}.{sa}.k_conv1d.weight",
                         f"{pre}.{sa}.v_conv1d.weight"],
                "A_log": [f"{pre}.{sa}.A_log"], "dt_bias": [f"{pre}.{sa}.dt_bias"],
                "gdn_norm": [f"{pre}.{sa}.o_norm.weight"], "out": [f"{pre}.{sa}.o_proj"]})
        if c.index_topk:         # DSA lightning indexer (DeepSeek-V3.2 names)
            ix = f"{pre}.{sa}.indexer"
            table.update({"idx_wq_b": [f"{ix}.wq_b"], "idx_wk": [f"{ix}.wk"], "idx_w": [f"{ix}.weights_proj"],
                          "idx_k_norm_w": [f"{ix}.k_norm.weight"], "idx_k_norm_b": [f"{ix}.k_norm.bias"]})
        if f.get("shared"):
            table["shared.gate_up"] = [f"{pre}.{f['shared']}.gate_proj", f"{pre}.{f['shared']}.up_proj"]
            table["shared.down"] = [f"{pre}.{f['shared']}.down_proj"]
        if f.get("shared_gate"):
            table["shared_gate"] = [f"{pre}.{f['shared_gate']}.weight"]
        if rest.endswith(".bias") and rest[:-5] in table:
            return [p + ".bias" for p in table[rest[:-5]]]
        if rest not in table:
            raise KeyError(f"no checkpoint mapping for {name}")
        return table[rest]

    def _get(self, hf_name: str) -> torch.Tensor:
        self.used.add(hf_name)
        return self.ckpt.get(hf_name)

    # ------------------------------------------------------------------ factory interface
    def normal(self, name, shape, std=None, dtype=torch.bfloat16):
        parts = self._hf(name)
        ts = [self._get(p_) for p_ in parts]
        t = torch.cat(ts, 0) if len(ts) > 1 else ts[0]       # KDA: q / k / v convs, channel order
        if name.endswith(".conv") and t.dim() == 3:          # conv1d weight [ch, 1, k]
            t = t[:, 0, :]
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name}: checkpoint shape {tuple(t.shape)} != {tuple(shape)}")
        return t.to(device=self.device, dtype=dtype, copy=True)

    def ones(self, shape, dtype=torch.bfloat16, name: str | None = None):
        return self._get(self._hf(name)[0]).to(device=self.device, dtype=dtype, copy=True).view(*shape)

    zeros = ones

    def param(self, name: str, make, n: int):
        ref = make(n)
        t = self._get(self._hf(name)[0])       # any shape with n elements (KDA keeps A_log [1, 1, nv, 1])
        return t.to(device=self.device, dtype=ref.dtype, copy=True).reshape(ref.shape)

    def _gptq_int4_experts(self, base: str, E: int) -> dict | None:
        """The layer's GPTQ experts as INT4 rows (None when any projection is not in that form)."""
        f = self.fam
        opt = lambda p, n: self._get(p + n) if (p + n) in self.ckpt else None

        def rows(prefix):
            return gptq_to_int4_rows(self._get(prefix + ".qweight"), self._get(prefix + ".scales"),
                                     opt(prefix, ".qzeros"), opt(prefix, ".g_idx"), self.gptq_zero_offset)
        w13, s13, w2, s2 = [], [], [], []
        for e in range(E):
            g, u, d = (rows(f"{base}.{e}.{f[k]}") for k in ("gate", "up", "down"))
            if g is None or u is None or d is None:
                return None
            w13.append(torch.cat([g[0], u[0]], 0))
            s13.append(torch.cat([g[1], u[1]], 0))
            w2.append(d[0])
            s2.append(d[1])
        return {"fmt": "int4", "w13": torch.stack(w13), "w2": torch.stack(w2), "s13": torch.stack(s13),
                "s2": torch.stack(s2)}

    def _gptq(self, prefix: str) -> torch.Tensor:
        """A GPTQ-quantized projection, dequantized to fp32 [out, in]."""
        opt = lambda k: self._get(prefix + k) if (prefix + k) in self.ckpt else None
        return dequant_gptq(self._get(prefix + ".qweight"), self._get(prefix + ".scales"), opt(".qzeros"),
                            opt(".g_idx"), bits=self.gptq_bits, zero_offset=self.gptq_zero_offset)

    def _dense_part(self, prefix: str) -> torch.Tensor:
        """A non-GPTQ part of a fused projection, as fp32 [out, in] (fp8 parts with their scales)."""
        w = self._get(prefix + ".weight")
        if w.dtype == torch.float8_e4m3fn:
            return dequant_fp8_block(w, self._get(prefix + ".weight_scale_inv").float())
        return w.float()

    def linear(self, name, n, k, fmt="bf16", bias=False, std=None) -> Linear:
        parts = self._hf(name)
        if any((p + ".qweight") in self.ckpt for p in parts):   # GPTQ INT4: dequantized, then this layer's format
            w = torch.cat([self._gptq(p) if (p + ".qweight") in self.ckpt else self._dense_part(p)
                           for p in parts], 0)
            if tuple(w.shape) != (n, k):
                raise ValueError(f"{name}: checkpoint shape {tuple(w.shape)} != {(n, k)}")
            b = torch.cat([self._get(p + ".bias") for p in parts], 0) if bias else None
            if fmt == "fp8":
                q, sc = quant_fp8_block(w)
                return Linear(q.to(self.device), sc.to(self.device),
                              None if b is None else b.to(device=self.device, dtype=torch.bfloat16))
            return Linear(w.to(device=self.device, dtype=torch.bfloat16), None,
                          None if b is None else b.to(device=self.device, dtype=torch.bfloat16))
        ws = [self._get(p + ".weight") for p in parts]
        w = torch.cat(ws, 0) if len(ws) > 1 else ws[0]
        scale = None
        if w.dtype == torch.float8_e4m3fn:
            ss = [self._get(p + ".weight_scale_inv").float() for p in parts]
            if all(x.shape[0] % 128 == 0 for x in ws[:-1]):
                scale = torch.cat(ss, 0) if len(ss) > 1 else ss[0]
            else:   # part boundaries inside a 128-row scale block: widen and re-block
                deq = torch.cat([dequant_fp8_block(x, s_) for x, s_ in zip(ws, ss)], 0)
                w, scale = quant_fp8_block(deq)
        elif w.dtype != torch.bfloat16:
            w = w.to(torch.bfloat16)
        if tuple(w.shape) != (n, k):
            raise ValueError(f"{name}: checkpoint shape {tuple(w.shape)} != {(n, k)}")
        b = None
        if bias:
            bs = [self._get(p + ".bias") for p in parts]
            b = torch.cat(bs, 0).to(torch.bfloat16)
        d = self.device        # copies: the model must not alias the checkpoint mapping
        return Linear(w.to(d, copy=True), None if scale is None else scale.to(d, copy=True),
                      None if b is None else b.to(d, copy=True))

    def experts(self, name, E, H, I, fmt) -> dict:
        pre, _ = self._layer_prefix(name)
        f = self.fam
        base = f"{pre}.{f['experts']}"
        if f"{base}.0.{f['gate']}.qweight" in self.ckpt:
            # GPTQ INT4 experts: kept at 4 bits ("int4": the CPU tier's format; GPU-resident
            # experts dequantize it when prepared) when the layer is 4-bit, 128-grouped, in
            # input order; else dequantized, then held as fp8-128 or bf16 per the model's format
            rows = self._gptq_int4_experts(base, E) if self.gptq_bits == 4 else None
            if rows is not None:
                return rows
            w13 = torch.stack([torch.cat([self._gptq(f"{base}.{e}.{f['gate']}"),
                                          self._gptq(f"{base}.{e}.{f['up']}")], 0) for e in range(E)])
            w2 = torch.stack([self._gptq(f"{base}.{e}.{f['down']}") for e in range(E)])
            if fmt == "fp8":
                q13, s13 = quant_fp8_block(w13)
                q2, s2 = quant_fp8_block(w2)
                return {"fmt": "fp8", "w13": q13, "w2": q2, "s13": s13, "s2": s2}
            return {"fmt": "bf16", "w13": w13.to(torch.bfloat16), "w2": w2.to(torch.bfloat16)}
        g0 = self.ckpt.get(f"{base}.0.{f['gate']}.weight")
        if g0.dtype == torch.uint8:
            fmt = "nvfp4" if f"{base}.0.{f['gate']}.weight_scale_2" in self.ckpt else "mxfp4"
        elif g0.dtype == torch.float8_e4m3fn:
            fmt = "fp8"
        else:
            fmt = "bf16"

        def stack(proj_list, suffix):
            rows = []
            for e in range(E):
                ts = [self._get(f"{base}.{e}.{f[pj]}.{suffix}") for pj in proj_list]
                rows.append(torch.cat(ts, 0) if len(ts) > 1 else ts[0])
            return torch.stack(rows)

        out = {"fmt": fmt, "w13": stack(["gate", "up"], "weight"), "w2": stack(["down"], "weight")}
        if fmt == "fp8":
            out["s13"] = stack(["gate", "up"], "weight_scale_inv").float()
            out["s2"] = stack(["down"], "weight_scale_inv").float()
        elif fmt in ("mxfp4", "nvfp4"):
            out["s13"] = stack(["gate", "up"], "weight_scale").view(torch.uint8)
            out["s2"] = stack(["down"], "weight_scale").view(torch.uint8)
            if fmt == "nvfp4":
                out["s13"] = out["s13"].view(torch.float8_e4m3fn)
                out["s2"] = out["s2"].view(torch.float8_e4m3fn)
                g = torch.tensor([[float(self._get(f"{base}.{e}.{f[pj]}.weight_scale_2"))
                                   for pj in ("gate", "up")] for e in range(E)])
                out["s13"] = _fold_nvfp4_halves(out["s13"], g, I)
                out["gs13"] = g.max(1).values
                out["gs2"] = torch.tensor([float(self._get(f"{base}.{e}.{f['down']}.weight_scale_2"))
                                           for e in range(E)])
        for k in ("w13", "w2", "s13", "s2"):
            if k in out and fmt in ("bf16", "fp8") and self.device.type == "cuda":
                pass   # the sink / prepare_experts moves what stays on the GPU
        return out

    def close(self):
        self.ckpt.close()


def _fold_nvfp4_halves(s13: torch.Tensor, g: torch.Tensor, I: int) -> torch.Tensor:
    """One global scale per expert: the half whose global scale is smaller gets its e4m3
    group scales multiplied by (its scale / the larger one) (exact when the ratio is a
    power of two, else rounded to e4m3)."""
    gmax = g.max(1).values
    if torch.all(g[:, 0] == g[:, 1]):
        return s13
    s = s13.float().clone()
    for half in (0, 1):
        r = (g[:, half] / gmax).view(-1, 1, 1)
        sl = slice(0, I) if half == 0 else slice(I, 2 * I)
        s[:, sl] = s[:, sl] * r
    return s.to(torch.float8_e4m3fn)


def load_model(path, device="cuda", expert_sink=None, cfg: ModelConfig | None = None):
    """Build a model from an HF checkpoint directory (config.json + *.safetensors)."""
    from .model import build_model
    src = CheckpointSource(path, cfg, device)
    m = build_model(src.cfg, device=device, expert_sink=expert_sink, source=src)
    return m, src


# ---------------------------------------------------------------------------- export (tests, tooling)
def export_hf(model, cfg: ModelConfig, path) -> None:
    """Write a model built by this framework as an HF-style checkpoint of cfg's family
    (inverse of CheckpointSource; used to test the name mapping and for tooling)."""
    from ..utils.safetensors import save_file
    from .layers import DenseMLP, GQAAttention, MoEBlock
    from .mla import MLAAttention
    from .deltanet import GatedDeltaNet, KimiDeltaAttention
    src = CheckpointSource.__new__(CheckpointSource)
    src.cfg, src.fam = cfg, _family_names(cfg)
    out: dict[str, torch.Tensor] = {}

    def put_linear(internal: str, lin: Linear, split: list[int] | None = None, gate_up_inter=False):
        w, s = lin.weight.cpu(), None if lin.scale is None else lin.scale.cpu()
        if gate_up_inter:
            w = _deinterleave(w)
            s = None if s is None else _deinterleave_scale(s)
        parts = src._hf(internal)
        split = split or [w.shape[0]]
        r0 = 0
        for p, n in zip(parts, split):
            out[p + ".weight"] = w[r0:r0 + n].clone()
            if s is not None:
                out[p + ".weight_scale_inv"] = s[r0 // 128:(r0 + n + 127) // 128].clone()
            if lin.bias is not None:
                out[p + ".bias"] = lin.bias.cpu()[r0:r0 + n].clone()
            r0 += n

    def put(internal: str, t: torch.Tensor):
        out[src._hf(internal)[0]] = t.detach().cpu().clone()

    put("model.embed", model.embed_tokens)
    if not cfg.tie_embeddings:
        put("lm_head", model.lm_head)
    put("model.norm", model.norm.weight)
    layer_list = [(f"model.layers.{i}", l) for i, l in enumerate(model.layers)]
    layer_list += [(f"model.mtp{j}.{cfg.num_layers - 1}", m.layer) for j, m in enumerate(model.mtp)]
    for name, l in layer_list:
        put(name + ".attn_norm", l.attn_norm.weight)
        put(name + ".mlp_norm", l.mlp_norm.weight)
        a = l.attn
        if isinstance(a, GQAAttention):
            qd = cfg.num_heads * cfg.head_dim * (2 if cfg.attn_output_gate else 1)
            put_linear(name + ".qkv", a.qkv, [qd, a.nkv * a.hd, a.nkv * a.vd])
            put_linear(name + ".o", a.o)
            if a.q_norm is not None:
                put(name + ".q_norm", a.q_norm)
                put(name + ".k_norm", a.k_norm)
            if a.sinks is not None:
                put(name + ".sinks", a.sinks)
        elif isinstance(a, MLAAttention):
            if a.q_a is not None:
                put_linear(name + ".q_a", a.q_a)
                put(name + ".q_a_norm", a.q_a_norm)
            put_linear(name + ".q_b", a.q_b)
            put_linear(name + ".kv_a", a.kv_a)
            put(name + ".kv_a_norm", a.kv_a_norm)
            put_linear(name + ".kv_b", a.kv_b)
            put_linear(name + ".o", a.o)
            if a.indexer is not None:
                ix = a.indexer
                put_linear(name + ".idx_wq_b", ix.wq_b)
                put_linear(name + ".idx_wk", ix.wk)
                put_linear(name + ".idx_w", ix.weights_proj)
                put(name + ".idx_k_norm_w", ix.k_norm_w)
                put(name + ".idx_k_norm_b", ix.k_norm_b)
        elif isinstance(a, KimiDeltaAttention):
            kd, vd = a.nk * a.dk, a.nv * a.dv
            put_linear(name + ".kda_qkv", a.in_qkv, [kd, kd, vd])
            for suf, lin in (("kda_b", a.in_b), ("kda_f_a", a.f_a), ("kda_f_b", a.f_b), ("kda_g_a", a.g_a),
                             ("kda_g_b", a.g_b), ("out", a.out)):
                put_linear(name + "." + suf, lin)
            cw = a.conv_w.detach().cpu().unsqueeze(1)
            for p_, (r0, n_) in zip(src._hf(name + ".conv"), ((0, kd), (kd, kd), (2 * kd, vd))):
                out[p_] = cw[r0:r0 + n_].clone()
            put(name + ".A_log", a.A_log)
            put(name + ".dt_bias", a.dt_bias)
            put(name + ".gdn_norm", a.norm_w)
        elif isinstance(a, GatedDeltaNet):
            put_linear(name + ".qkvz", a.in_qkvz)
            put_linear(name + ".ba", a.in_ba)
            out[src._hf(name + ".conv")[0]] = a.conv_w.detach().cpu().unsqueeze(1).clone()
            put(name + ".A_log", a.A_log)
            put(name + ".dt_bias", a.dt_bias)
            put(name + ".gdn_norm", a.norm_w)
            put_linear(name + ".out", a.out)
        mlp = l.mlp
        if isinstance(mlp, DenseMLP):
            I = mlp.down.weight.shape[1]
            put_linear(name + ".mlp.gate_up", mlp.gate_up, [I, I], gate_up_inter=mlp.interleaved)
            put_linear(name + ".mlp.down", mlp.down)
        elif isinstance(mlp, MoEBlock):
            put(name + ".router", mlp.gate)
            if mlp.gate_bias is not None:
                put(name + ".router_bias", mlp.gate_bias)
            ex = mlp.experts
            pre, _ = src._layer_prefix(name + ".experts")
            base = f"{pre}.{src.fam['experts']}"
            fam = src.fam
            for e in range(ex.num_experts):
                w13, w2 = ex.w13[e].cpu(), ex.w2[e].cpu()
                s13 = None if ex.s13 is None else ex.s13[e].cpu()
                if ex.interleaved:
                    w13 = _deinterleave(w13)
                    if s13 is not None and ex.fmt in ("mxfp4", "nvfp4"):      # per-row scales
                        s13 = _deinterleave(s13.view(torch.uint8)).view(s13.dtype)
                    elif s13 is not None:
                        s13 = _deinterleave_scale(s13)
                I = w13.shape[0] // 2
                out[f"{base}.{e}.{fam['gate']}.weight"] = w13[:I].clone()
                out[f"{base}.{e}.{fam['up']}.weight"] = w13[I:].clone()
                out[f"{base}.{e}.{fam['down']}.weight"] = w2.clone()
                if ex.fmt == "fp8":
                    out[f"{base}.{e}.{fam['gate']}.weight_scale_inv"] = s13[:I // 128].clone()
                    out[f"{base}.{e}.{fam['up']}.weight_scale_inv"] = s13[I // 128:].clone()
                    out[f"{base}.{e}.{fam['down']}.weight_scale_inv"] = ex.s2[e].cpu().clone()
                elif ex.fmt in ("mxfp4", "nvfp4"):
                    out[f"{base}.{e}.{fam['gate']}.weight_scale"] = s13[:I].clone()
                    out[f"{base}.{e}.{fam['up']}.weight_scale"] = s13[I:].clone()
                    out[f"{base}.{e}.{fam['down']}.weight_scale"] = ex.s2[e].cpu().clone()
                    if ex.fmt == "nvfp4":
                        for pj in ("gate", "up"):
                            out[f"{base}.{e}.{fam[pj]}.weight_scale_2"] = ex.gs13[e].cpu().reshape(()).clone()
                        out[f"{base}.{e}.{fam['down']}.weight_scale_2"] = ex.gs2[e].cpu().reshape(()).clone()
            if mlp.shared is not None:
                I = mlp.shared.down.weight.shape[1]
                put_linear(name + ".shared.gate_up", mlp.shared.gate_up, [I, I],
                           gate_up_inter=mlp.shared.interleaved)
                put_linear(name + ".shared.down", mlp.shared.down)
            if mlp.shared_gate is not None:
                put(name + ".shared_gate", mlp.shared_gate)
    for j, m in enumerate(model.mtp):
        put(f"model.mtp{j}.enorm", m.enorm.weight)
        put(f"model.mtp{j}.hnorm", m.hnorm.weight)
        put(f"model.mtp{j}.head_norm", m.head_norm.weight)
        put_linear(f"mtp{j}.eh", m.eh_proj)
    save_file(out, path)


def _deinterleave(w: torch.Tensor) -> torch.Tensor:
    """Inverse of interleave_gate_up: 128-row blocks (gate, up) -> [gate; up]."""
    raw = w.view(torch.uint8) if w.dtype == torch.float8_e4m3fn else w
    I = raw.shape[0] // 2
    b = raw.reshape(I // 128, 2, 128, -1)
    r = torch.cat([b[:, 0].reshape(I, -1), b[:, 1].reshape(I, -1)], 0)
    return r.view(torch.float8_e4m3fn) if w.dtype == torch.float8_e4m3fn else r


def _deinterleave_scale(s: torch.Tensor) -> torch.Tensor:
    """Scales [2I/128, K/128] of interleaved rows -> gate blocks then up blocks."""
    n = s.shape[0] // 2
    b = s.reshape(n, 2, -1)
    return torch.cat([b[:, 0], b[:, 1]], 0)
