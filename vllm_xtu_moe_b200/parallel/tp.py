"""Tensor parallelism over the GPUs of one node (attention / dense / shared expert split
across ranks, routed experts split by expert id), the reference's TP=2 + EP layout
(X1/X2: vLLM column/row-parallel linears, experts divided over TP ranks, partial sums
reduced after o_proj and after the MoE block, vllm_xiaotu_moe/hybrid_model.py:943-967,
1987, 2041).

* ``TPWeightFactory`` wraps any weight source (seeded synthetic or a checkpoint) and
  hands the model builder this rank's slices: query / key-value heads of the fused
  qkv, o_proj input columns, gate/up rows and down columns of dense and shared MLPs,
  DeltaNet key/value heads, MLA heads, and an expert range [r*E/T, (r+1)*E/T).  fp8
  block-scaled tensors are sliced exactly when the cut falls on 128-row/column
  boundaries and re-blocked otherwise.
* ``TPReducer`` sums the ranks' partial outputs through the peer-memory heap: a
  one-shot kernel (every rank reads every peer) for decode-sized tensors and a two-shot
  kernel (reduce one slice, store it into every rank) for prefill-sized ones; both sum
  in rank order, so every rank holds bit-identical activations and samples the same
  tokens.  ``nccl`` mode uses ``torch.distributed.all_reduce`` instead (baseline).
* ``build_tp_model`` builds the rank's model and installs the reducer in every layer.
"""
from __future__ import annotations

import dataclasses

import torch
import torch.distributed as dist

from ..models.config import ModelConfig
from ..models.layers import Linear, MoEBlock
from ..models.model import WeightFactory, build_model
from ..ops import _native as N
from ..ops.quant import dequant_fp8_block, quant_fp8_block
from .comm import PeerGroup


def local_config(cfg: ModelConfig, tp: int) -> ModelConfig:
    """Per-rank sizes (heads, intermediate widths); expert count stays global (router)."""
    def div(x, what):
        if x % tp:
            raise ValueError(f"{what}={x} is not divisible by tensor-parallel size {tp}")
        return x // tp
    kw = dict(num_heads=div(cfg.num_heads, "num_heads"))
    if not cfg.is_mla:
        for key in ("num_kv_heads", "swa_num_kv_heads"):
            n = getattr(cfg, key)
            if not n:
                continue
            kw[key] = n // tp if n >= tp else 1
            if n >= tp:
                div(n, key)
            elif tp % n:
                raise ValueError(f"tp must be a multiple of {key} when kv heads are replicated")
    if cfg.dense_intermediate:
        kw["dense_intermediate"] = div(cfg.dense_intermediate, "dense_intermediate")
    if cfg.shared_intermediate:
        kw["shared_intermediate"] = div(cfg.shared_intermediate, "shared_intermediate")
    if cfg.linear_num_key_heads:
        kw["linear_num_key_heads"] = div(cfg.linear_num_key_heads, "linear_num_key_heads")
        kw["linear_num_value_heads"] = div(cfg.linear_num_value_heads, "linear_num_value_heads")
    if cfg.num_experts:
        div(cfg.num_experts, "num_experts")
    return cfg.replace(**kw)


def _runs(idx: list[int]) -> list[tuple[int, int]]:
    out = []
    for i in idx:
        if out and out[-1][1] == i:
            out[-1] = (out[-1][0], i + 1)
        else:
            out.append((i, i + 1))
    return out


def _take(lin: Linear, rows: list[int] | None, cols: list[int] | None) -> Linear:
    w, s, b = lin.weight, lin.scale, lin.bias
    ri = None if rows is None else torch.tensor(rows, device=w.device)
    ci = None if cols is None else torch.tensor(cols, device=w.device)
    if s is None:
        if ri is not None:
            w = w.index_select(0, ri)
        if ci is not None:
            w = w.index_select(1, ci)
        return Linear(w.contiguous(), None, None if b is None else (b if ri is None else b.index_select(0, ri)))
    aligned = all(a % 128 == 0 and (e - a) % 128 == 0 for a, e in _runs(rows or [])) and \
        all(a % 128 == 0 and (e - a) % 128 == 0 for a, e in _runs(cols or []))
    if aligned:
        wq = w.view(torch.uint8)
        if ri is not None:
            wq = wq.index_select(0, ri)
            s = s.index_select(0, torch.tensor(sorted({r // 128 for r in rows}), device=w.device))
        if ci is not None:
            wq = wq.index_select(1, ci)
            s = s.index_select(1, torch.tensor(sorted({c // 128 for c in cols}), device=w.device))
        w = wq.contiguous().view(torch.float8_e4m3fn)
    else:                                  # cut inside a scale block: widen, slice, re-block
        d = dequant_fp8_block(w, s)
        if ri is not None:
            d = d.index_select(0, ri)
        if ci is not None:
            d = d.index_select(1, ci)
        w, s = quant_fp8_block(d.contiguous())
    if b is not None and ri is not None:
        b = b.index_select(0, ri)
    return Linear(w, s.contiguous(), b)


class TPWeightFactory:
    """This rank's slices of the tensors of a full-size source (see module docstring)."""

    def __init__(self, base, full: ModelConfig, rank: int, tp: int):
        self.base, self.full, self.rank, self.tp = base, full, rank, tp
        self.device = base.device
        self.expert_lo = 0

    # -------------------------------------------------------------- index helpers
    def _heads(self, n: int) -> list[int]:
        per = n // self.tp
        return list(range(self.rank * per, (self.rank + 1) * per))

    def _kv_heads(self, n: int | None = None) -> list[int]:
        n = self.full.num_kv_heads if n is None else n
        if n >= self.tp:
            return self._heads(n)
        return [self.rank * n // self.tp]

    def _layer(self, name: str) -> int:
        """Decoder-layer index in a tensor name ("model.layers.<i>. ..."; MTP layers: the last)."""
        c = self.full
        parts = name.split(".")
        if "layers" in parts:
            j = parts.index("layers") + 1
            if j < len(parts) and parts[j].isdigit():
                return min(int(parts[j]), c.num_layers - 1)
        return c.num_layers - 1

    @staticmethod
    def _expand(heads: list[int], width: int, base: int = 0) -> list[int]:
        return [base + h * width + i for h in heads for i in range(width)]

    def _rows_cols(self, name: str):
        """-> (full_n, full_k, rows or None, cols or None) for a sliced linear, or None if replicated."""
        c, T = self.full, self.tp
        H = c.hidden_size
        suf = name.rsplit(".", 1)[-1]
        if suf == "qkv":
            hd, vd = c.head_dim, c.gqa_v_dim
            kvh = c.kv_heads(self._layer(name))
            qw = hd * (2 if c.attn_output_gate else 1)
            nq, nk = c.num_heads * qw, kvh * hd
            rows = (self._expand(self._heads(c.num_heads), qw) + self._expand(self._kv_heads(kvh), hd, nq) +
                    self._expand(self._kv_heads(kvh), vd, nq + nk))
            return nq + nk + kvh * vd, H, rows, None
        if suf == "o" and c.is_mla:
            return H, c.num_heads * c.v_head_dim, None, self._expand(self._heads(c.num_heads), c.v_head_dim)
        if suf == "o":
            return H, c.num_heads * c.gqa_v_dim, None, self._expand(self._heads(c.num_heads), c.gqa_v_dim)
        if suf == "q_b":
            w = c.qk_nope_head_dim + c.qk_rope_head_dim
            return c.num_heads * w, c.q_lora_rank or H, self._expand(self._heads(c.num_heads), w), None
        if suf == "kv_b":
            w = c.qk_nope_head_dim + c.v_head_dim
            return c.num_heads * w, c.kv_lora_rank, self._expand(self._heads(c.num_heads), w), None
        if suf.startswith("kda_"):
            nk, nv, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
            if suf == "kda_qkv":     # blocked [Q | K | V]
                rows = (self._expand(self._heads(nk), dk) + self._expand(self._heads(nk), dk, nk * dk) +
                        self._expand(self._heads(nv), dv, 2 * nk * dk))
                return 2 * nk * dk + nv * dv, H, rows, None
            if suf == "kda_b":
                return nv, H, self._heads(nv), None
            if suf == "kda_f_b":
                return nv * dk, dk, self._expand(self._heads(nv), dk), None
            if suf == "kda_g_b":
                return nv * dv, dk, self._expand(self._heads(nv), dv), None
            return None              # kda_f_a, kda_g_a: the low-rank down-projections are replicated
        if suf in ("qkvz", "ba", "out") and c.linear_num_key_heads:
            nk, nv, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
            r = nv // nk
            if suf == "qkvz":
                w = 2 * dk + 2 * r * dv
                return nk * w, H, self._expand(self._heads(nk), w), None
            if suf == "ba":
                return nk * 2 * r, H, self._expand(self._heads(nk), 2 * r), None
            return H, nv * dv, None, self._expand(self._heads(nv), dv)
        if suf == "gate_up":
            I = c.dense_intermediate if ".mlp." in name else c.shared_intermediate * max(1, c.num_shared_experts)
            per = I // T
            g = list(range(self.rank * per, (self.rank + 1) * per))
            return 2 * I, H, g + [I + i for i in g], None
        if suf == "down":
            I = c.dense_intermediate if ".mlp." in name else c.shared_intermediate * max(1, c.num_shared_experts)
            per = I // T
            return H, I, None, list(range(self.rank * per, (self.rank + 1) * per))
        return None

    # -------------------------------------------------------------- factory interface
    def linear(self, name, n, k, fmt="bf16", bias=False, std=None) -> Linear:
        spec = self._rows_cols(name)
        if spec is None:
            return self.base.linear(name, n, k, fmt, bias, std)
        fn, fk, rows, cols = spec
        full = self.base.linear(name, fn, fk, fmt, bias, std)
        out = _take(full, rows, cols)
        assert tuple(out.weight.shape) == (n, k), (name, tuple(out.weight.shape), (n, k))
        return out

    def normal(self, name, shape, std=None, dtype=torch.bfloat16):
        c = self.full
        if name.endswith(".conv") and c.linear_num_key_heads:
            nk, nv, dk, dv = c.linear_num_key_heads, c.linear_num_value_heads, c.linear_key_head_dim, c.linear_value_head_dim
            full = self.base.normal(name, (2 * nk * dk + nv * dv, shape[1]), std, dtype)
            kh = self._heads(nk)
            ch = self._expand(kh, dk) + self._expand(kh, dk, nk * dk) + self._expand(self._heads(nv), dv, 2 * nk * dk)
            return full.index_select(0, torch.tensor(ch, device=full.device)).contiguous()
        return self.base.normal(name, shape, std, dtype)

    def ones(self, shape, dtype=torch.bfloat16, name=None):
        return self.base.ones(shape, dtype, name=name)

    def zeros(self, shape, dtype=torch.bfloat16, name=None):
        return self.base.zeros(shape, dtype, name=name)

    def param(self, name, make, n):
        c = self.full
        if name.endswith(".dt_bias") and c.linear_kind == "kda":
            full_n = c.linear_num_value_heads * c.linear_key_head_dim      # one bias per (head, key dim)
        elif name.endswith((".A_log", ".dt_bias")):
            full_n = c.linear_num_value_heads
        else:
            full_n = c.num_heads if name.endswith(".sinks") else n
        t = self.base.param(name, make, full_n)
        if full_n != n:
            t = t[self.rank * n:(self.rank + 1) * n].contiguous()
        return t

    def experts(self, name, E, H, I, fmt) -> dict:
        raw = self.base.experts(name, E, H, I, fmt)
        El = E // self.tp
        lo = self.rank * El
        self.expert_lo = lo
        return {k: (v[lo:lo + El].contiguous() if isinstance(v, torch.Tensor) else v) for k, v in raw.items()}


class TPReducer:
    """Sum of the ranks' partial [T, H] outputs (P2P one-shot / two-shot, or NCCL).

    mode "fused" adds the decode form of the row-parallel output projection (the
    GEMM -> reduce-scatter fusion at decode sizes): the GEMV's epilogue stores each rank's partial rows straight into every rank's
    receive buffer over NVLink and flags them (``xtu_gemv_tp``); the next RMSNorm sums
    them in rank order, adds the residual and normalises (``xtu_tp_sum_rmsnorm``), so no
    separate all-reduce or copy runs.  Larger steps use the one-shot / two-shot kernels."""

    ONESHOT_BYTES = 256 << 10
    FUSED_MAX_TOKENS = 16

    def __init__(self, max_tokens: int, hidden: int, group=None, device=None, mode: str = "p2p"):
        self.mode = mode
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_max = max_tokens * hidden
        self.hidden = hidden
        if mode in ("p2p", "fused"):
            nb = self.n_max * 2
            self.slot = self.FUSED_MAX_TOKENS * hidden
            sizes = [nb, nb] + ([2 * self.world * self.slot * 2, self.world * 4] if mode == "fused" else [])
            self.pg = PeerGroup(PeerGroup.heap_bytes_for(*sizes), group=group, device=device)
            self.inb = self.pg.alloc((self.n_max,), torch.bfloat16)
            self.outb = self.pg.alloc((self.n_max,), torch.bfloat16)
            if mode == "fused":
                d = self.pg.device
                self.recv = self.pg.alloc((2 * self.world * self.slot,), torch.bfloat16)
                self.tpflags = self.pg.alloc((self.world,), torch.int32)
                # ep_c, ep_p (epochs the consumer / producer last finished), done_p, done_c
                self.ctl = torch.zeros(4, dtype=torch.int32, device=d)
                self.pg.barrier()   # every rank's flags are zero before any use
        self.calls = 0
        self.fused_calls = 0

    # ------------------------------------------------------------------ fused decode form
    def fusable(self, x: torch.Tensor, lin) -> bool:
        T, K = x.shape
        return (self.mode == "fused" and x.is_cuda and T <= self.FUSED_MAX_TOKENS and lin.bias is None
                and lin.weight.shape[0] == self.hidden and K % 64 == 0 and x.dtype == torch.bfloat16
                and (K * lin.weight.element_size()) % 128 == 0)

    def linear_scatter(self, x: torch.Tensor, lin) -> "PendingTPSum":
        """Row-parallel ``lin(x)`` whose partial goes to every rank's receive buffer."""
        from ..ops import gemm as G
        x = G.tma_rows(x)
        T, K = x.shape
        ws, cnt = G._gemv_split_ws(x.device)
        c = self.ctl
        N.call("xtu_gemv_tp", lin.weight.data_ptr(), N.ptr(lin.scale), int(lin.scale is not None), self.hidden, K,
               x.data_ptr(), x.stride(0), T, ws.data_ptr(), cnt.data_ptr(), self.recv.ptr(), self.slot, self.pg.rank,
               self.world, c[2:].data_ptr(), self.tpflags.ptr(), c[0:].data_ptr(), c[1:].data_ptr(),
               N.status_buffer(x.device).data_ptr(), N.stream_ptr(x.device))
        self.fused_calls += 1
        return PendingTPSum(self, T)

    def sum_rmsnorm(self, T: int, residual: torch.Tensor, norm) -> tuple[torch.Tensor, torch.Tensor]:
        """(RMSNorm(sum of the ranks' partials + residual), the new residual)."""
        H = self.hidden
        y = torch.empty(T, H, dtype=torch.bfloat16, device=residual.device)
        r_out = torch.empty_like(y)
        c = self.ctl
        N.call("xtu_tp_sum_rmsnorm", self.recv.local.data_ptr(), self.slot, self.world, T, H,
               self.tpflags.local.data_ptr(), c[1:].data_ptr(), c[0:].data_ptr(), c[3:].data_ptr(),
               residual.contiguous().data_ptr(), r_out.data_ptr(), norm.weight.data_ptr(), y.data_ptr(),
               float(norm.eps), int(norm.add_one), N.status_buffer(residual.device).data_ptr(), self.pg.timeout_ns,
               N.stream_ptr(residual.device))
        self.calls += 1
        return y, r_out

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if isinstance(x, PendingTPSum):
            raise TypeError("a pending fused TP sum is finished by sum_rmsnorm, not reduced again")
        self.calls += 1
        if self.mode == "nccl":
            y = x.contiguous()
            dist.all_reduce(y, group=self.group)
            return y
        n = x.numel()
        if n > self.n_max or n % 8:
            raise ValueError(f"TP reduce of {n} elements (capacity {self.n_max}, multiple of 8 required)")
        self.inb.local[:n].copy_(x.reshape(-1))
        pg = self.pg
        if n * 2 <= self.ONESHOT_BYTES:
            out = torch.empty_like(x)
            N.call("xtu_allreduce_oneshot", self.inb.ptr(), out.data_ptr(), n, 0, pg.flags.ptr(),
                   pg.epoch.data_ptr(), pg.rank, pg.world, pg.status.data_ptr(), pg.timeout_ns,
                   N.stream_ptr(x.device))
            return out
        N.call("xtu_allreduce_twoshot", self.inb.ptr(), self.outb.ptr(), n, 0, pg.flags.ptr(), pg.epoch.data_ptr(),
               pg.rank, pg.world, pg.status.data_ptr(), pg.timeout_ns, N.stream_ptr(x.device))
        return self.outb.local[:n].view_as(x).clone()

    def close(self):
        if self.mode in ("p2p", "fused"):
            self.pg.close()


class PendingTPSum:
    """A row-parallel projection whose ranks' partials are in flight to every rank's
    receive buffer; ``finish`` sums them inside the following RMSNorm."""

    def __init__(self, reducer: TPReducer, T: int):
        self.reducer, self.T = reducer, T

    def finish(self, residual: torch.Tensor, norm) -> tuple[torch.Tensor, torch.Tensor]:
        return self.reducer.sum_rmsnorm(self.T, residual, norm)


class TPRowLinear:
    """Output projection of a TP attention block: decode-size calls take the fused
    GEMV -> peer-scatter path (returning a PendingTPSum), others run the plain linear."""

    def __init__(self, lin, reducer: TPReducer):
        self.lin, self.reducer = lin, reducer
        self.weight, self.scale, self.bias = lin.weight, lin.scale, lin.bias

    @property
    def out_features(self) -> int:
        return self.lin.out_features

    def __call__(self, x: torch.Tensor, out_dtype=torch.bfloat16):
        if out_dtype == torch.bfloat16 and self.reducer.fusable(x, self.lin):
            return self.reducer.linear_scatter(x, self.lin)
        return self.lin(x, out_dtype)

    def tensors(self):
        return self.lin.tensors()


def build_tp_model(cfg: ModelConfig, rank: int, tp: int, device, seed: int = 0, source=None,
                   reducer: TPReducer | None = None, num_layers: int | None = None, tiering=None):
    """This rank's shard of the model (random init or ``source``) with the reducer installed.

    ``tiering`` (a :class:`~vllm_xtu_moe_b200.tiering.executor.TieredExperts` of this rank):
    the rank's E / tp routed experts of every MoE layer go to its tiers (CPU engine, hot
    pool, ring) instead of HBM; each layer's executor serves only the pairs routed to the
    rank's experts, and the layer's partial joins the attention / shared-expert partials in
    the same reduction, as the GPU-resident experts do."""
    base = source if source is not None else WeightFactory(seed, device)
    f = TPWeightFactory(base, cfg, rank, tp)
    lcfg = local_config(cfg, tp)
    lo_by_layer = {}

    def sink(layer, raw):
        lo_by_layer.setdefault(layer, []).append(f.expert_lo)
        if tiering is not None:
            return tiering.expert_sink(layer, raw, lo=f.expert_lo)
        from ..ops import moe as M
        return M.prepare_experts(raw["fmt"], raw["w13"], raw["w2"], raw.get("s13"), raw.get("s2"),
                                 raw.get("gs13"), raw.get("gs2"))

    m = build_model(lcfg, device=device, seed=seed, expert_sink=sink, num_layers=num_layers, source=f)
    El = cfg.num_experts // tp if cfg.num_experts else 0
    for l in m.layers + [mt.layer for mt in m.mtp]:
        l.reduce = reducer
        if reducer is not None and reducer.mode == "fused" and hasattr(l.attn, "o"):
            l.attn.o = TPRowLinear(l.attn.o, reducer)   # GQA / MLA output projection
        if isinstance(l.mlp, MoEBlock):
            l.mlp.expert_lo = rank * El
    if tiering is not None:
        tiering.attach(m)
    m.tp = (rank, tp)
    return m
