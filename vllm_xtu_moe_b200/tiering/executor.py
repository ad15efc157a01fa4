"""Tiered routed-expert execution: which pairs of an MoE layer run where.

``TieredExperts`` is handed to ``LLM(..., tiering=...)``.  While the model is built,
``expert_sink`` receives every MoE layer's routed experts in checkpoint layout and
either keeps them GPU-resident (kernel layout, like an untiered model) or moves them
into a C++ CPU engine (single NUMA-sharded host copy) and returns ``None``.
``attach`` then gives each host-tier MoE block a ``LayerExecutor``, which decides per
call (the reference's per-layer ``apply``, vllm_xiaotu_moe/mixed_experts.py:1919-3306):

1. long prefill (T >= ``gpu_prefill_min_tokens``, bf16/fp8 experts, not capturing):
   every expert streamed through the GPU ring (:mod:`.ring`);
2. hot-expert pool present: route split on the device -> pool pairs run on the GPU
   (grouped GEMM / GEMV) while the CPU engine runs the rest on the host (bridge on a
   side stream, joined by an event); one combine adds pool rows, the fp32 CPU
   partial and the shared expert;
3. otherwise: the CPU engine alone (bridge), combined with the shared expert.

The CPU part of (2) and (3) goes through one of two bridges: the host-function bridge
(D2H copies, a host-function node, H2D copy, on a side stream), or -- with
``XIAOTU_MOE_ASYNC`` -- the asynchronous bridge, where a kernel posts the request into
mapped host memory, one worker thread serves every tiered layer, and a second kernel
reads the result back with a bounded wait.  Expert deferral (``XIAOTU_MOE_DEFER``, the
reference's vllm_xiaotu_moe/mixed_experts.py:233-276) builds on the latter: in decode,
layer L's CPU-expert result is read back in layer L + 1 and added to that layer's MoE
output, so the CPU computes while the GPU runs layer L + 1's attention; the last main
layer reads back both its predecessor's and its own result.

Every path is graph-capturable except (1), which is host-orchestrated; decode
graphs therefore contain route split + pool GEMV + bridge + combine.
"""
from __future__ import annotations

import torch

from ..config import EngineConfig, get_engine_config, parse_layer_list
from ..ops import moe as M
from .cpu_engine import AsyncCpuBridge, CpuBridge, CpuExpertEngine
from .host import HostExperts, alloc_expert_slots
from .policy import load_pin_table
from .pool import LayerPool
from .ring import ExpertRing

GPU_FMTS = ("bf16", "fp8", "mxfp4", "nvfp4")


class LayerExecutor:
    def __init__(self, owner: "TieredExperts", layer: int, engine: CpuExpertEngine, host: HostExperts | None,
                 pool: LayerPool | None, lo: int = 0):
        self.owner, self.layer = owner, layer
        self.engine, self.host, self.pool = engine, host, pool
        # global id of this tier's first expert: under expert parallelism a rank holds the
        # experts [lo, lo + E) and leaves every other pair to the rank that owns it
        self.lo = lo
        self.bridge: CpuBridge | None = None
        self.calls = {"ring": 0, "hybrid": 0, "cpu": 0, "async": 0, "deferred": 0}
        self.is_mtp = False
        self.engine_index = -1            # index in the shared async bridge

    def _bridge(self, K: int) -> CpuBridge:
        if self.bridge is None:
            self.bridge = CpuBridge(self.engine, K, self.owner.bridge_tokens)
        return self.bridge

    def __call__(self, block, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, sh: torch.Tensor | None):
        o = self.owner
        act = block.cfg.swiglu_limit
        T, H = x.shape
        if not x.is_cuda:
            y = self._cpu_deferred(self.engine.forward(x, ids, w, lo=self.lo), T)
            if sh is not None:
                y = y + sh.float()
            return y.to(x.dtype)
        ids = ids.to(torch.int32).contiguous()
        w = w.float().contiguous()
        x = x.contiguous()
        capturing = torch.cuda.is_current_stream_capturing()
        if (o.ring is not None and self.host is not None and not capturing and T >= o.gpu_prefill_min_tokens):
            self.calls["ring"] += 1
            return o.ring.run_layer(self.host, x, ids, w, o.workspace(T, ids.shape[1], x.device), shared=sh,
                                    act_limit=act, lo=self.lo)
        if o.use_async and T <= o.bridge_tokens:
            return self._async(x, ids, w, sh, act)
        extra = torch.empty(T, H, dtype=torch.float32, device=x.device)
        main = torch.cuda.current_stream()
        if self.pool is not None and self.pool.nslots > 0:
            self.calls["hybrid"] += 1
            gpu_ids = torch.empty_like(ids)
            cpu_ids = torch.empty_like(ids)
            M.route_split(ids, self.pool.slotmap, self.lo, gpu_ids, cpu_ids, self.pool.hits)
            self._cpu(x, cpu_ids, w, extra, main, T)
            ws = o.pool_workspace(T, ids.shape[1], self.pool.nslots, x.device)
            M.moe_experts_partial(x, gpu_ids, w, self.pool.slots, ws, lo=0, act_limit=act)
            main.wait_stream(o.side)
            return M.moe_combine(ws, gpu_ids, 0, self.pool.nslots, shared=sh, extra=extra)
        self.calls["cpu"] += 1
        self._cpu(x, ids, w, extra, main, T)
        main.wait_stream(o.side)
        ws = o.pool_workspace(T, ids.shape[1], 1, x.device)
        return M.moe_combine(ws, ids, 0, 0, shared=sh, extra=extra)

    def reference_experts(self, block):
        """The host tier's experts as a dequantizable view (the in-service self-check's
        oracle): expert e is copied from the engine's shards into a one-expert GPU slot."""
        if self.host is None:
            return None
        return _HostExpertView(self.host, self.engine.E)

    def _cpu_deferred(self, y: torch.Tensor, T: int) -> torch.Tensor:
        """Host-tensor form of expert deferral (the oracle of the device path): returns the
        fp32 CPU-expert part this layer adds, given its own result `y`."""
        o = self.owner
        prev = o.cpu_pending
        if prev is not None and prev.shape[0] != T:      # left by an aborted forward
            prev = None
        if o.defer_ok(self, T):
            o.cpu_pending = y
            return prev if prev is not None else torch.zeros_like(y)
        o.cpu_pending = None
        return y if prev is None else y + prev

    def _async(self, x, ids, w, sh, act):
        """CPU experts through the asynchronous bridge, with expert deferral when enabled.
        Requests are read back in the order they were posted: the previous layer's (when
        deferred) before this layer's."""
        o = self.owner
        T, H = x.shape
        K = ids.shape[1]
        br = o.async_bridge(K)
        pool = self.pool if self.pool is not None and self.pool.nslots > 0 else None
        if pool is not None:
            gpu_ids, cpu_ids = torch.empty_like(ids), torch.empty_like(ids)
            M.route_split(ids, pool.slotmap, self.lo, gpu_ids, cpu_ids, pool.hits)
        else:
            gpu_ids, cpu_ids = ids, ids
        prev = o.defer_pending
        if prev is not None and prev != T:               # left by an aborted forward: drop it
            br.wait(torch.empty(prev, H, dtype=torch.float32, device=x.device))
            prev = None
        br.post(x, cpu_ids, w, engine=self.engine_index, lo=self.lo, hi=self.lo + self.engine.E)
        if pool is not None:
            ws = o.pool_workspace(T, K, pool.nslots, x.device)
            M.moe_experts_partial(x, gpu_ids, w, pool.slots, ws, lo=0, act_limit=act)
            nslots = pool.nslots
        else:
            ws = o.pool_workspace(T, K, 1, x.device)
            nslots = 0
        extra = torch.empty(T, H, dtype=torch.float32, device=x.device)
        if prev is not None:
            br.wait(extra)                               # the previous layer's CPU part
        if o.defer_ok(self, T):
            self.calls["deferred"] += 1
            o.defer_pending = T
            if prev is None:
                extra = None
        else:
            self.calls["async"] += 1
            br.wait(extra, accumulate=prev is not None)
            o.defer_pending = None
        return M.moe_combine(ws, gpu_ids, 0, nslots, shared=sh, extra=extra)

    def _cpu(self, x, ids, w, extra, main, T):
        """CPU-engine partial of the pairs in `ids` (ids < 0 are skipped) into `extra`, on the side stream."""
        o = self.owner
        o.side.wait_stream(main)
        if T <= o.bridge_tokens:
            self._bridge(ids.shape[1]).enqueue(x, ids, w, extra, self.lo, self.lo + self.engine.E, stream=o.side)
        else:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("CPU expert call above the bridge's token limit inside graph capture")
            with torch.cuda.stream(o.side):
                y = self.engine.forward(x.cpu(), ids.cpu(), w.cpu(), lo=self.lo)
                extra.copy_(y, non_blocking=False)


class _HostExpertView:
    """``num_experts`` + ``dequant(e)`` over a HostExperts (what ops.moe.moe_ref reads)."""

    def __init__(self, host: HostExperts, num_experts: int):
        self.host, self.num_experts = host, num_experts

    def dequant(self, e: int):
        h = self.host
        slot = alloc_expert_slots(h.fmt, 1, h.H, h.I, torch.device("cuda", torch.cuda.current_device()))
        st = torch.cuda.current_stream()
        h.copy_slot(e, slot, 0, st)
        st.synchronize()
        return slot.dequant(0)


class TieredExperts:
    """Expert placement of one model on one GPU: resident layers, hot pools, ring, CPU tier."""

    def __init__(self, cfg, *, device="cuda", engine_config: EngineConfig | None = None,
                 resident_layers: set[int] | None = None, pool_experts: dict[int, list[int]] | int | None = None,
                 ring: bool = True, max_tokens: int = 16384, bridge_tokens: int = 256,
                 gpu_prefill_min_tokens: int | None = None, threads: int | None = None):
        self.cfg = cfg
        self.device = torch.device(device)
        ec = engine_config or get_engine_config()
        self.ec = ec
        self.resident = (resident_layers if resident_layers is not None
                         else parse_layer_list(ec.resident_layers) if ec.resident_layers else set())
        if pool_experts is None and ec.pin and ec.pin_table:
            pool_experts = load_pin_table(ec.pin_table)
            if ec.pin_max_per_layer:
                pool_experts = {l: v[: ec.pin_max_per_layer] for l, v in pool_experts.items()}
        self.pool_experts = pool_experts or {}
        self.want_ring = ring
        self.max_tokens = max_tokens
        self.bridge_tokens = bridge_tokens
        self.gpu_prefill_min_tokens = (ec.gpu_prefill_min_tokens if gpu_prefill_min_tokens is None
                                       else gpu_prefill_min_tokens)
        self.threads = ec.moe_threads if threads is None else threads
        self._pending: list[tuple[int, CpuExpertEngine, HostExperts | None, LayerPool | None, int]] = []
        self.executors: list[LayerExecutor] = []
        self.ring: ExpertRing | None = None
        self._ws: dict = {}
        self.side = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.swaps = 0
        self.defer = bool(ec.moe_defer)
        self.use_async = bool(ec.moe_async) or self.defer   # deferral runs on the async bridge
        self._async_bridge: AsyncCpuBridge | None = None
        self.defer_pending: int | None = None     # T of the request posted by the previous layer, if deferred
        self.cpu_pending: torch.Tensor | None = None   # the same on the host-tensor path
        self._last_main: LayerExecutor | None = None

    # ---------------------------------------------------------------- build
    def _pool_list(self, layer: int, lo: int, E: int) -> list[int]:
        """This tier's pool experts of `layer` as local indices (the PIN table names global ids;
        an int asks for the first N experts of the tier)."""
        p = self.pool_experts
        if isinstance(p, int):
            return list(range(min(p, E)))
        return [e - lo for e in p.get(layer, []) if lo <= e < lo + E]

    def expert_sink(self, layer: int, raw: dict, lo: int = 0):
        """Routed experts of one layer (checkpoint layout).  ``lo``: global id of the first
        expert in ``raw`` (a tensor / expert parallel rank's share starts at rank * E / world)."""
        fmt = raw["fmt"]
        if layer in self.resident:
            e = M.prepare_experts(fmt, raw["w13"], raw["w2"], raw.get("s13"), raw.get("s2"), raw.get("gs13"),
                                  raw.get("gs2"))
            return e
        c = self.cfg
        mode = {"on": 1, "off": 0}.get(self.ec.moe_int8, 2)
        eng = CpuExpertEngine(fmt, raw["w13"].cpu(), raw["w2"].cpu(), _cpu(raw.get("s13")), _cpu(raw.get("s2")),
                              _cpu(raw.get("gs13")), _cpu(raw.get("gs2")), threads=self.threads,
                              act_limit=c.swiglu_limit, int8_mode=mode, int8_min_tokens=self.ec.moe_int8_min_tokens,
                              deadline_ms=self.ec.pool_deadline_ms)
        host = pool = None
        # "int4" (GPTQ kept at 4 bits) has no GPU slot format: its pairs all run on the CPU tier
        if self.device.type == "cuda" and fmt in GPU_FMTS:
            scales = HostExperts.gpu_scales_from_checkpoint(fmt, _cpu(raw.get("s13")), _cpu(raw.get("s2")),
                                                            _cpu(raw.get("gs13")), _cpu(raw.get("gs2")))
            host = HostExperts(eng, scales)
            experts = self._pool_list(layer, lo, int(raw["w13"].shape[0]))
            if experts:
                pool = LayerPool(host, experts, self.device, window=self.ec.pin_window if not self.ec.pin_static
                                 else 0, hyst=self.ec.pin_hyst, maxswap=self.ec.pin_maxswap)
            if self.want_ring and self.ring is None:
                te = max(1, min(self.ec.stage_tile_e, int(raw["w13"].shape[0])))
                self.ring = ExpertRing(fmt, c.hidden_size, c.moe_intermediate, te, max(2, self.ec.stage_nslots),
                                       self.device)
        self._pending.append((layer, eng, host, pool, lo))
        return None

    def attach(self, model) -> None:
        blocks = [l.mlp for l in model.layers] + [m.layer.mlp for m in getattr(model, "mtp", [])]
        n_main = len(model.layers)
        it = iter(self._pending)
        for i, b in enumerate(blocks):
            if getattr(b, "experts", "dense") is None and getattr(b, "executor", None) is None:
                layer, eng, host, pool, lo = next(it)
                ex = LayerExecutor(self, layer, eng, host, pool, lo)
                ex.is_mtp = i >= n_main
                b.executor = ex
                self.executors.append(ex)
                if not ex.is_mtp:
                    self._last_main = ex
        self._pending = []

    def defer_ok(self, ex: LayerExecutor, T: int) -> bool:
        """May `ex` leave its CPU result for the next layer?  Only in decode-sized steps,
        only main-model layers up to XIAOTU_MOE_DEFER_MAXLAYER, never the last one (it
        reads back before the final norm)."""
        if not self.defer or T > self.ec.moe_defer_maxq or ex.is_mtp or ex is self._last_main:
            return False
        return self.ec.moe_defer_maxlayer < 0 or ex.layer <= self.ec.moe_defer_maxlayer

    def async_bridge(self, K: int) -> AsyncCpuBridge:
        """The one asynchronous bridge of this model: every tiered layer's engine registered,
        one worker thread."""
        if self._async_bridge is None:
            first = self.executors[0]
            br = AsyncCpuBridge(first.engine, K, self.bridge_tokens, slots=2, spin_idle_us=self.ec.moe_spin_idle_us,
                                timeout_ms=self.ec.moe_async_timeout_ms, device=self.device)
            first.engine_index = 0
            for ex in self.executors[1:]:
                ex.engine_index = br.add_engine(ex.engine)
            self._async_bridge = br
        return self._async_bridge

    # ---------------------------------------------------------------- runtime
    def workspace(self, T: int, K: int, device) -> M.MoEWorkspace:
        key = ("ring", K)
        ws = self._ws.get(key)
        if ws is None or ws.max_tokens < T:
            ws = M.MoEWorkspace(max(T, self.max_tokens), K, self.cfg.num_experts, self.cfg.hidden_size,
                                self.cfg.moe_intermediate, device)
            self._ws[key] = ws
        return ws

    def pool_workspace(self, T: int, K: int, nslots: int, device) -> M.MoEWorkspace:
        key = ("pool", K, T)
        ws = self._ws.get(key)
        if ws is None or ws.num_experts < nslots:
            ws = M.MoEWorkspace(max(T, 16), K, max(nslots, 1), self.cfg.hidden_size, self.cfg.moe_intermediate,
                                device)
            self._ws[key] = ws
        return ws

    def step_done(self) -> None:
        """Once per engine step, outside graph capture: windowed pool adaptation."""
        for ex in self.executors:
            if ex.pool is not None:
                ev, _ = ex.pool.maybe_adapt()
                self.swaps += len(ev)

    def vram_bytes(self) -> dict:
        pools = sum(ex.pool.nbytes() for ex in self.executors if ex.pool is not None)
        ring = self.ring.bytes if self.ring is not None else 0
        ws = sum(w.nbytes() for w in self._ws.values())
        return {"pools": pools, "ring": ring, "workspaces": ws}

    def stats(self, hit_rate: bool = False) -> dict:
        """Call counts per path; ``hit_rate``: also the share of routed pairs the hot-expert
        pools served (synchronises the device)."""
        out = {"ring": 0, "hybrid": 0, "cpu": 0, "async": 0, "deferred": 0, "swaps": self.swaps}
        for ex in self.executors:
            for k, v in ex.calls.items():
                out[k] += v
        if hit_rate:
            hit = tot = 0
            for ex in self.executors:
                if ex.pool is not None and ex.pool.nslots > 0:
                    h, t = ex.pool.hit_counts()
                    hit, tot = hit + h, tot + t
            out["pool_hit_rate"] = hit / tot if tot else None
        return out

    def shutdown(self) -> None:
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        if self._async_bridge is not None:
            self._async_bridge.close()
            self._async_bridge = None
        for ex in self.executors:
            if ex.bridge is not None:
                ex.bridge.close()
            if ex.host is not None:
                ex.host.close()
            ex.engine.close()
        self.executors = []


def _cpu(t):
    return None if t is None else t.detach().cpu()
