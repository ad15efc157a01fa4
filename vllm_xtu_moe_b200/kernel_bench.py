"""Per-kernel microbenchmarks on the shapes of the serving configs, timed with CUDA
events (warm-up, L2 flushed between iterations) and reported against the measured
peaks of the GPU (copy bandwidth, dense bf16 GEMM rate).

    python -m vllm_xtu_moe_b200.kernel_bench --op moe_prefill_fp8 [--tokens 8192]
    python -m vllm_xtu_moe_b200.kernel_bench --op all

Each op prints one JSON line: the shape, device time per call, the algorithmic
bytes and FLOPs of one call, and the achieved fractions of the measured peaks.
These are also the small cases that kernel profiles are captured on.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch

from .ops import attention as A
from .ops import basic as B
from .ops import gemm as G
from .ops import moe as M
from .ops import _native as N_
from .ops.attention import AttnMetadata
from .ops.quant import quant_fp8_block
from .ops.router import router_topk, zipf_bias

_PEAKS = Path(__file__).resolve().parent.parent / "MEASURED_PEAKS.json"


def peaks() -> dict:
    if _PEAKS.exists():
        p = json.loads(_PEAKS.read_text())
        return {"hbm_gbs": p["hbm_gbs"], "bf16_tflops": p["bf16_tflops"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def time_fn(fn, iters: int = 10, warmup: int = 3, flush: bool = True) -> float:
    """Median device milliseconds per call; a 256 MB write between calls evicts L2.  A
    0.1 ms device-side spin before the start event keeps the host's launch cost of `fn`
    out of the measured interval (the GPU is still busy when `fn` is enqueued)."""
    scratch = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if flush else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        if scratch is not None:
            scratch.fill_(1)
        torch.cuda._sleep(200_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    torch.cuda.synchronize()
    ts.sort()
    return ts[len(ts) // 2]


def time_graph(fns, reps: int = 7) -> float:
    """Median device milliseconds per call of `fns` (callables) replayed back to back from one
    CUDA graph, as the decode step runs them: launch gaps and programmatic-dependent-launch
    overlap included, host launch cost excluded.  Callers pass enough distinct weight copies
    that one pass over them exceeds L2."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for f in fns:
            f()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for f in fns:
            f()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        torch.cuda._sleep(200_000)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) / len(fns))
    ts.sort()
    del g
    return ts[len(ts) // 2]


def _report(op: str, shape: dict, ms: float, nbytes: float, flops: float) -> dict:
    pk = peaks()
    tbs = nbytes / (ms * 1e-3) / 1e12
    tfl = flops / (ms * 1e-3) / 1e12
    return {"op": op, "shape": shape, "ms": round(ms, 4), "bytes": int(nbytes), "flops": int(flops),
            "tb_s": round(tbs, 3), "tflop_s": round(tfl, 1),
            "frac_hbm": round(tbs * 1e3 / pk["hbm_gbs"], 3), "frac_bf16": round(tfl / pk["bf16_tflops"], 3),
            "peaks": pk["source"]}


def _experts(E, H, I, fmt, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w13 = torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.02
    w2 = torch.randn(E, H, I, device="cuda", generator=g) * 0.02
    if fmt == "fp8":
        q13, s13 = quant_fp8_block(w13)
        q2, s2 = quant_fp8_block(w2)
        del w13, w2
        ex = M.prepare_experts("fp8", q13, q2, s13, s2)
    elif fmt == "mxfp4":
        from .ops.quant import quant_mxfp4
        p13, s13 = quant_mxfp4(w13)
        p2, s2 = quant_mxfp4(w2)
        del w13, w2
        ex = M.prepare_experts("mxfp4", p13, p2, s13, s2)
    elif fmt == "nvfp4":
        from .ops.quant import quant_nvfp4
        r13 = [quant_nvfp4(w13[e]) for e in range(E)]
        r2 = [quant_nvfp4(w2[e]) for e in range(E)]
        del w13, w2
        p13, s13, gs13 = (torch.stack([r[i] for r in r13]) for i in range(3))
        p2, s2, gs2 = (torch.stack([r[i] for r in r2]) for i in range(3))
        ex = M.prepare_experts("nvfp4", p13, p2, s13, s2, gs13.float(), gs2.float())
    else:
        ex = M.prepare_experts("bf16", w13.to(torch.bfloat16), w2.to(torch.bfloat16))
        del w13, w2
    torch.cuda.empty_cache()
    return ex


def _routes(T, E, K, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    logits = torch.randn(T, E, device="cuda", generator=g) + zipf_bias(E, 1.1, seed).cuda()
    return router_topk(logits, K, "softmax")


def bench_moe(T: int, fmt: str, E=128, H=4096, I=1408, K=8, iters=10) -> dict:
    ex = _experts(E, H, I, fmt)
    ids, w = _routes(T, E, K)
    x = (torch.randn(T, H, device="cuda") * 0.5).to(torch.bfloat16)
    ws = M.MoEWorkspace(T, K, E, H, I, x.device)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    fn = lambda: M.fused_moe(x, ids, w, ex, ws, out=out)
    ms = time_fn(fn, iters)
    active = torch.unique(ids).numel()
    per = {"fp8": 1.0, "bf16": 2.0, "mxfp4": 0.5 + 1 / 32, "nvfp4": 0.5 + 1 / 16}[fmt]
    wb = per * 3 * H * I * active
    nbytes = wb + T * H * 2 * 2 + T * K * H * 2 * 3
    flops = 2 * T * K * 3 * H * I
    return _report(f"moe_{'decode' if T <= G.GEMV_MAX_M else 'prefill'}_{fmt}",
                   dict(T=T, E=E, H=H, I=I, K=K, active_experts=active), ms, nbytes, flops)


_REF_ROOT = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


def load_reference_module(name: str):
    """A module of the reference plugin, unmodified, from its install in baseline/_ref.

    The plugin package's ``__init__`` (which patches a vLLM tree that is not installed
    here) is not executed: an empty package object stands in for it, so the reference's
    kernel modules (plain torch + Triton) import exactly as written."""
    import importlib
    import sys
    import types
    pkg = "vllm_xiaotu_moe"
    root = _REF_ROOT / pkg
    if not root.is_dir():
        raise FileNotFoundError(f"{root} missing: install the reference into baseline/_ref")
    if pkg not in sys.modules or not hasattr(sys.modules[pkg], "__path__"):
        m = types.ModuleType(pkg)
        m.__path__ = [str(root)]
        sys.modules[pkg] = m
    return importlib.import_module(f"{pkg}.{name}")


def bench_moe_vs_reference(T: int, E=128, H=4096, I=1408, K=8, iters=10) -> dict:
    """One fp8-128 MoE layer (GLM-4.5-Air shape) through this library's kernels and through
    the reference's own Triton kernels on the same GPU, weights and routes: the prefill
    entry ``gpu_moe_layer_fp8`` (vllm_xiaotu_moe/gpu_prefill_fp8.py:458) or, at decode
    sizes, ``gpu_moe_decode_fp8`` (vllm_xiaotu_moe/decode_moe_fp8.py:103)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    w13 = torch.randn(E, 2 * I, H, device="cuda", generator=g) * 0.02
    w2 = torch.randn(E, H, I, device="cuda", generator=g) * 0.02
    q13, s13 = quant_fp8_block(w13)
    q2, s2 = quant_fp8_block(w2)
    del w13, w2
    ex = M.prepare_experts("fp8", q13, q2, s13, s2)
    # the reference's K-major layout: w13t [E, H, 2I], s13t [E, H/128, 2I/128]; w2t [E, I, H]
    w13t = q13.view(torch.uint8).transpose(1, 2).contiguous()
    s13t = s13.transpose(1, 2).contiguous()
    w2t = q2.view(torch.uint8).transpose(1, 2).contiguous()
    s2t = s2.transpose(1, 2).contiguous()
    del q13, q2
    torch.cuda.empty_cache()
    ids, w = _routes(T, E, K)
    x = (torch.randn(T, H, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    ws = M.MoEWorkspace(T, K, E, H, I, x.device)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    ours = lambda: M.fused_moe(x, ids, w, ex, ws, out=out)
    decode = T <= 32
    if decode:
        ref_mod = load_reference_module("decode_moe_fp8")
        ref = lambda: ref_mod.gpu_moe_decode_fp8(x, ids, w, w13t, s13t, w2t, s2t, H, I, K, device=x.device)
        entry = "decode_moe_fp8.gpu_moe_decode_fp8"
    else:
        ref_mod = load_reference_module("gpu_prefill_fp8")
        ref = lambda: ref_mod.gpu_moe_layer_fp8(x, ids, w, w13t, s13t, w2t, s2t, H, I, K, device=x.device)
        entry = "gpu_prefill_fp8.gpu_moe_layer_fp8"
    ours()
    y_ref = ref().float()
    torch.cuda.synchronize()
    rel = float((out.float() - y_ref).norm() / y_ref.norm().clamp_min(1e-12))
    ms_ours = time_fn(ours, iters)
    ms_ref = time_fn(ref, iters)
    active = torch.unique(ids).numel()
    nbytes = 3 * H * I * active + T * H * 2 * 2 + T * K * H * 2 * 3
    flops = 2 * T * K * 3 * H * I
    r = _report(f"moe_{'decode' if decode else 'prefill'}_fp8_vs_reference",
                dict(T=T, E=E, H=H, I=I, K=K, active_experts=active), ms_ours, nbytes, flops)
    r.update({"reference_entry": entry, "reference_ms": round(ms_ref, 4),
              "speedup_vs_reference": round(ms_ref / ms_ours, 2), "rel_err_vs_reference": round(rel, 5)})
    return r


def bench_moe_w8a8(T: int, E=128, H=4096, I=1408, K=8, iters=10) -> dict:
    """The fp8 MoE layer in W8A8 mode (XTU_FP8_MMA=1: activations quantized per (row, 128),
    kind::f8f6f4 MMAs with per-128 block-scale promotion), beside the default bf16-activation
    path on the same weights and routes; reports both and the relative difference."""
    ex = _experts(E, H, I, "fp8")
    ids, w = _routes(T, E, K)
    x = (torch.randn(T, H, device="cuda") * 0.5).to(torch.bfloat16)
    ws = M.MoEWorkspace(T, K, E, H, I, x.device)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    fn = lambda: M.fused_moe(x, ids, w, ex, ws, out=out)
    ms_bf16 = time_fn(fn, iters)
    ref = out.float().clone()
    G.FP8_MMA = True
    try:
        ms = time_fn(fn, iters)
        fn()
        torch.cuda.synchronize()
    finally:
        G.FP8_MMA = False
    rel = float((out.float() - ref).norm() / ref.norm())
    active = torch.unique(ids).numel()
    r = _report("moe_prefill_fp8_w8a8", dict(T=T, E=E, H=H, I=I, K=K, active_experts=active), ms,
                3 * H * I * active + T * H * 2 * 2 + T * K * H * 2, 2 * T * K * 3 * H * I)
    r.update({"bf16_activation_ms": round(ms_bf16, 4), "speedup_vs_bf16_activations": round(ms_bf16 / ms, 2),
              "rel_diff_vs_bf16_activations": round(rel, 4)})
    return r


def bench_gemv(N: int, Kd: int, M_: int, fmt: str, iters=20, graph: bool = False) -> dict:
    """Decode GEMV y[M, N] = x W^T.  graph: the per-call time of calls replayed from one CUDA
    graph over distinct weight copies (more than 2x L2 in all); else single calls with an L2
    flush before each."""
    w = torch.randn(N, Kd, device="cuda") * 0.02
    if fmt == "fp8":
        w, s = quant_fp8_block(w)
    else:
        w, s = w.to(torch.bfloat16), None
    x = torch.randn(M_, Kd, device="cuda").to(torch.bfloat16)
    wbytes = w.numel() * w.element_size()
    if graph:
        copies = [w] + [w.clone() for _ in range(max(1, (260 << 20) // wbytes))]
        y = torch.empty(M_, N, device="cuda", dtype=torch.bfloat16)
        ms = time_graph([lambda c=c: G.gemv(x, c, s, out=y) for c in copies] * 2)
    else:
        ms = time_fn(lambda: G.linear(x, w, s), iters)
    nbytes = wbytes + M_ * (Kd + N) * 2
    return _report(f"gemv_{fmt}" + ("_graph" if graph else ""), dict(N=N, K=Kd, M=M_), ms, nbytes,
                   2 * M_ * N * Kd)


def bench_gemm(Mr: int, N: int, Kd: int, fmt: str, iters=10) -> dict:
    w = torch.randn(N, Kd, device="cuda") * 0.02
    if fmt == "fp8":
        w, s = quant_fp8_block(w)
    else:
        w, s = w.to(torch.bfloat16), None
    x = torch.randn(Mr, Kd, device="cuda").to(torch.bfloat16)
    fn = lambda: G.linear(x, w, s)
    ms = time_fn(fn, iters)
    nbytes = w.numel() * w.element_size() + Mr * (Kd + N) * 2
    return _report(f"gemm_{fmt}", dict(M=Mr, N=N, K=Kd), ms, nbytes, 2 * Mr * N * Kd)


def _cache(Bn, kv, Hkv, D, bs=64):
    nb_per = (kv + bs - 1) // bs
    nb = Bn * nb_per
    kc = (torch.randn(nb, Hkv, bs, D, device="cuda") * 0.5).to(torch.bfloat16)
    vc = (torch.randn(nb, Hkv, bs, D, device="cuda") * 0.5).to(torch.bfloat16)
    bt = torch.arange(nb, dtype=torch.int32, device="cuda").view(Bn, nb_per)
    return kc, vc, bt


def bench_attn_decode(Bn=4, kv=15000, Hq=96, Hkv=8, D=128, ql=1, kv_dtype="bf16", iters=20,
                      splits: int | None = None) -> dict:
    """GQA decode attention over the paged cache: ``ql`` query positions per sequence (5 =
    an MTP k=4 verification step), bf16 or fp8 (e4m3) cache; ``splits`` overrides the
    split-KV factor."""
    kc, vc, bt = _cache(Bn, kv, Hkv, D)
    if kv_dtype == "fp8":
        from .ops.basic import to_e4m3
        kc = to_e4m3(kc, 1.0)
        vc = to_e4m3(vc.transpose(2, 3).contiguous(), 1.0)
    T = Bn * ql
    q = (torch.randn(T, Hq, D, device="cuda") * 0.5).to(torch.bfloat16)
    d = "cuda"
    meta = AttnMetadata(num_seqs=Bn, q_start=torch.arange(0, T + 1, ql, dtype=torch.int32, device=d),
                        kv_len=torch.full((Bn,), kv, dtype=torch.int32, device=d), block_table=bt,
                        slot_mapping=torch.zeros(T, dtype=torch.int32, device=d),
                        positions=torch.full((T,), kv - 1, dtype=torch.int32, device=d), max_q_len=ql,
                        max_kv_len=kv, is_decode=True)
    per_sm = (2 if ql * (Hq // Hkv) <= 32 else 1) if D in (64, 128) else 1
    meta.num_splits = splits or A.choose_splits(Bn, Hkv, kv, ctas_per_sm=per_sm)
    ws = torch.empty(A.num_split_workspace(T, Hq, D, meta.num_splits), dtype=torch.float32, device=d)
    out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=d)
    fn = lambda: A.paged_attention(q, kc, vc, meta, out=out, workspace=ws)
    ms = time_fn(fn, iters)
    nbytes = 2 * Bn * kv * Hkv * D * (1 if kv_dtype == "fp8" else 2)
    flops = 4 * T * kv * Hq * D
    return _report("attention_decode", dict(B=Bn, kv=kv, Hq=Hq, Hkv=Hkv, D=D, q_len=ql, kv_dtype=kv_dtype,
                                            splits=meta.num_splits), ms, nbytes, flops)


def bench_mla_decode(Bn=4, kv=15000, Hq=128, iters=20) -> dict:
    """DeepSeek-V3 absorbed MLA decode over the 576-wide latent cache (V = first 512 dims)."""
    d = "cuda"
    nb_per = (kv + 63) // 64
    kc = (torch.randn(Bn * nb_per, 1, 64, 576, device=d) * 0.5).to(torch.bfloat16)
    bt = torch.arange(Bn * nb_per, dtype=torch.int32, device=d).view(Bn, nb_per)
    q = (torch.randn(Bn, Hq, 576, device=d) * 0.5).to(torch.bfloat16)
    meta = AttnMetadata(num_seqs=Bn, q_start=torch.arange(Bn + 1, dtype=torch.int32, device=d),
                        kv_len=torch.full((Bn,), kv, dtype=torch.int32, device=d), block_table=bt,
                        slot_mapping=torch.zeros(Bn, dtype=torch.int32, device=d),
                        positions=torch.full((Bn,), kv - 1, dtype=torch.int32, device=d), max_q_len=1,
                        max_kv_len=kv, is_decode=True)
    meta.num_splits = A.choose_splits(Bn, 2, kv)
    ws = torch.empty(A.num_split_workspace(Bn, Hq, 512, meta.num_splits), dtype=torch.float32, device=d)
    out = torch.empty(Bn, Hq, 512, dtype=torch.bfloat16, device=d)
    fn = lambda: A.paged_attention(q, kc, None, meta, 1.0 / 192 ** 0.5, v_dim=512, out=out, workspace=ws)
    ms = time_fn(fn, iters)
    nbytes = Bn * kv * 576 * 2
    flops = 2 * Bn * Hq * kv * (576 + 512)
    return _report("mla_decode", dict(B=Bn, kv=kv, Hq=Hq, splits=meta.num_splits), ms, nbytes, flops)


def bench_attn_prefill(T=8192, Hq=96, Hkv=8, D=128, iters=5) -> dict:
    kc, vc, bt = _cache(1, T, Hkv, D)
    q = (torch.randn(T, Hq, D, device="cuda") * 0.5).to(torch.bfloat16)
    d = "cuda"
    meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T], dtype=torch.int32, device=d),
                        kv_len=torch.tensor([T], dtype=torch.int32, device=d), block_table=bt,
                        slot_mapping=torch.zeros(T, dtype=torch.int32, device=d),
                        positions=torch.arange(T, dtype=torch.int32, device=d), max_q_len=T, max_kv_len=T,
                        is_decode=False)
    out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=d)
    fn = lambda: A.paged_attention(q, kc, vc, meta, out=out)
    ms = time_fn(fn, iters)
    flops = 4 * Hq * D * T * (T + 1) / 2
    nbytes = 2 * T * Hkv * D * 2 + 2 * T * Hq * D * 2
    return _report("attention_prefill_causal", dict(T=T, Hq=Hq, Hkv=Hkv, D=D), ms, nbytes, flops)


def bench_deltanet(T=15000, nk=16, nv=32, dk=128, dv=128, kw=4, iters=3) -> dict:
    """Qwen3-Next linear-attention layer core (conv + gated delta rule) over one long prompt."""
    from .models.config import get_preset
    from .models.deltanet import DeltaNetState
    from .ops.deltanet import deltanet_fwd
    cfg = get_preset("qwen3-next-80b-a3b")
    r = nv // nk
    W = 2 * dk + 2 * r * dv
    d = "cuda"
    qkvz = (torch.randn(T, nk * W, device=d) * 0.5).to(torch.bfloat16)
    conv_w = torch.randn(2 * nk * dk + nv * dv, kw, device=d) * 0.3
    g = -torch.rand(T, nv, device=d) * 0.5
    beta = torch.rand(T, nv, device=d)
    st = DeltaNetState(cfg, 1, d)
    meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T], dtype=torch.int32, device=d),
                        kv_len=torch.tensor([T], dtype=torch.int32, device=d),
                        block_table=torch.zeros(1, 1, dtype=torch.int32, device=d),
                        slot_mapping=torch.zeros(T, dtype=torch.int32, device=d),
                        positions=torch.zeros(T, dtype=torch.int32, device=d), max_q_len=T, max_kv_len=T,
                        is_decode=False, seq_slots=torch.zeros(1, dtype=torch.int32, device=d),
                        seq_fresh=torch.ones(1, dtype=torch.int32, device=d))
    fn = lambda: deltanet_fwd(qkvz, conv_w, g, beta, meta, st, nk, nv, dk, dv, chunked=True)
    ms = time_fn(fn, iters)
    serial = lambda: deltanet_fwd(qkvz, conv_w, g, beta, meta, st, nk, nv, dk, dv, chunked=False)
    ms_serial = time_fn(serial, iters)
    flops = T * nv * dk * dv * 2 * 4
    nbytes = qkvz.numel() * 2 + T * nv * dv * 4
    r = _report("deltanet_prefill", dict(T=T, nk=nk, nv=nv, dk=dk, dv=dv), ms, nbytes, flops)
    r.update({"token_serial_ms": round(ms_serial, 3), "speedup_vs_token_serial": round(ms_serial / ms, 2)})
    return r


def bench_ring(T=16384, E=128, H=4096, I=1408, K=8, tile_e=16, nslots=2, iters=3) -> dict:
    """Streamed prefill ring on one GLM-4.5-Air-shaped fp8 MoE layer held by the CPU engine:
    the ring's host-link rate against a pinned ``cudaMemcpyAsync`` of the same bytes in this
    run, and its copy / compute overlap.  ``ring_ms``: one layer through the ring (device
    time on the compute stream); ``copy_ms``: the same expert copies alone on the ring's
    copy stream; ``compute_ms``: the layer with every expert GPU-resident;
    ``overlap`` = (copy_ms + compute_ms - ring_ms) / min(copy_ms, compute_ms) (1 = the
    shorter of the two fully hidden)."""
    from .ops.quant import quant_fp8_block
    from .tiering.cpu_engine import CpuExpertEngine
    from .tiering.host import HostExperts
    from .tiering.ring import ExpertRing
    g = torch.Generator(device="cuda").manual_seed(0)
    q13, s13, q2, s2 = [], [], [], []
    for e0 in range(0, E, 16):          # quantize on the GPU in slices, keep the host copy
        n = min(16, E - e0)
        a, sa = quant_fp8_block(torch.randn(n, 2 * I, H, device="cuda", generator=g) * 0.02)
        b, sb = quant_fp8_block(torch.randn(n, H, I, device="cuda", generator=g) * 0.02)
        q13.append(a.cpu()); s13.append(sa.cpu()); q2.append(b.cpu()); s2.append(sb.cpu())
    q13, s13, q2, s2 = torch.cat(q13), torch.cat(s13), torch.cat(q2), torch.cat(s2)
    eng = CpuExpertEngine("fp8", q13, q2, s13, s2)
    host = HostExperts(eng, HostExperts.gpu_scales_from_checkpoint("fp8", s13, s2))
    res = M.prepare_experts("fp8", q13.cuda(), q2.cuda(), s13.cuda(), s2.cuda())
    del q13, q2
    ring = ExpertRing("fp8", H, I, tile_e, nslots, "cuda")
    x = (torch.randn(T, H, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    logits = torch.randn(T, E, device="cuda", generator=g)
    ids, w = router_topk(logits, K)
    ws = M.MoEWorkspace(T, K, E, H, I, "cuda")
    nbytes = E * host.expert_bytes()
    # pinned host -> device peak of this box: one copy of the layer's bytes
    src = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    dst = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    peak_ms = time_fn(lambda: dst.copy_(src, non_blocking=True), iters, flush=False)
    del src, dst
    slots = ring.slots[0]

    def copies():
        st = ring.copy_stream
        st.wait_stream(torch.cuda.current_stream())
        for e in range(E):
            host.copy_slot(e, slots, e % tile_e, st)
        torch.cuda.current_stream().wait_stream(st)

    copy_ms = time_fn(copies, iters, flush=False)
    compute_ms = time_fn(lambda: M.fused_moe(x, ids, w, res, ws), iters)
    ring_ms = time_fn(lambda: ring.run_layer(host, x, ids, w, ws), iters)
    out_ring = ring.run_layer(host, x, ids, w, ws).float()
    out_res = M.fused_moe(x, ids, w, res, ws).float()
    rel = float((out_ring - out_res).norm() / out_res.norm())
    host.close()
    eng.close()
    gb = nbytes / 1e9
    r = {"op": "ring_prefill_fp8", "shape": dict(T=T, E=E, H=H, I=I, K=K, tile_e=tile_e, nslots=nslots),
         "layer_gb": round(gb, 3), "pinned_copy_gbs": round(gb / (peak_ms * 1e-3), 1),
         "copy_ms": round(copy_ms, 3), "copy_gbs": round(gb / (copy_ms * 1e-3), 1),
         "copy_frac_of_pinned": round(peak_ms / copy_ms, 3), "compute_ms": round(compute_ms, 3),
         "ring_ms": round(ring_ms, 3), "ring_gbs": round(gb / (ring_ms * 1e-3), 1),
         "ring_frac_of_pinned": round(peak_ms / ring_ms, 3),
         "overlap": round((copy_ms + compute_ms - ring_ms) / min(copy_ms, compute_ms), 3),
         "prefill_tok_s_per_layer": round(T / (ring_ms * 1e-3), 1), "rel_diff_vs_resident": round(rel, 5)}
    return r


def bench_kda(T=15000, nh=32, dk=128, dv=128, kw=4, iters=3) -> dict:
    """Kimi Delta Attention layer core (conv over blocked q|k|v rows + the delta rule with a
    decay per key dim) over one long prompt, Kimi-Linear head shapes."""
    from .models.config import get_preset
    from .models.deltanet import DeltaNetState
    from .ops.deltanet import deltanet_fwd
    cfg = get_preset("kimi-linear-48b-a3b")
    d = "cuda"
    ch = 2 * nh * dk + nh * dv
    qkv = (torch.randn(T, ch, device=d) * 0.5).to(torch.bfloat16)
    conv_w = torch.randn(ch, kw, device=d) * 0.3
    g = -torch.rand(T, nh, dk, device=d) * 0.5
    beta = torch.rand(T, nh, device=d)
    st = DeltaNetState(cfg, 1, d)
    meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T], dtype=torch.int32, device=d),
                        kv_len=torch.tensor([T], dtype=torch.int32, device=d),
                        block_table=torch.zeros(1, 1, dtype=torch.int32, device=d),
                        slot_mapping=torch.zeros(T, dtype=torch.int32, device=d),
                        positions=torch.zeros(T, dtype=torch.int32, device=d), max_q_len=T, max_kv_len=T,
                        is_decode=False, seq_slots=torch.zeros(1, dtype=torch.int32, device=d),
                        seq_fresh=torch.ones(1, dtype=torch.int32, device=d))
    fn = lambda: deltanet_fwd(qkv, conv_w, g, beta, meta, st, nh, nh, dk, dv, blocked=True)
    ms = time_fn(fn, iters)
    flops = T * nh * dk * dv * 2 * 5
    nbytes = qkv.numel() * 2 + g.numel() * 4 + T * nh * dv * 4
    return _report("kda_prefill", dict(T=T, nh=nh, dk=dk, dv=dv), ms, nbytes, flops)


def bench_moe_verify(T: int, E=128, H=4096, I=1408, K=8, iters=10) -> dict:
    """A verification-size MoE layer as the model runs it (GLM-4.5-Air shapes, fp8 experts
    and shared expert): router + permute in one launch, the row gather, the grouped GEMVs
    with the shared expert as one more grid row, the combine.  Bytes = the active experts'
    and the shared expert's weights."""
    from .models.layers import DenseMLP, Linear
    ex = _experts(E, H, I, "fp8")
    w13 = torch.randn(1, 2 * I, H, device="cuda") * 0.02
    w2 = torch.randn(1, H, I, device="cuda") * 0.02
    q13, s13 = quant_fp8_block(w13)
    q2, s2 = quant_fp8_block(w2)
    sh = M.prepare_experts("fp8", q13, q2, s13, s2)
    mlp = DenseMLP(Linear(sh.w13[0], sh.s13[0]), Linear(sh.w2[0], sh.s2[0]), interleaved=True)
    x = (torch.randn(T, H, device="cuda") * 0.5).to(torch.bfloat16)
    gate = (torch.randn(E, H, device="cuda") * 0.02).to(torch.bfloat16)
    ws = M.MoEWorkspace(T, K, E, H, I, x.device)

    def fn():
        ids, w = M.route_decode(x, gate, None, K, "sigmoid", 1, 1, True, 1.0, ws, 0, E)
        return M.fused_moe(x, ids, w, ex, ws, shared_mlp=mlp, permuted=True), ids

    ms = time_fn(lambda: fn(), iters)
    active = torch.unique(fn()[1]).numel()
    nbytes = 3 * H * I * (active + 1)
    return _report("moe_verify_fp8", dict(T=T, E=E, H=H, I=I, K=K, active_experts=active), ms, nbytes,
                   2 * T * (K + 1) * 3 * H * I)


def bench_router_decode(T: int, E=128, H=4096, K=8, iters=20) -> dict:
    """Decode router + permute in one launch (GLM-4.5-Air: 128 experts, sigmoid + bias,
    top-8) for T tokens; bytes = the bf16 gate weights and the tokens."""
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    gate = (torch.randn(E, H, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.randn(E, device="cuda") * 0.01
    ws = M.MoEWorkspace(max(T, 16), K, E, H, 1408, x.device)
    fn = lambda: M.route_decode(x, gate, bias, K, "sigmoid", 1, 1, True, 1.0, ws, 0, E)
    ms = time_fn(fn, iters)
    return _report("router_decode", dict(T=T, E=E, H=H, K=K), ms, E * H * 2 + T * H * 2, 2 * T * E * H)


def bench_rmsnorm(T=16384, H=4096, iters=20) -> dict:
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    r = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    w = torch.ones(H, device="cuda").to(torch.bfloat16)
    fn = lambda: B.rmsnorm(x, w, 1e-6, residual=r)
    ms = time_fn(fn, iters)
    return _report("rmsnorm_residual", dict(T=T, H=H), ms, 4 * T * H * 2, 0)


def _one_rank_group():
    """A 1-rank process group (NCCL) so the fused multi-GPU kernels run on one GPU: their
    peer stores then land in this GPU's own receive buffers."""
    import os
    import socket
    import torch.distributed as dist
    if not dist.is_initialized():
        sk = socket.socket()
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
        sk.close()
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))


def bench_tp_fused(M_=4, N=4096, Kd=6144, iters=20) -> dict:
    """TP decode output projection (GLM-4.5-Air o_proj slice at TP=2): the fused GEMV whose
    epilogue scatters the partial rows to the ranks' receive buffers, then the sum +
    residual + RMSNorm kernel that consumes them."""
    from .models.layers import Linear, RMSNorm
    from .parallel.tp import TPReducer
    _one_rank_group()
    red = TPReducer(16, N, device=torch.device("cuda", 0), mode="fused")
    w, s = quant_fp8_block(torch.randn(N, Kd, device="cuda") * 0.02)
    lin = Linear(w, s)
    norm = RMSNorm(torch.ones(N, device="cuda", dtype=torch.bfloat16), 1e-5)
    x = torch.randn(M_, Kd, device="cuda").to(torch.bfloat16)
    res = torch.randn(M_, N, device="cuda").to(torch.bfloat16)
    fn = lambda: red.linear_scatter(x, lin).finish(res, norm)
    ms = time_fn(fn, iters)
    N_.check_status()
    nbytes = w.numel() + M_ * (Kd + 3 * N) * 2
    out = _report("tp_gemv_scatter_sum_rmsnorm", dict(M=M_, N=N, K=Kd, world=1), ms, nbytes, 2 * M_ * N * Kd)
    # the same work unfused on one GPU: plain GEMV, then residual add + RMSNorm
    out["plain_gemv_ms"] = round(time_fn(lambda: lin(x), iters), 4)
    out["plain_pair_ms"] = round(time_fn(lambda: norm(lin(x), res), iters), 4)
    red.close()
    return out


def bench_ep_fused(T=256, E=32, K=8, H=7168, I=2048, iters=10) -> dict:
    """The expert-parallel MoE layer (dispatch -> grouped GEMM with SwiGLU -> down GEMM whose
    epilogue stores the weighted rows to their source rank -> combine) on one rank."""
    from .ops.router import router_topk, zipf_bias
    from .parallel.comm import PeerGroup
    from .parallel.ep import EPMoE
    _one_rank_group()
    d = torch.device("cuda", 0)
    q13, s13 = quant_fp8_block(torch.randn(E, 2 * I, H, device=d) * 0.02)
    q2, s2 = quant_fp8_block(torch.randn(E, H, I, device=d) * 0.02)
    ex = M.prepare_experts("fp8", q13, q2, s13, s2)
    del q13, q2
    torch.cuda.empty_cache()   # keep only the layer's buffers on the device
    pg = PeerGroup(EPMoE.heap_bytes(E, K, H, T, 1), device=d)
    layer = EPMoE(ex, E, K, max_tokens=T, pg=pg)
    x = torch.randn(T, H, device=d).to(torch.bfloat16)
    ids, w = router_topk(torch.randn(T, E, device=d) + zipf_bias(E, 1.1, seed=7).to(d), K, "softmax")
    fn = lambda: layer.forward(x, ids, w)
    ms = time_fn(fn, iters)
    N_.check_status()
    active = torch.unique(ids).numel()
    nbytes = 3 * H * I * active + T * K * H * 2 * 2
    out = _report("ep_moe_layer_fused", dict(T=T, E=E, K=K, H=H, I=I, world=1, active_experts=active), ms, nbytes,
                  2 * T * K * 3 * H * I)
    pg.close()
    return out


def bench_cpu_bridge(layers=46, T=1, E=8, H=4096, I=256, K=2, reps=20) -> dict:
    """Round trip of the CPU-expert bridges in a CUDA graph of `layers` MoE calls, each a
    small CPU engine call (so the bridge, not the engine, is what is timed):
    host-function bridge (D2H copies -> host function -> H2D copy) against the
    asynchronous bridge (post kernel -> polling worker -> bounded wait kernel)."""
    import time
    from .tiering.cpu_engine import AsyncCpuBridge, CpuBridge, CpuExpertEngine
    g = torch.Generator().manual_seed(1)
    w13 = (torch.randn(E, 2 * I, H, generator=g) / H ** 0.5).to(torch.bfloat16)
    w2 = (torch.randn(E, H, I, generator=g) / I ** 0.5).to(torch.bfloat16)
    eng = CpuExpertEngine("bf16", w13, w2, threads=4)
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    ids = torch.randint(0, E, (T, K), device="cuda", dtype=torch.int32)
    wts = torch.full((T, K), 1.0 / K, device="cuda")
    out = torch.empty(T, H, device="cuda")
    hb = CpuBridge(eng, K, 16)
    ab = AsyncCpuBridge(eng, K, 16)

    def host_fn():
        for _ in range(layers):
            hb.enqueue(x, ids, wts, out, 0, E)

    def async_fn():
        for _ in range(layers):
            ab.post(x, ids, wts)
            ab.wait(out)

    res = {}
    for name, fn in (("host_function", host_fn), ("async", async_fn)):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        gr.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            gr.replay()
            torch.cuda.synchronize()
            ts.append(time.perf_counter() - t0)
        ts.sort()
        res[name + "_us_per_layer"] = round(ts[len(ts) // 2] / layers * 1e6, 2)
        del gr
    N_.check_status()
    ref = eng.forward(x.cpu(), ids.cpu(), wts.cpu())
    res["max_err"] = float((out.cpu() - ref).abs().max())
    res["engine_us_per_call"] = round(ab.stats()["busy_ms"] * 1e3 / max(1, ab.stats()["runs"]), 2)
    ab.close()
    hb.close()
    eng.close()
    return {"op": "cpu_bridge_round_trip", "shape": dict(layers=layers, T=T, E=E, H=H, I=I, K=K), **res}


OPS = {
    "moe_prefill_fp8": lambda a: bench_moe(a.tokens or 8192, "fp8"),
    "moe_prefill_bf16": lambda a: bench_moe(a.tokens or 8192, "bf16"),
    "moe_decode_fp8": lambda a: bench_moe(a.tokens or 4, "fp8"),
    "gemv_fp8": lambda a: bench_gemv(14336, 4096, a.tokens or 4, "fp8"),
    "gemv_fp8_oproj": lambda a: bench_gemv(4096, 12288, a.tokens or 4, "fp8"),
    "gemv_fp8_graph": lambda a: [bench_gemv(n, k, a.tokens or 20, "fp8", graph=True)
                                 for n, k in ((14336, 4096), (4096, 12288))],
    "lm_head_bf16": lambda a: bench_gemv(151552, 4096, a.tokens or 20, "bf16", iters=10),
    "gemm_fp8": lambda a: bench_gemm(a.tokens or 8192, 14336, 4096, "fp8"),
    "gemm_bf16": lambda a: bench_gemm(a.tokens or 8192, 14336, 4096, "bf16"),
    "attention_decode": lambda a: [bench_attn_decode(ql=ql, kv_dtype=kd) for kd in ("bf16", "fp8") for ql in (1, 5)],
    # MTP k=4 verification shape (5 rows per sequence) at several split-KV factors
    "attention_verify": lambda a: [bench_attn_decode(ql=5, splits=sp) for sp in (4, 8, 9, 16, 18)],
    "mla_decode": lambda a: bench_mla_decode(),
    "attention_prefill": lambda a: bench_attn_prefill(min(a.tokens or 8192, 16384)),
    "rmsnorm": lambda a: bench_rmsnorm(),
    "moe_verify_fp8": lambda a: [bench_moe_verify(t) for t in ((a.tokens,) if a.tokens else (10, 20))],
    "router_decode": lambda a: [bench_router_decode(t) for t in ((a.tokens,) if a.tokens else (4, 20, 32))],
    "tp_fused": lambda a: bench_tp_fused(),
    "ep_fused": lambda a: bench_ep_fused(),
    "deltanet_prefill": lambda a: bench_deltanet(T=a.tokens or 15000),
    "kda_prefill": lambda a: bench_kda(T=a.tokens or 15000),
    "ring_prefill": lambda a: [bench_ring(T=t) for t in ((a.tokens,) if a.tokens else (4096, 16384))],
    "cpu_bridge": lambda a: bench_cpu_bridge(),
    "moe_vs_reference": lambda a: [bench_moe_vs_reference(t) for t in a.sizes],
    # the small-M range that speculative verification produces (C x (k + 1) rows), GLM-4.5-Air shapes
    "moe_fp8_smallm": lambda a: [bench_moe(t, "fp8") for t in (4, 8, 16, 17, 20, 24, 32, 40, 64)],
    "linear_fp8_smallm": lambda a: [bench_gemv(14336, 4096, t, "fp8") for t in (4, 16, 17, 20, 32, 40, 64)],
    # Qwen3-Next-shaped packed-4-bit decode MoE (512 experts top-10, H 2048, I 512)
    "moe_decode_mxfp4": lambda a: [bench_moe(t, "mxfp4", E=512, H=2048, I=512, K=10) for t in (1, 4, 16)],
    "moe_decode_nvfp4": lambda a: [bench_moe(t, "nvfp4", E=512, H=2048, I=512, K=10) for t in (1, 4, 16)],
    "moe_w8a8": lambda a: [bench_moe_w8a8(t) for t in a.sizes if t > G.GEMV_MAX_M],
}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="all", choices=["all"] + list(OPS))
    ap.add_argument("--tokens", type=int, default=None, help="token count of the prefill ops (op default)")
    ap.add_argument("--sizes", default="1,4,16,512,2048,8192",
                    help="token counts of the moe_vs_reference sweep")
    a = ap.parse_args(argv)
    a.sizes = [int(t) for t in a.sizes.split(",")]
    torch.manual_seed(0)
    for name in (OPS if a.op == "all" else [a.op]):
        if a.op == "all" and name == "moe_vs_reference" and not _REF_ROOT.is_dir():
            continue
        r = OPS[name](a)
        for line in (r if isinstance(r, list) else [r]):
            print(json.dumps(line), flush=True)
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
