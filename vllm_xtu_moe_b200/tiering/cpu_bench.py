"""CPU expert engine benchmark: this library's engine against the reference's own C++
engine (``xiaotu_moe``, built from its source with its scripts/build_engine_variants.sh,
NO_CUDA=1, into baseline/_ref/xiaotu_moe/build) on the same host, weights and routes.

    python -m vllm_xtu_moe_b200.tiering.cpu_bench [--fmt fp8,mxfp4] [--batch 1,4,16,64,512,2048]
        [--experts 128 --hidden 4096 --inter 1408 --top-k 8] [--threads N] [--reps 5]

Each line: per-layer milliseconds (median of ``--reps`` after one warm-up call) and the
routed-expert TFLOP/s (2 * 3 * H * I per token-expert pair) of both engines at batch size
B, and their ratio.  Routing: uniform random experts per token (as the reference's
scripts/bench_cpu_engine.py does by default).  Both engines get the same thread count.
The reference's published figures for its engine (EPYC 9654, docs/BENCHMARKS.md:164-175):
decode per layer 0.745 ms at B=1; FP8-128 0.73-0.98 TFLOP/s and MXFP4 1.73-2.00 TFLOP/s at
B = 512..8192.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np
import torch

_REF = Path(__file__).resolve().parent.parent.parent / "baseline" / "_ref"


def _ref_module():
    if not (_REF / "xiaotu_moe").is_dir():
        raise FileNotFoundError(f"{_REF}/xiaotu_moe missing (install the reference into baseline/_ref)")
    if str(_REF) not in sys.path:
        sys.path.insert(0, str(_REF))
    import xiaotu_moe
    return xiaotu_moe, xiaotu_moe.load()


def _weights(fmt: str, E: int, H: int, I: int, seed: int = 0, slice_e: int = 8):
    """Random experts quantized to `fmt`, a few experts at a time (the quantizers' fp32
    temporaries of a whole layer would not fit a small host)."""
    from ..ops.quant import quant_fp8_block, quant_mxfp4
    quant = quant_fp8_block if fmt == "fp8" else quant_mxfp4
    g = torch.Generator().manual_seed(seed)
    parts = []
    for e0 in range(0, E, slice_e):
        n = min(slice_e, E - e0)
        p13, s13 = quant(torch.randn(n, 2 * I, H, generator=g) * 0.02)
        p2, s2 = quant(torch.randn(n, H, I, generator=g) * 0.02)
        parts.append((p13, p2, s13, s2))
    return tuple(torch.cat([p[i] for p in parts]) for i in range(4))


def _time(fn, reps: int) -> float:
    fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts) * 1e3


def run(fmt: str, batches: list[int], E: int, H: int, I: int, K: int, threads: int, reps: int) -> list[dict]:
    from .cpu_engine import CpuExpertEngine
    w13, w2, s13, s2 = _weights(fmt, E, H, I)
    ours = CpuExpertEngine(fmt, w13, w2, s13, s2, threads=threads, int8_mode=0 if fmt == "fp8" else 2)
    mod, m = _ref_module()
    cfg = m.MOEConfigV2()
    cfg.num_processes, cfg.process_id, cfg.gpu_id = 1, 0, 0
    cfg.has_gate_proj = True
    cfg.expert_num, cfg.top_k, cfg.hidden_size, cfg.intermediate_size = E, K, H, I
    cfg.max_batch_size, cfg.max_num_seqs = 8192, 256
    cfg.group_min_len, cfg.group_max_len = 10, 8192 + 128
    cfg.activation_type = 0
    cfg.use_gpu_prefill = False
    if fmt == "fp8":
        cfg.groupN = cfg.groupK = cfg.stride = 128
        ref = m.MOE_FP8(cfg, w13.view(torch.uint8).numpy(), w2.view(torch.uint8).numpy(), s13.float().numpy(),
                        s2.float().numpy(), 0, 0)
    else:
        cfg.groupN, cfg.groupK, cfg.stride = 1, 32, 32
        ref = m.MOE_MXFP4(cfg, w13.numpy(), w2.numpy(), s13.view(torch.uint8).numpy(),
                          s2.view(torch.uint8).numpy(), 0, 0)
    rng = np.random.default_rng(7)
    out = []
    for B in batches:
        x = (torch.randn(B, H, generator=torch.Generator().manual_seed(B)) * 0.5).to(torch.bfloat16)
        ids = torch.from_numpy(rng.integers(0, E, size=(B, K)).astype(np.int32))
        wts = torch.from_numpy(rng.uniform(0, 1, size=(B, K)).astype(np.float32))
        y = torch.empty(B, H, dtype=torch.float32)
        xb = x.view(torch.int16).numpy().view(np.uint16)
        yr = np.zeros((B, H), dtype=np.float32)
        ms_ours = _time(lambda: ours.forward(x, ids, wts, out=y), reps)
        ms_ref = _time(lambda: ref.cpu_prefill(B, K, ids.numpy(), wts.numpy(), xb, yr), reps)
        rel = float(np.linalg.norm(y.numpy() - yr) / max(1e-12, np.linalg.norm(yr)))
        flops = 2.0 * 3 * H * I * B * K
        out.append({"op": f"cpu_engine_{fmt}", "B": B, "E": E, "H": H, "I": I, "K": K, "threads": ours.info()["threads"],
                    "ms": round(ms_ours, 3), "tflop_s": round(flops / ms_ours / 1e9, 3),
                    "reference_ms": round(ms_ref, 3), "reference_tflop_s": round(flops / ms_ref / 1e9, 3),
                    "speedup_vs_reference": round(ms_ref / ms_ours, 2), "rel_diff_vs_reference": round(rel, 5),
                    "reference_variant": getattr(mod, "__variant__", "?"), "avx512": ours.info()["avx512"]})
    ours.close()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--fmt", default="fp8,mxfp4")
    ap.add_argument("--batch", default="1,4,16,64,512,2048")
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--hidden", type=int, default=4096)
    ap.add_argument("--inter", type=int, default=1408)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--threads", type=int, default=0, help="0: one per core")
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args(argv)
    threads = a.threads or (os.cpu_count() or 1)
    os.environ.setdefault("XIAOTU_MOE_THREADS", str(threads))
    for fmt in a.fmt.split(","):
        for line in run(fmt, [int(b) for b in a.batch.split(",")], a.experts, a.hidden, a.inter, a.top_k, threads,
                        a.reps):
            print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
