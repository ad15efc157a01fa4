"""Serving benchmark: prefill tok/s & decode tok/s for long synthetic prompts at
concurrency C, with ONE model spread over the N GPUs of one node.

Model: GLM-4.5-Air-style MoE (benchmark config 4: 46 layers, hidden 4096, GQA 96/8 x 128,
partial RoPE, 128 experts top-8 + 1 shared, I=1408, fp8 e4m3 weights with 128x128 block
scales, bf16 activations, one MTP layer; random init).  On N GPUs the model runs tensor
parallel over all N ranks for attention, dense MLP and the shared expert (query / KV
heads and MLP columns split N ways) and expert parallel for the routed experts (rank r
holds experts [r*128/N, (r+1)*128/N)) -- the reference's "TP + EP" layout
(vllm_xiaotu_moe/hybrid_model.py:254-326, 2019-2044) with the partial sums reduced
over NVLink by the library's own kernels: at decode the output projection's GEMV stores
its partial rows into every rank's receive buffer and the next RMSNorm sums them; other
reductions run the one-shot / two-shot peer-memory all-reduce.  NCCL only sets up the
process group.  Every rank holds bit-identical activations, so all ranks sample the same
tokens and take the same engine steps.

One *step* = one serving round: C requests of ``--prompt-len`` uniform random token ids
are submitted together, prefilled (chunked), then decoded for ``--output-len`` tokens each
(greedy; MTP speculative decoding with ``--num-spec`` drafts, k=4 by default as config 4
specifies).  C defaults to 4 per GPU (weak scaling: the work per GPU stays fixed as N
grows).  After the timed steps one round each at C = 1, 2 and 4 gives the concurrency
sweep the metric names.  Weights (~110 GB over the N GPUs) and the KV cache are read
every step, far beyond the 126 MB L2, so no L2 flush is needed between steps.

``value`` is the device-timed aggregate decode throughput (CUDA events on the launching
stream around the decode window, max over ranks); prefill tok/s and the decode step time
are reported beside it.  ``e2e`` repeats the measurement through the public API
(``LLM.generate``) with a host clock, including the host->device copy of each round's
prompts and the device->host read of every sampled token.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
       (N > 1: launch with torch.distributed.run, one process per GPU)
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

METRIC = "prefill tok/s & decode tok/s (15K prompt, C=1/2/4); decode step ms"
BASELINE_DECODE = {1: 29.8, 2: 31.6, 4: 37.2}     # GLM-5.3-Flash decode tok/s, README_EN.md:78-80
BASELINE_PREFILL = {1: 1477.0, 2: 1441.0, 4: 1394.0}
ROOT = os.path.dirname(os.path.abspath(__file__))


WEIGHTS_DTYPE = {("fp8", "fp8"): "fp8 e4m3, 128x128 fp32 block scales (experts and dense)",
                 ("mxfp4", "bf16"): "experts MXFP4 (e2m1, e8m0 scales per 32), dense bf16"}
MODEL_LABEL = {"glm-4.5-air": " (GLM-4.5-Air-style, BASELINE config 4)",
               "qwen3-next-80b-a3b": " (Qwen3-Next-style hybrid, BASELINE config 3)",
               "deepseek-v3": " (DeepSeek-V3 shape, BASELINE config 5)"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="glm-4.5-air")
    ap.add_argument("--concurrency", type=int, default=None, help="requests per round (default 4 per GPU)")
    ap.add_argument("--prompt-len", type=int, default=14500)
    ap.add_argument("--output-len", type=int, default=256)
    ap.add_argument("--num-spec", type=int, default=4, help="MTP draft tokens per step (0 = off)")
    ap.add_argument("--max-batched-tokens", type=int, default=16384)
    ap.add_argument("--no-sweep", action="store_true", help="skip the C = 1/2/4 rounds after the timed steps")
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer layers (invalidates the number)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--tiered", action="store_true",
                    help="experts held once in host DRAM (CPU engine per rank), a hot-expert pool of "
                         "--pool-experts per layer in HBM, prefill through the streamed expert ring, decode "
                         "through the asynchronous CPU bridge with expert deferral (VLLM_EXPERTS_LOAD_DEVICE=cpu)")
    ap.add_argument("--pool-experts", type=int, default=32, help="--tiered: hot-pool experts per MoE layer")
    ap.add_argument("--resident-layers", type=int, default=0,
                    help="--tiered: the first N MoE layers keep their experts GPU-resident (BASELINE config 3: 12)")
    ap.add_argument("--cpu-int8", default="auto", choices=["auto", "on", "off"],
                    help="--tiered: INT8 activations in the CPU engine (XIAOTU_MOE_INT8; MXFP4 experts)")
    ap.add_argument("--kv-cache-dtype", default="bf16", choices=["bf16", "fp8"],
                    help="KV cache storage: bf16, or e4m3 with per-layer scales (decode reads half the bytes)")
    ap.add_argument("--zipf", type=float, default=1.1,
                    help="--tiered: Zipf(s) expert-popularity bias of the router (0 = unbiased random router)")
    return ap.parse_args()


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def reference_arm(args):
    """Run the reference through its public entry point: the vLLM general plugin
    ``vllm_xiaotu_moe`` (pyproject.toml:28-29) installed unmodified in baseline/_ref, which a
    stock ``vllm serve`` imports in every process.  The plugin is imported here exactly as vLLM
    would; when that fails, the real exception is reported on the ``unavailable`` line."""
    rank = int(os.environ.get("RANK", "0"))
    ref = os.path.join(ROOT, "baseline", "_ref")
    line = {"impl": "reference"}
    if not os.path.isdir(os.path.join(ref, "vllm_xiaotu_moe")):
        line["unavailable"] = "reference not installed in baseline/_ref (pip install --target baseline/_ref failed)"
    else:
        sys.path.insert(0, ref)
        try:
            import vllm_xiaotu_moe            # noqa: F401  (the plugin module vLLM loads)
            from vllm_xiaotu_moe import hybrid_model
            hybrid_model.register()
            # the plugin imported and registered: its serving path still needs the patched
            # vLLM tree (patches/, scripts/apply_xtu_patches.sh), its CPU engine .so built by
            # scripts/build_engine_variants.sh and real checkpoints, none of which exist offline
            line["unavailable"] = ("reference plugin imports, but serving needs the patched vLLM tree from "
                                   "patches/ and real checkpoints (not available offline)")
        except Exception as e:                # noqa: BLE001 - report whatever the plugin raised
            line["unavailable"] = (f"reference plugin import failed: {type(e).__name__}: {e} "
                                   f"(it needs the vLLM tree patched by patches/; vLLM 0.22 stock is installed)")
    if rank == 0:
        print(json.dumps(line), flush=True)


def copy_rate(seqs: list[list[int]], n: int = 8) -> float:
    """Benchmark health ("deg"): the share of n-grams of the generated tokens that repeat an
    earlier n-gram of the same sequence (0 = no loops, 1 = a loop from the start)."""
    rep = tot = 0
    for s in seqs:
        seen = set()
        for i in range(len(s) - n + 1):
            g = tuple(s[i:i + n])
            rep += g in seen
            seen.add(g)
            tot += 1
    return rep / tot if tot else 0.0


def main():
    args = parse()
    if os.environ.get("XTU_BENCH_WATCHDOG"):
        import faulthandler
        faulthandler.dump_traceback_later(int(os.environ["XTU_BENCH_WATCHDOG"]), repeat=True)
    if args.impl == "reference":
        return reference_arm(args)
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=600))

    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.config import get_preset
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.ops import _native as N

    cfg = get_preset(args.model)
    C = args.concurrency or 4 * world
    P, O, k = args.prompt_len, args.output_len, args.num_spec
    bs = 64
    max_c = max(C, 4)
    per_seq_blocks = (P + O + 2 * k + 2 + bs - 1) // bs + 1
    rc = RunnerConfig(block_size=bs, max_seqs=max_c, max_batched_tokens=args.max_batched_tokens,
                      max_model_len=P + O + 64, use_cuda_graph=True,
                      graph_batch_sizes=tuple(b for b in (1, 2, 4, 8, 16, 32, 64) if b <= max_c) or (1,),
                      num_spec=k, num_blocks=max_c * per_seq_blocks, kv_cache_dtype=args.kv_cache_dtype)
    t0 = time.time()
    max_rows = max(args.max_batched_tokens, max_c * (1 + k))
    tiering = order = None
    if args.tiered:
        import dataclasses
        from vllm_xtu_moe_b200.config import get_engine_config
        from vllm_xtu_moe_b200.tiering.executor import TieredExperts
        from vllm_xtu_moe_b200.tiering.skew import zipf_order
        moe_layers = [i for i in range(cfg.num_layers + cfg.num_mtp_layers) if cfg.is_moe_layer(i)]
        order = zipf_order(cfg.num_experts, moe_layers, seed=1234) if args.zipf > 0 else None
        # the hot pool seeded with each layer's most popular experts (a PIN table profiled on
        # this traffic); it keeps adapting to the observed routes
        pool = {l: order[l][: args.pool_experts] for l in moe_layers} if order else args.pool_experts
        ec = dataclasses.replace(get_engine_config(), experts_load_device="cpu", moe_async=True, moe_defer=True,
                                 moe_int8=args.cpu_int8)
        threads = max(1, (os.cpu_count() or 1) // world)
        resident = set(moe_layers[: args.resident_layers])
        if isinstance(pool, dict):
            pool = {l: v for l, v in pool.items() if l not in resident}
        tiering = TieredExperts(cfg, device=dev, engine_config=ec, resident_layers=resident, pool_experts=pool,
                                ring=True, max_tokens=args.max_batched_tokens, bridge_tokens=max(64, max_rows),
                                threads=threads)
    if world > 1:
        from vllm_xtu_moe_b200.parallel.tp import TPReducer, build_tp_model
        reducer = TPReducer(max_rows, cfg.hidden_size, device=dev, mode="fused")
        model = build_tp_model(cfg, rank, world, dev, seed=1234, reducer=reducer, num_layers=args.layers,
                               tiering=tiering)
    else:
        reducer = None
        model = build_model(cfg, device=dev, seed=1234, num_layers=args.layers,
                            expert_sink=tiering.expert_sink if tiering is not None else None)
    if order is not None:
        from vllm_xtu_moe_b200.tiering.skew import apply_zipf_router_bias
        apply_zipf_router_bias(model, order, s=args.zipf)
    llm = LLM(model, device=str(dev), runner_config=rc, tiering=tiering)
    torch.cuda.synchronize()
    init_s = time.time() - t0
    # the same prompts on every rank: one model instance serves them (tensor parallel)
    gen = torch.Generator().manual_seed(7919)

    def prompts(c):
        return [torch.randint(0, cfg.vocab_size, (P,), generator=gen).tolist() for _ in range(c)]

    stream = torch.cuda.current_stream()

    def one_round(c):
        """Returns (prefill_ms, decode_ms, decode_steps, accepted, proposed), device-timed."""
        ev0, ev_p, ev1 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        reqs = [llm.add_request(p, SamplingParams(max_tokens=O, ignore_eos=True)) for p in prompts(c)]
        ev0.record(stream)
        prefill_done = False
        dsteps = 0
        while llm.scheduler.has_work():
            plan = llm.scheduler.schedule()
            if plan is None:
                raise RuntimeError("scheduler has work but scheduled nothing")
            if plan.is_decode and not prefill_done:
                ev_p.record(stream)
                prefill_done = True
            llm.step(plan)
            dsteps += int(plan.is_decode)
        if not prefill_done:
            ev_p.record(stream)
        ev1.record(stream)
        torch.cuda.synchronize()
        return (ev0.elapsed_time(ev_p), ev_p.elapsed_time(ev1), dsteps, sum(r.accepted for r in reqs),
                sum(r.proposed for r in reqs))

    def log(msg):
        if rank == 0:
            print(f"[bench +{time.time() - t0:.1f}s] {msg}", file=sys.stderr, flush=True)

    log(f"init {init_s:.1f}s, weights on this rank {llm.model.nbytes() / 2**30:.1f} GiB, kv blocks {rc.num_blocks}, "
        f"world {world}, C {C}, MTP k {k}")
    for i in range(args.warmup):       # warm-up rounds (also capture the decode CUDA graphs)
        a, b, s, acc, prop = one_round(C)
        N.check_status()
        log(f"warmup {i}: prefill {a:.1f} ms, decode {b:.1f} ms / {s} steps, accepted {acc}/{prop}")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    n_launch0 = N.launches()
    pre_ms, dec_ms, dsteps, acc_t, prop_t = [], [], [], 0, 0
    ev_a, ev_b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev_a.record(stream)
    for i in range(args.steps):
        a, b, s, acc, prop = one_round(C)
        log(f"step {i}: prefill {a:.1f} ms, decode {b:.1f} ms / {s} steps, accepted {acc}/{prop}")
        pre_ms.append(a)
        dec_ms.append(b)
        dsteps.append(s)
        acc_t += acc
        prop_t += prop
    ev_b.record(stream)
    torch.cuda.synchronize()
    total_ms = ev_a.elapsed_time(ev_b)
    launches = N.launches() - n_launch0
    clocks = sampler.stop()
    N.check_status()
    if world > 1:
        dist.barrier()

    # ---- concurrency sweep (one device-timed round each; not part of the K timed steps)
    sweep = {}
    if not args.no_sweep:
        for c in (1, 2, 4):
            if c > max_c:
                continue
            a, b, s, acc, prop = one_round(c)
            v = torch.tensor([a, b, float(s)], dtype=torch.float64, device=dev)
            if world > 1:
                dist.all_reduce(v, op=dist.ReduceOp.MAX)
            a, b, s = v.tolist()
            sweep[str(c)] = {"prefill_tok_s": round(c * P / (a / 1e3), 1),
                             "decode_tok_s": round(c * (O - 1) / (b / 1e3), 2),
                             "decode_step_ms": round(b / max(1.0, s), 3),
                             "vs_baseline_decode": round(c * (O - 1) / (b / 1e3) / BASELINE_DECODE[c], 3),
                             "vs_baseline_prefill": round(c * P / (a / 1e3) / BASELINE_PREFILL[c], 3),
                             "mtp_accept_rate": round(acc / prop, 4) if prop else None}
            log(f"sweep C={c}: {sweep[str(c)]}")

    # ---- the same C with plain decoding (no drafts), for the cost of the MTP verification
    mtp_off = None
    if k > 0 and not args.no_sweep:
        llm.set_speculation(0)
        one_round(C)                     # warm-up: captures the plain decode graphs
        a, b, s, _, _ = one_round(C)
        v = torch.tensor([a, b, float(s)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(v, op=dist.ReduceOp.MAX)
        a, b, s = v.tolist()
        mtp_off = {"decode_tok_s": round(C * (O - 1) / (b / 1e3), 2), "decode_step_ms": round(b / max(1.0, s), 3),
                   "prefill_tok_s": round(C * P / (a / 1e3), 1)}
        log(f"C={C} without drafts: {mtp_off}")
        llm.set_speculation(k)

    # ---- e2e through the public API (host clock, includes H2D of prompts and D2H of tokens)
    e2e = None
    deg = None
    if not args.no_e2e:
        e2e_dec, e2e_pre = [], []
        r = llm.runner
        b_in0, b_out0, st0 = r.h2d_bytes, r.d2h_bytes, r.steps
        for _ in range(min(2, max(1, args.steps))):
            ps = prompts(C)
            torch.cuda.synchronize()
            t_a = time.perf_counter()
            outs = llm.generate(ps, SamplingParams(max_tokens=O, ignore_eos=True))
            t_b = time.perf_counter()
            ttft = max(o.ttft_s for o in outs)
            deg = copy_rate([o.token_ids for o in outs])
            e2e_pre.append(C * P / ttft)
            e2e_dec.append(C * (O - 1) / max(1e-9, (t_b - t_a) - ttft))
        v = torch.tensor([min(e2e_dec), min(e2e_pre)], dtype=torch.float64, device=dev)
        if world > 1:      # the slowest rank's view (all ranks serve the same requests)
            dist.all_reduce(v, op=dist.ReduceOp.MIN)
        n_st = max(1, r.steps - st0)
        e2e = {"value": round(v[0].item(), 2), "unit": "tok/s", "prefill_tok_s": round(v[1].item(), 1),
               # counted from the pinned H2D copies (token ids, positions, slots, block tables)
               # and the D2H token reads of the engine steps inside the e2e window
               "h2d_bytes_per_step": round((r.h2d_bytes - b_in0) / n_st),
               "d2h_bytes_per_step": round((r.d2h_bytes - b_out0) / n_st)}

    tier_stats = None
    if tiering is not None:
        tier_stats = tiering.stats(hit_rate=True)
        if tiering.ring is not None:
            tier_stats["ring_gib_streamed"] = round(tiering.ring.copied_bytes / 2**30, 1)

    # ---- aggregate over ranks: every rank serves the same C requests; take the slowest
    mean_pre = sum(pre_ms) / len(pre_ms)
    mean_dec = sum(dec_ms) / len(dec_ms)
    step_ms = total_ms / args.steps
    vals = torch.tensor([mean_pre, mean_dec, step_ms, sum(dsteps) / len(dsteps)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    mean_pre, mean_dec, step_ms, avg_dsteps = vals.tolist()
    decode_tok_s = C * (O - 1) / (mean_dec / 1e3)
    prefill_tok_s = C * P / (mean_pre / 1e3)
    if rank == 0:
        base = BASELINE_DECODE.get(C)
        line = {
            "metric": METRIC, "value": round(decode_tok_s, 2), "unit": "tok/s (decode, aggregate)",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 2),
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": round(decode_tok_s / base, 3) if base else None,
            "dtype": "bf16", "weights_dtype": WEIGHTS_DTYPE.get((cfg.expert_fmt, cfg.dense_fmt),
                                                                f"experts {cfg.expert_fmt}, dense {cfg.dense_fmt}"),
            "data": "synthetic (uniform random token ids, random-init weights)",
            "prefill_tok_s": round(prefill_tok_s, 1),
            "prefill_vs_baseline": round(prefill_tok_s / BASELINE_PREFILL[C], 3) if C in BASELINE_PREFILL else None,
            "deg": None if deg is None else round(deg, 4),
            "decode_step_ms": round(mean_dec / max(1.0, avg_dsteps), 3),
            "mtp_accept_rate": round(acc_t / prop_t, 4) if prop_t else None,
            "tokens_per_decode_step": round(C * (O - 1) / max(1.0, avg_dsteps), 3),
            "by_concurrency": sweep,
            "mtp_off": mtp_off,
            "config": {"model": cfg.name + MODEL_LABEL.get(args.model, ""), "global_batch": C,
                       "concurrency": C, "concurrency_per_gpu": C / world, "seq_len": P, "output_len": O,
                       "parallelism": (f"tp{world}+ep{world}" if world > 1 else "single GPU (tp1, ep1)"),
                       "collectives": ("library peer-memory kernels over NVLink (fused decode o_proj -> "
                                       "RMSNorm reduction, one-/two-shot all-reduce); NCCL for set-up only"
                                       if world > 1 else "none"),
                       "weights": f"experts {cfg.expert_fmt}, dense {cfg.dense_fmt}, block 128x128",
                       "experts_placement": (
                           f"{args.resident_layers} MoE layers GPU-resident, the others in "
                           f"host DRAM once per rank (CPU engine, {tiering.threads} threads, INT8 activations "
                           f"{args.cpu_int8}), hot pool "
                           f"{args.pool_experts}/{cfg.num_experts} experts per layer in HBM, prefill through the "
                           f"streamed expert ring, decode via the async CPU bridge with deferral; router "
                           f"Zipf({args.zipf}) popularity bias" if tiering is not None
                           else "GPU-resident (all experts fit in HBM)"),
                       "mtp_draft_tokens": k, "max_batched_tokens": args.max_batched_tokens,
                       "kv_cache_dtype": args.kv_cache_dtype,
                       "l2": "inputs larger than L2 (weights + KV cache read every step); no flush",
                       "layers": args.layers or cfg.num_layers},
            "clocks": clocks, "e2e": e2e, "gpu_launches": launches, "init_s": round(init_s, 1),
        }
        if tiering is not None:
            line["tiering"] = tier_stats
        if args.layers:
            line["invalid"] = "debug run with fewer layers"
        print(json.dumps(line), flush=True)
    llm.shutdown()
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        if reducer is not None:
            reducer.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    main()
