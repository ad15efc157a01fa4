"""Profile window around engine steps: builds a preset model, prefills C prompts of P
tokens, warms up, then runs ``--steps`` decode steps between cudaProfilerStart/Stop so
an external profiler started with ``--profile-from-start off`` sees only those steps.

    python -m vllm_xtu_moe_b200.utils.profile_step --model glm-4.5-air --prompt-len 14500 \\
        --concurrency 4 --steps 2 [--layers N] [--graph] [--num-spec K] [--kv-cache-dtype fp8]

``--num-spec K``: the steps are MTP verification steps (K drafts per request; the
drafts of a random model are rejected, so every step verifies K + 1 rows per request).
"""
from __future__ import annotations

import argparse

import torch

from ..engine import LLM, SamplingParams
from ..engine.runner import RunnerConfig
from ..models.config import get_preset


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="glm-4.5-air")
    ap.add_argument("--prompt-len", type=int, default=14500)
    ap.add_argument("--concurrency", type=int, default=4)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--num-spec", type=int, default=0)
    ap.add_argument("--kv-cache-dtype", default="bf16")
    a = ap.parse_args(argv)
    cfg = get_preset(a.model)
    rc = RunnerConfig(block_size=64, max_seqs=a.concurrency, max_batched_tokens=16384,
                      max_model_len=a.prompt_len + 64 + 4 * a.num_spec, use_cuda_graph=a.graph,
                      num_spec=a.num_spec, kv_cache_dtype=a.kv_cache_dtype,
                      graph_batch_sizes=tuple(b for b in (1, 2, 4, 8, 16) if b <= a.concurrency) or (1,))
    llm = LLM(cfg, device="cuda:0", seed=1, runner_config=rc, num_layers=a.layers)
    g = torch.Generator().manual_seed(0)
    for _ in range(a.concurrency):
        llm.add_request(torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).tolist(),
                        SamplingParams(max_tokens=a.steps + 8))
    while llm.scheduler.waiting or any(r.status.name != "DECODE" for r in llm.scheduler.running):
        llm.step()
    for _ in range(3):
        llm.step()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(a.steps):
        llm.step()
    e.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"decode {s.elapsed_time(e) / a.steps:.2f} ms/step ({cfg.num_layers if a.layers is None else a.layers} "
          f"layers, graph={a.graph}, num_spec={a.num_spec}, kv={a.kv_cache_dtype})", flush=True)


if __name__ == "__main__":
    main()
