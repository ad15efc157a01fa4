"""Tensor-parallel decode step: the same TP model with its output-projection reduction
done three ways — ``fused`` (GEMV epilogue scatters each rank's partial rows over
NVLink, the next RMSNorm sums them), ``p2p`` (one-shot P2P all-reduce kernel) and
``nccl`` (NCCL all-reduce, eager) — timed through the engine.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29513 -m vllm_xtu_moe_b200.parallel.tp_bench [--layers 46]

Per mode: C requests with P-token prompts are prefilled, then ``--steps`` decode steps
are timed with CUDA events on the launching stream (max over ranks); one JSON line per
mode on rank 0.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..engine import LLM, SamplingParams
from ..engine.runner import RunnerConfig
from ..models.config import get_preset
from .groups import init_distributed
from .tp import TPReducer, TPRowLinear, build_tp_model


def _set_mode(model, reducer: TPReducer) -> None:
    for l in model.layers + [mt.layer for mt in model.mtp]:
        l.reduce = reducer
        o = getattr(l.attn, "o", None)
        if o is None:
            continue
        base = o.lin if isinstance(o, TPRowLinear) else o
        l.attn.o = TPRowLinear(base, reducer) if reducer.mode == "fused" else base


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="glm-4.5-air")
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--concurrency", type=int, default=4)
    ap.add_argument("--prompt-len", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--modes", default="fused,p2p,nccl")
    a = ap.parse_args(argv)
    rank, world, dev = init_distributed()
    if world < 2:
        raise SystemExit("run with 2 or more ranks (torch.distributed.run --nproc-per-node N)")
    cfg = get_preset(a.model)
    if a.layers:
        cfg = cfg.replace(num_layers=a.layers)
    cfg = cfg.replace(num_mtp_layers=0)
    C, P = a.concurrency, a.prompt_len
    model = None
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist() for _ in range(C)]
    stream = torch.cuda.current_stream()
    for mode in a.modes.split(","):
        red = TPReducer(16384, cfg.hidden_size, device=dev, mode=mode)   # covers a prefill chunk
        if model is None:
            model = build_tp_model(cfg, rank, world, dev, seed=11, reducer=red)
        _set_mode(model, red)
        graphs = mode != "nccl"
        rc = RunnerConfig(block_size=64, max_seqs=C, max_model_len=P + a.steps + 64, max_batched_tokens=16384,
                          use_cuda_graph=graphs, graph_batch_sizes=(1, 2, 4, 8, 16),
                          num_blocks=C * ((P + a.steps + 128) // 64 + 2))
        llm = LLM(model, device=str(dev), runner_config=rc)
        for p in prompts:
            llm.add_request(p, SamplingParams(max_tokens=a.steps + 8, ignore_eos=True))
        while llm.scheduler.waiting or any(r.status.name != "DECODE" for r in llm.scheduler.running):
            llm.step()
        for _ in range(4):       # warm-up decode steps (also capture the graphs)
            llm.step()
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        n = 0
        for _ in range(a.steps):
            plan = llm.scheduler.schedule()
            if plan is None or not plan.is_decode:
                break
            llm.step(plan)
            n += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([e0.elapsed_time(e1) / max(1, n)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            print(json.dumps({"op": "tp_decode_step", "model": cfg.name, "layers": cfg.num_layers, "world": world,
                              "mode": mode, "cuda_graph": graphs, "concurrency": C, "context": P, "steps": n,
                              "decode_step_ms": round(t.item(), 3),
                              "decode_tok_s": round(C * 1e3 / t.item(), 1),
                              "fused_reductions": red.fused_calls}), flush=True)
        llm.shutdown()
        del llm
        torch.cuda.synchronize(dev)
        dist.barrier()
        red.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
