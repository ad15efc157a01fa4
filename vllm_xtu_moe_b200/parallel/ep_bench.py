"""Expert-parallel MoE layer sweep (the single-layer EP configuration): hidden 7168,
256 routed experts top-8 + 1 shared expert, SwiGLU intermediate 2048, fp8 e4m3
weights with 128x128 block scales, activations N(0, 1), router logits N(0, 1) plus a
seeded Zipf(1.1) per-expert bias.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port 29511 -m vllm_xtu_moe_b200.parallel.ep_bench [--tokens 1,8,64,512,4096,8192]

For each tokens-per-rank value it times (CUDA events on the launching stream, after
warm-up, max over ranks) the fused P2P layer and the all-to-all (NCCL) baseline, and
prints one JSON line per size with the roofline: the slowest of the FLOPs at the
measured bf16 GEMM rate (the fp8 weights are widened to bf16 on chip), the bytes that
must cross NVLink at 770 GB/s per direction, and the active experts' weight bytes at
the measured HBM bandwidth.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from ..kernel_bench import peaks
from ..ops import basic as B
from ..ops import gemm as G
from ..ops.quant import quant_fp8_block
from ..ops.router import router_topk, zipf_bias
from .comm import PeerGroup
from .ep import EPMoE
from .groups import init_distributed

NVLINK_GBS = 770.0     # measured peer copy, per direction per GPU


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,8,64,512,4096,8192")
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    rank, world, dev = init_distributed()
    if world < 2:
        raise SystemExit("run with 2 or more ranks (torch.distributed.run --nproc-per-node N)")
    E, K, H, I = a.experts, a.top_k, a.hidden, a.inter
    El = E // world
    sizes = [int(t) for t in a.tokens.split(",")]
    Tmax = max(sizes)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    # this rank's experts only (random init, quantized per 128x128 block)
    w13 = torch.randn(El, 2 * I, H, device=dev, generator=g) * 0.02
    q13, s13 = quant_fp8_block(w13)
    del w13
    w2 = torch.randn(El, H, I, device=dev, generator=g) * 0.02
    q2, s2 = quant_fp8_block(w2)
    del w2
    from ..ops.moe import prepare_experts
    ex = prepare_experts("fp8", q13, q2, s13, s2)
    sh_gu, sh_gu_s = quant_fp8_block(torch.randn(2 * I, H, device=dev, generator=g) * 0.02)
    sh_dn, sh_dn_s = quant_fp8_block(torch.randn(H, I, device=dev, generator=g) * 0.02)
    gate = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    bias = zipf_bias(E, 1.1, seed=7).to(dev)
    torch.cuda.empty_cache()
    pg = PeerGroup(EPMoE.heap_bytes(E, K, H, Tmax, world), device=dev)
    layer = EPMoE(ex, E, K, max_tokens=Tmax, pg=pg)
    pk = peaks()

    def shared(x):
        return G.linear(B.silu_mul(G.linear(x, sh_gu, sh_gu_s)), sh_dn, sh_dn_s)

    def timeit(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        ts = []
        for _ in range(a.iters):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        ts.sort()
        t = torch.tensor([ts[len(ts) // 2]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    for T in sizes:
        x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
        logits = torch.randn(T, E, device=dev, generator=g) + bias
        ids, w = router_topk(logits, K, "softmax")
        fused = timeit(lambda: layer.forward(x, ids, w, shared=shared(x)))
        coll = timeit(lambda: layer.forward_collective(x, ids, w, shared=shared(x)))
        # roofline (per rank): routed pairs computed here ~ T*K on average
        all_ids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(all_ids, ids.contiguous())
        active = torch.unique(torch.cat(all_ids).view(-1))
        mine = ((active // El) == rank).sum().item()
        flops = 2 * T * K * 3 * H * I + 2 * T * 3 * H * I
        t_flop = flops / (pk["bf16_tflops"] * 1e12)
        remote = T * K * (world - 1) / world
        t_link = (remote * H * 2) / (NVLINK_GBS * 1e9)          # each direction carries one copy
        t_hbm = (mine + 1) * 3 * H * I / (pk["hbm_gbs"] * 1e9)
        roof = max(t_flop, t_link, t_hbm) * 1e3
        if rank == 0:
            print(json.dumps({"op": "ep_moe_layer", "world": world, "tokens_per_rank": T, "E": E, "K": K, "H": H,
                              "I": I, "fused_ms": round(fused, 4), "nccl_ms": round(coll, 4),
                              "speedup_vs_nccl": round(coll / fused, 2), "roofline_ms": round(roof, 4),
                              "bound": ["flops", "nvlink", "hbm"][[t_flop, t_link, t_hbm].index(max(t_flop, t_link,
                                                                                                     t_hbm))],
                              "frac_of_roofline": round(roof / fused, 3), "peaks": pk["source"]}), flush=True)
    torch.cuda.synchronize(dev)
    dist.barrier()
    pg.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
