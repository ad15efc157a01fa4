"""Multi-process paths: expert-parallel MoE (collective baseline on gloo/CPU; fused P2P
path on 2 GPUs), the P2P all-reduce, and a bounded barrier whose peer never comes."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_xtu_moe_b200.ops import moe as M
from vllm_xtu_moe_b200.ops.quant import quant_fp8_block


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, backend):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    from datetime import timedelta
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(rank)
        kw["device_id"] = torch.device("cuda", rank)
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60), **kw)


def _layer(E, H, I, fmt, seed=0):
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    if fmt == "fp8":
        q13, s13 = quant_fp8_block(w13)
        q2, s2 = quant_fp8_block(w2)
        return q13, q2, s13, s2
    return w13.to(torch.bfloat16), w2.to(torch.bfloat16), None, None


def _inputs(T, E, K, H, rank, seed=1):
    g = torch.Generator().manual_seed(seed + rank)
    x = (torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand(T, K, generator=g)
    return x, ids, (w / w.sum(1, keepdim=True)).float()


# ----------------------------------------------------------------------------- CPU (gloo)
def _collective_worker(rank, world, port):
    from vllm_xtu_moe_b200.parallel.ep import EPMoE, shard_experts
    _init(rank, world, port, "gloo")
    E, H, I, K, T = 8, 64, 128, 2, 7 + rank
    w13, w2, s13, s2 = _layer(E, H, I, "bf16")
    ex = shard_experts("bf16", w13, w2, s13, s2, rank, world, "cpu")
    layer = EPMoE(ex, E, K, max_tokens=16)
    x, ids, w = _inputs(T, E, K, H, rank)
    y = layer.forward_collective(x, ids, w).float()
    full = M.prepare_experts("bf16", w13, w2)
    ref = M.moe_ref(x, ids, w, full).float()
    err = (y - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item() + 1e-3, err
    dist.destroy_process_group()


def test_ep_collective_baseline_gloo():
    mp.spawn(_collective_worker, args=(2, _port()), nprocs=2)


# ----------------------------------------------------------------------------- GPU (2 ranks)
def _need_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


def _ep_worker(rank, world, port, fmt, T):
    from vllm_xtu_moe_b200.ops import _native as N
    from vllm_xtu_moe_b200.parallel.comm import PeerGroup
    from vllm_xtu_moe_b200.parallel.ep import EPMoE, shard_experts
    _init(rank, world, port, "nccl")
    d = torch.device("cuda", rank)
    E, H, I, K = 16, 512, 256, 4
    w13, w2, s13, s2 = _layer(E, H, I, fmt)
    ex = shard_experts(fmt, w13, w2, s13, s2, rank, world, d)
    cap = 64
    pg = PeerGroup(EPMoE.heap_bytes(E, K, H, cap, world), device=d)
    layer = EPMoE(ex, E, K, max_tokens=cap, pg=pg)
    full = M.prepare_experts(fmt, w13.to(d), w2.to(d), None if s13 is None else s13.to(d),
                             None if s2 is None else s2.to(d))
    for it in range(3):                                  # repeated calls reuse every buffer
        x, ids, w = _inputs(T, E, K, H, rank, seed=10 * it)
        x, ids, w = x.to(d), ids.to(d), w.to(d)
        sh = (torch.randn(T, H, device=d) * 0.1).to(torch.bfloat16)
        y = layer.forward(x, ids, w, shared=sh).float()
        yc = layer.forward_collective(x, ids, w, shared=sh).float()
        ref = M.fused_moe(x, ids, w, full, shared=sh).float()
        torch.cuda.synchronize(d)
        N.check_status(d)
        tol = 2e-2 * ref.abs().max().item() + 1e-3
        assert (y - ref).abs().max().item() <= tol, (it, (y - ref).abs().max().item())
        assert (yc - ref).abs().max().item() <= tol
    pg.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("fmt,T", [("bf16", 5), ("fp8", 37), ("fp8", 64)])
def test_ep_fused_matches_single_gpu(fmt, T):
    _need_two_gpus()
    mp.spawn(_ep_worker, args=(2, _port(), fmt, T), nprocs=2)


def _allreduce_worker(rank, world, port):
    from vllm_xtu_moe_b200.ops import _native as N
    from vllm_xtu_moe_b200.parallel.comm import P2PAllReduce, PeerGroup
    _init(rank, world, port, "nccl")
    d = torch.device("cuda", rank)
    pg = PeerGroup(1 << 22, device=d)
    ar = P2PAllReduce(pg, 1 << 16, torch.bfloat16)
    for n in (8, 4096, 1 << 16):
        x = (torch.arange(n, device=d) % 97).to(torch.bfloat16) * (rank + 1)
        y = ar(x)
        torch.cuda.synchronize(d)
        N.check_status(d)
        exp = (torch.arange(n, device=d) % 97).float() * sum(r + 1 for r in range(world))
        assert torch.equal(y.float(), exp.to(torch.bfloat16).float()), n
    pg.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_p2p_allreduce():
    _need_two_gpus()
    mp.spawn(_allreduce_worker, args=(2, _port()), nprocs=2)


def _timeout_worker(rank, world, port):
    from vllm_xtu_moe_b200.ops import _native as N
    from vllm_xtu_moe_b200.parallel.comm import PeerGroup
    _init(rank, world, port, "nccl")
    d = torch.device("cuda", rank)
    pg = PeerGroup(1 << 20, device=d, timeout_ns=300_000_000)
    pg.barrier()                          # both ranks: passes
    torch.cuda.synchronize(d)
    N.check_status(d)
    if rank == 0:                         # rank 1 never arrives at this one
        pg.barrier()
        torch.cuda.synchronize(d)         # returns after the bounded wait, context intact
        with pytest.raises(RuntimeError, match="peer"):
            N.check_status(d)             # raises and resets the status word
        assert torch.ones(4, device=d).sum().item() == 4.0
    dist.barrier()
    pg.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
def test_peer_barrier_times_out_instead_of_hanging():
    _need_two_gpus()
    mp.spawn(_timeout_worker, args=(2, _port()), nprocs=2)
