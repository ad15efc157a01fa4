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


# ----------------------------------------------------------------------------- tensor parallel
def _tp_cfg(name):
    from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
    cfg = get_preset(name)
    if name == "mimo-v2-flash":     # 2 full-attention KV heads, 4 sliding-window ones, window 8
        return scaled_down(cfg, layers=4, hidden=256, experts=8).replace(
            num_heads=4, num_kv_heads=2, swa_num_kv_heads=4, head_dim=64, v_head_dim=32, rotary_dim=32,
            sliding_window=8, moe_intermediate=256, dense_intermediate=512, num_mtp_layers=0, dense_fmt="bf16",
            expert_fmt="bf16")
    return scaled_down(cfg, layers=4 if ("qwen" in name or "kimi" in name) else 2, hidden=256, experts=8).replace(
        num_heads=4, num_kv_heads=2, head_dim=64 if not cfg.is_mla else cfg.head_dim, moe_intermediate=256,
        shared_intermediate=256, dense_intermediate=512, linear_num_key_heads=2, linear_num_value_heads=4,
        linear_key_head_dim=32, linear_value_head_dim=32, q_lora_rank=64 if cfg.is_mla else 0,
        kv_lora_rank=64 if cfg.is_mla else 0, qk_nope_head_dim=32 if cfg.is_mla else 0,
        v_head_dim=32 if cfg.is_mla else 0, rotary_dim=32 if cfg.rotary_dim else None, num_mtp_layers=0,
        dense_fmt="bf16", expert_fmt="bf16")


def _tp_logits(model, device):
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    llm = LLM(model, device=device, runner_config=RunnerConfig(block_size=64 if device != "cpu" else 16, max_seqs=2,
                                                                max_model_len=256, max_batched_tokens=128,
                                                                use_cuda_graph=False))
    for p in ([3, 4, 5, 6, 7, 8, 9, 10, 11], list(range(20, 60))):
        llm.add_request(p, SamplingParams(max_tokens=1))
    plan = llm.scheduler.schedule()
    ids, meta = llm.runner.build_meta(plan)
    rows = torch.tensor([meta.q_start_host[i + 1] - 1 for i in range(meta.num_seqs)], device=model.device)
    _, _, _, logits = llm.runner.forward(ids, meta, rows)
    return logits.float().cpu()


def _tp_cpu_worker(rank, world, port, name):
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.parallel.tp import TPReducer, build_tp_model
    _init(rank, world, port, "gloo")
    cfg = _tp_cfg(name)
    ref = build_model(cfg, device="cpu", seed=4)
    ref.act_dtype = torch.float32
    red = TPReducer(256, cfg.hidden_size, mode="nccl")
    m = build_tp_model(cfg, rank, world, "cpu", seed=4, reducer=red)
    m.act_dtype = torch.float32
    a, b = _tp_logits(ref, "cpu"), _tp_logits(m, "cpu")
    assert red.calls == 2 * cfg.num_layers
    err = (a - b).abs().max().item() / a.abs().max().item()
    assert err < 1e-3, (name, err)
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["glm-4.5-air", "qwen3-next-80b-a3b", "deepseek-v3", "kimi-linear-48b-a3b",
                                  "mimo-v2-flash"])
def test_tensor_parallel_matches_single_rank_cpu(name):
    mp.spawn(_tp_cpu_worker, args=(2, _port(), name), nprocs=2)


def _tp_tiered_cpu_worker(rank, world, port):
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.parallel.tp import TPReducer, build_tp_model
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    _init(rank, world, port, "gloo")
    cfg = _tp_cfg("glm-4.5-air").replace(expert_fmt="fp8")
    ref = build_model(cfg, device="cpu", seed=4)
    ref.act_dtype = torch.float32
    red = TPReducer(256, cfg.hidden_size, mode="nccl")
    tier = TieredExperts(cfg, device="cpu", resident_layers=set(), threads=2)
    m = build_tp_model(cfg, rank, world, "cpu", seed=4, reducer=red, tiering=tier)
    m.act_dtype = torch.float32
    ex = [l.mlp.executor for l in m.layers if getattr(l.mlp, "executor", None) is not None]
    assert ex and all(e.lo == rank * cfg.num_experts // world and e.engine.E == cfg.num_experts // world for e in ex)
    a, b = _tp_logits(ref, "cpu"), _tp_logits(m, "cpu")
    assert sum(e.calls["cpu"] for e in ex) == 0       # host tensors take the engine directly
    err = (a - b).abs().max().item() / a.abs().max().item()
    assert err < 3e-2, err
    tier.shutdown()
    dist.destroy_process_group()


def test_tensor_parallel_with_cpu_tier_matches_single_rank():
    """Each of 2 ranks keeps its half of the routed experts in its own CPU engine (expert
    parallel tiers under tensor-parallel attention); the reduced logits match one resident rank."""
    mp.spawn(_tp_tiered_cpu_worker, args=(2, _port()), nprocs=2)


def _tp_gpu_worker(rank, world, port, mode="p2p"):
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.ops import _native as N
    from vllm_xtu_moe_b200.parallel.tp import TPReducer, build_tp_model
    _init(rank, world, port, "nccl")
    d = torch.device("cuda", rank)
    cfg = _tp_cfg("glm-4.5-air").replace(hidden_size=512, num_heads=8, dense_fmt="fp8", expert_fmt="fp8")
    ref = build_model(cfg, device=d, seed=4)
    red = TPReducer(256, cfg.hidden_size, device=d, mode=mode)
    m = build_tp_model(cfg, rank, world, d, seed=4, reducer=red)
    a, b = _tp_logits(ref, str(d)), _tp_logits(m, str(d))
    torch.cuda.synchronize(d)
    N.check_status(d)
    err = (a - b).abs().max().item() / a.abs().max().item()
    assert err < 5e-2, err
    if mode == "fused":
        # decode steps (<= 16 tokens) take the GEMV -> peer-scatter -> sum-in-norm path; greedy
        # generation through the engine, eager and CUDA-graph decode, matches the one-GPU model
        for graph in (False, True):
            rc = dict(block_size=64, max_seqs=2, max_model_len=256, max_batched_tokens=128, use_cuda_graph=graph)
            n0 = red.fused_calls
            prompts = [[3, 4, 5, 6, 7, 8, 9], list(range(20, 60))]
            sp = SamplingParams(max_tokens=6)
            got = [r.token_ids for r in LLM(m, device=str(d), runner_config=RunnerConfig(**rc)).generate(prompts, sp)]
            want = [r.token_ids for r in LLM(ref, device=str(d), runner_config=RunnerConfig(**rc)).generate(prompts, sp)]
            torch.cuda.synchronize(d)
            N.check_status(d)
            assert red.fused_calls > n0
            same = sum(x == y for g, w in zip(got, want) for x, y in zip(g, w))
            assert same >= 0.8 * sum(len(w) for w in want), (got, want)
    # both ranks hold identical activations -> identical logits
    other = [torch.empty_like(b) for _ in range(world)]
    dist.all_gather_object(other, b)
    assert torch.equal(other[0], other[1])
    red.close()
    dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.multigpu
@pytest.mark.parametrize("mode", ["p2p", "fused"])
def test_tensor_parallel_p2p_matches_single_gpu(mode):
    _need_two_gpus()
    mp.spawn(_tp_gpu_worker, args=(2, _port(), mode), nprocs=2)


# ----------------------------------------------------------------------------- pipeline parallel
def _pp_worker(rank, world, port, name, backend):
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.ops import _native as N
    from vllm_xtu_moe_b200.parallel.pp import PipelineStage, stage_bounds
    _init(rank, world, port, backend)
    gpu = backend == "nccl"
    dev = f"cuda:{rank}" if gpu else "cpu"
    cfg = _tp_cfg(name)
    if cfg.layer_types is not None:
        cfg = cfg.replace(layer_types=(cfg.layer_types * 2)[:5])
    cfg = cfg.replace(num_layers=5)
    if gpu:
        cfg = cfg.replace(hidden_size=512, num_heads=8, dense_fmt="fp8", expert_fmt="fp8")
    full = build_model(cfg, device=dev, seed=4)
    if not gpu:
        full.act_dtype = torch.float32
    stage = PipelineStage(full, rank, world)
    assert (stage.lo, stage.hi) == stage_bounds(5, world, rank) and len(stage.layers) == stage.hi - stage.lo
    bs = 64 if gpu else 16

    def rc():
        return RunnerConfig(block_size=bs, max_seqs=2, max_model_len=256, max_batched_tokens=128,
                            use_cuda_graph=False)
    prompts = [[3, 4, 5, 6, 7, 8, 9], list(range(20, 45))]
    sp = SamplingParams(max_tokens=4)
    got = [r.token_ids for r in LLM(stage, device=dev, runner_config=rc()).generate(prompts, sp)]
    ref = [r.token_ids for r in LLM(full, device=dev, runner_config=rc()).generate(prompts, sp)]
    assert got == ref, (rank, got, ref)   # the same kernels on the same rows: identical tokens

    # micro-batches: a batch through the stages with non-blocking sends, vs one local pass
    llm = LLM(full, device=dev, runner_config=rc())
    caches_ref = llm.runner.caches
    st_caches = stage.allocate_caches(llm.runner.rc.num_blocks, bs, 2, swa_blocks=llm.runner.rc.swa_blocks)
    batches = []
    for p in prompts:
        llm.add_request(p, SamplingParams(max_tokens=1))
    plan = llm.scheduler.schedule()
    ids, meta = llm.runner.build_meta(plan)
    batches.append((ids, meta))
    outs = stage.forward_microbatches(batches, st_caches)
    if stage.last:
        ref_h = full.forward(ids, meta, caches_ref)
        assert torch.equal(outs[0], ref_h)
    if gpu:
        torch.cuda.synchronize()
        N.check_status(torch.device(dev))
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["glm-4.5-air", "mimo-v2-flash"])
def test_pipeline_stages_match_single_rank_cpu(name):
    """Layers cut into 3 stages over gloo ranks give the single-rank tokens (MiMo: with the
    sliding-window layers' bounded pool on every stage)."""
    mp.spawn(_pp_worker, args=(3, _port(), name, "gloo"), nprocs=3)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_pipeline_stages_nccl_match_single_gpu():
    _need_two_gpus()
    mp.spawn(_pp_worker, args=(2, _port(), "glm-4.5-air", "nccl"), nprocs=2)


_ONE_RANK_TP = r'''
import torch
from vllm_xtu_moe_b200.kernel_bench import _one_rank_group
from vllm_xtu_moe_b200.models.layers import Linear, RMSNorm
from vllm_xtu_moe_b200.ops import _native as N
from vllm_xtu_moe_b200.ops.quant import quant_fp8_block
from vllm_xtu_moe_b200.parallel.tp import TPReducer
_one_rank_group()
d = torch.device("cuda", 0)
g = torch.Generator(device=d).manual_seed(3)
H, K = 1024, 2048
red = TPReducer(16, H, device=d, mode="fused")
w, s = quant_fp8_block(torch.randn(H, K, device=d, generator=g) * 0.02)
lin = Linear(w, s)
norm = RMSNorm((torch.rand(H, device=d, generator=g) + 0.5).to(torch.bfloat16), 1e-5)
worst = 0.0
for it, M in enumerate((1, 4, 16, 4, 1)):          # consecutive calls flip the receive parity
    x = torch.randn(M, K, device=d, generator=g).to(torch.bfloat16)
    res = torch.randn(M, H, device=d, generator=g).to(torch.bfloat16)
    y, r = red.linear_scatter(x, lin).finish(res, norm)
    o = lin(x)
    r_ref = (o.float() + res.float()).to(torch.bfloat16)
    y_ref = norm(r_ref.clone())
    y_ref = y_ref[0] if isinstance(y_ref, tuple) else y_ref
    torch.cuda.synchronize()
    N.check_status()
    er = (r.float() - r_ref.float()).abs().max().item() / (r_ref.float().abs().max().item() + 1e-6)
    ey = (y.float() - y_ref.float()).abs().max().item() / (y_ref.float().abs().max().item() + 1e-6)
    worst = max(worst, er, ey)
red.close()
print("WORST", worst, "CALLS", red.fused_calls)
'''


@pytest.mark.gpu
def test_tp_fused_gemv_sum_rmsnorm_on_one_rank():
    """The fused TP decode path (GEMV whose epilogue stores to the ranks' receive slots,
    then sum + residual + RMSNorm) on a 1-rank group, against the plain GEMV and norm;
    successive calls alternate the receive parity."""
    import subprocess
    import sys
    r = subprocess.run([sys.executable, "-c", _ONE_RANK_TP], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    line = [l for l in r.stdout.splitlines() if l.startswith("WORST")][-1].split()
    assert float(line[1]) < 2e-2 and int(line[3]) == 5, line
