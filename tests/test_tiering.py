"""Expert tiering: swap policy, XTUP tables, planner (CPU); route split, CPU bridge,
hot-expert pool, prefill ring and the tiered executor against the all-GPU MoE (GPU)."""
import inspect
import struct

import pytest
import torch

from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
from vllm_xtu_moe_b200.ops import _native as N
from vllm_xtu_moe_b200.ops import moe as M
from vllm_xtu_moe_b200.ops.quant import quant_fp8_block
from vllm_xtu_moe_b200.tiering import planner as PL
from vllm_xtu_moe_b200.tiering.policy import load_pin_table, plan_swap, save_pin_table, table_from_counts


# ----------------------------------------------------------------------------- policy
def test_plan_swap_evicts_coldest_and_loads_hottest():
    res = [0, 1, 2, 3]
    counts = {0: 10, 1: 0, 2: 5, 3: 7, 8: 50, 9: 3}
    ev, ld = plan_swap(res, counts, 4, maxswap=2)
    # exact: victims (1:0) then (2:5); candidates 8:50, 9:3 -> 8 replaces 1; 9 (3) is not > 5*1.25
    assert ev == [1] and ld == [8]


def test_plan_swap_hysteresis_and_rate_limit():
    res = [0, 1, 2, 3, 4, 5, 6, 7]
    counts = {e: 10 for e in res} | {20: 12, 21: 12, 22: 30, 23: 40, 24: 50}
    ev, ld = plan_swap(res, counts, 8, hyst=0.25)     # default rate limit: nslots // 4 = 2
    assert len(ev) == 2 and ld == [24, 23]
    ev, ld = plan_swap(res, counts, 8, hyst=0.25, maxswap=5)
    assert ld == [24, 23, 22] and 20 not in ld and 21 not in ld   # 12 is within 25% of 10
    assert not set(ev) & set(ld)


def test_plan_swap_tie_order_and_empty_pool():
    res = [5, 6, 7, 8]
    counts = {9: 100}
    ev, _ = plan_swap(res, counts, 4, maxswap=1)
    assert ev == [5]                      # oldest resident among ties
    ev, _ = plan_swap(res, counts, 4, maxswap=1, preserve_oldest=True)
    assert ev == [8]                      # newest among ties in prefill windows
    assert plan_swap([], counts, 0) == ([], [])
    assert plan_swap(res, {}, 4) == ([], [])


def test_xtup_round_trip_and_bytes(tmp_path):
    table = {0: [3, 1, 2], 2: [7]}
    p = tmp_path / "t.xtup"
    save_pin_table(p, table, 16)
    raw = p.read_bytes()
    assert raw[:4] == b"XTUP"
    assert struct.unpack_from("<4sIIII", raw) == (b"XTUP", 1, 3, 16, 4)
    assert struct.unpack_from("<HH", raw, 20) == (0, 3)
    assert load_pin_table(p) == table
    p.write_bytes(b"NOPE" + raw[4:])
    with pytest.raises(ValueError):
        load_pin_table(p)


def test_table_from_counts():
    t = table_from_counts({0: [0, 5, 3, 0], 1: [1, 1, 0, 9]}, 2)
    assert t == {0: [1, 2], 1: [3, 0]}


def test_pool_flips_table_last_and_never_frees():
    """The slot map is updated only after the copies have completed (their event), evicted
    experts leave the map before their slots are overwritten, adaptation never blocks the
    host (no synchronize outside flush), and slots are never reallocated."""
    from vllm_xtu_moe_b200.tiering import pool
    adapt = inspect.getsource(pool.LayerPool.maybe_adapt)
    finish = inspect.getsource(pool.LayerPool._finish_swap)
    assert finish.index("self._swap_ev.query()") < finish.index("self.slotmap[e] = s")
    assert adapt.index("self.slotmap[v] = -1") < adapt.index("self._load(e, s)")
    assert ".synchronize()" not in adapt and ".cpu()" not in adapt
    assert "torch.empty(self.E" in adapt and "del " not in adapt and "alloc_expert_slots" not in adapt


# ----------------------------------------------------------------------------- planner
def test_planner_priorities():
    air = get_preset("glm-4.5-air")
    p = PL.plan(air, 178.0)
    moe = [i for i in range(air.num_layers) if air.is_moe_layer(i)]
    assert p.resident_layers == moe and p.free >= 0 and p.staging > 0
    ds = get_preset("deepseek-v3")
    p = PL.plan(ds, 178.0, max_model_len=32768)
    moe = [i for i in range(ds.num_layers) if ds.is_moe_layer(i)]
    assert 0 < len(p.resident_layers) < len(moe)
    mid = moe[len(moe) // 2]
    assert mid in p.resident_layers
    used = p.non_expert + p.kv + p.staging + p.drafter + len(p.resident_layers) * ds.num_experts * PL.expert_bytes(ds)
    used += p.pool_per_layer * len(p.pool_layers) * PL.expert_bytes(ds)
    assert used + p.free + 4 * PL.GiB == p.gpu_bytes
    env = p.to_env(48, 2)
    assert env["XIAOTU_GPF_STAGE_TILE_E"] == "48" and "XIAOTU_MOE_GPU_RESIDENT_LAYERS" in env
    small = PL.plan(ds, 20.0)
    assert small.notes and not small.resident_layers


def test_layer_ranges():
    assert PL._ranges([1, 2, 3, 7, 9, 10]) == "1-3,7,9-10"
    from vllm_xtu_moe_b200.config import parse_layer_list
    assert parse_layer_list("1-3,7,9-10") == {1, 2, 3, 7, 9, 10}


# ----------------------------------------------------------------------------- CPU model through the CPU tier
def _mini(fmt="fp8"):
    return scaled_down(get_preset("glm-4.5-air"), layers=2, hidden=512, experts=16).replace(
        num_heads=8, num_kv_heads=2, moe_intermediate=256, shared_intermediate=256, dense_intermediate=512,
        expert_fmt=fmt, dense_fmt="bf16", num_mtp_layers=0)


def test_cpu_tier_model_matches_resident():
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    cfg = _mini()
    ref = build_model(cfg, device="cpu", seed=2)
    tier = TieredExperts(cfg, device="cpu", resident_layers=set())
    m = build_model(cfg, device="cpu", seed=2, expert_sink=tier.expert_sink)
    tier.attach(m)
    blk_r, blk_t = ref.layers[1].mlp, m.layers[1].mlp
    assert blk_t.experts is None and blk_t.executor is not None
    x = (torch.randn(9, cfg.hidden_size) * 0.5).to(torch.bfloat16)
    a, b = blk_r(x).float(), blk_t(x).float()
    assert (a - b).abs().max().item() <= 2e-2 * a.abs().max().item() + 1e-3


# ----------------------------------------------------------------------------- GPU
_live = []


@pytest.fixture(autouse=True)
def _shutdown_tiers():
    yield
    while _live:
        _live.pop().shutdown()


def _raw_gpu(fmt, E, H, I, seed):
    from vllm_xtu_moe_b200.ops.quant import quant_mxfp4, quant_nvfp4
    g = torch.Generator().manual_seed(seed)
    w13 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    if fmt == "bf16":
        return dict(fmt=fmt, w13=w13.to(torch.bfloat16), w2=w2.to(torch.bfloat16))
    if fmt == "mxfp4":
        p13, s13 = quant_mxfp4(w13)
        p2, s2 = quant_mxfp4(w2)
        return dict(fmt=fmt, w13=p13, w2=p2, s13=s13, s2=s2)
    if fmt == "nvfp4":
        r13 = [quant_nvfp4(w13[e]) for e in range(E)]
        r2 = [quant_nvfp4(w2[e]) for e in range(E)]
        p13, s13, g13 = (torch.stack([r[i] for r in r13]) for i in range(3))
        p2, s2, g2 = (torch.stack([r[i] for r in r2]) for i in range(3))
        return dict(fmt=fmt, w13=p13, w2=p2, s13=s13, s2=s2, gs13=g13, gs2=g2)
    q13, s13 = quant_fp8_block(w13)
    q2, s2 = quant_fp8_block(w2)
    return dict(fmt=fmt, w13=q13, w2=q2, s13=s13, s2=s2)


def _routes(T, E, K, seed, skew=False):
    g = torch.Generator().manual_seed(seed)
    if skew:
        p = torch.tensor([1.0 / (1 + e) ** 1.2 for e in range(E)])
        ids = torch.stack([torch.multinomial(p, K, generator=g) for _ in range(T)])
    else:
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)])
    w = torch.rand(T, K, generator=g)
    return ids.int(), (w / w.sum(1, keepdim=True)).float()


@pytest.mark.gpu
def test_route_split_matches_torch():
    E, T, K = 64, 37, 8
    ids, _ = _routes(T, E, K, 1)
    slotmap = torch.full((E,), -1, dtype=torch.int32)
    for s, e in enumerate([3, 9, 11, 40, 63]):
        slotmap[e] = s
    d = "cuda"
    gi, ci = torch.empty(T, K, dtype=torch.int32, device=d), torch.empty(T, K, dtype=torch.int32, device=d)
    hits = torch.zeros(E, dtype=torch.int32, device=d)
    M.route_split(ids.to(d), slotmap.to(d), 0, gi, ci, hits)
    M.route_split(ids.to(d), slotmap.to(d), 0, gi, ci, hits)
    s = slotmap[ids.long()]
    assert torch.equal(gi.cpu(), torch.where(s >= 0, s, -1))
    assert torch.equal(ci.cpu(), torch.where(s >= 0, -1, ids))
    assert torch.equal(hits.cpu(), 2 * torch.bincount(ids.flatten().long(), minlength=E).int())


def _executor_case(fmt, pool_experts, T, skew=False, ring=True, min_tokens=64, window=0):
    from vllm_xtu_moe_b200.config import EngineConfig
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    E, H, I, K = 32, 512, 256, 4
    cfg = _mini(fmt).replace(num_experts=E, top_k=K, hidden_size=H, moe_intermediate=I)
    raw = _raw_gpu(fmt, E, H, I, 5)
    ec = EngineConfig(stage_tile_e=12, stage_nslots=2, pin_window=window)
    tier = TieredExperts(cfg, device="cuda", engine_config=ec, resident_layers=set(), pool_experts=pool_experts,
                         ring=ring, gpu_prefill_min_tokens=min_tokens, max_tokens=1024)
    _live.append(tier)
    assert tier.expert_sink(1, raw) is None
    cu = lambda k: raw[k].cuda() if k in raw else None
    res = M.prepare_experts(fmt, cu("w13"), cu("w2"), cu("s13"), cu("s2"), cu("gs13"), cu("gs2"))

    class Blk:
        experts = None
        executor = None

    Blk.cfg = cfg
    blk = Blk()

    class Mdl:
        layers = [type("L", (), {"mlp": blk})()]
        mtp = []

    tier.attach(Mdl)
    ids, w = _routes(T, E, K, 7, skew)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(3)) * 0.5).to(torch.bfloat16).cuda()
    sh = (torch.randn(T, H) * 0.1).to(torch.bfloat16).cuda()
    ids, w = ids.cuda(), w.cuda()
    ref = M.fused_moe(x, ids, w, res, shared=sh).float()
    return tier, blk, x, ids, w, sh, ref


def _close(a, b, tol=2e-2):
    err = (a.float() - b.float()).abs().max().item()
    return err <= tol * b.float().abs().max().item() + 1e-3, err


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["bf16", "fp8", "mxfp4", "nvfp4"])
@pytest.mark.parametrize("T", [1, 5, 40])
def test_hybrid_pool_plus_cpu_matches_gpu(fmt, T):
    tier, blk, x, ids, w, sh, ref = _executor_case(fmt, {1: [0, 3, 5, 7, 11, 20, 31]}, T, ring=False)
    y = blk.executor(blk, x, ids, w, sh)
    torch.cuda.synchronize()
    ok, err = _close(y, ref)
    assert ok, err
    assert tier.stats()["hybrid"] == 1
    hits = blk.executor.pool.hits.cpu()
    assert hits.sum().item() == ids.numel()


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["bf16", "fp8"])
def test_cpu_only_bridge_matches_gpu(fmt):
    tier, blk, x, ids, w, sh, ref = _executor_case(fmt, {}, 6, ring=False)
    y = blk.executor(blk, x, ids, w, sh)
    torch.cuda.synchronize()
    ok, err = _close(y, ref)
    assert ok, err
    assert tier.stats()["cpu"] == 1 and blk.executor.bridge.stats()["runs"] == 1


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["bf16", "fp8", "mxfp4", "nvfp4"])
def test_prefill_ring_matches_gpu(fmt):
    tier, blk, x, ids, w, sh, ref = _executor_case(fmt, {}, 300, ring=True, min_tokens=64)
    y = blk.executor(blk, x, ids, w, sh)
    torch.cuda.synchronize()
    ok, err = _close(y, ref)
    assert ok, err
    assert tier.stats()["ring"] == 1
    assert tier.ring.copied_bytes == 32 * tier.executors[0].host.expert_bytes()
    assert y.shape == ref.shape


@pytest.mark.gpu
def test_pool_adapts_to_hot_experts_and_stays_exact():
    tier, blk, x, ids, w, sh, ref = _executor_case("fp8", {1: [20, 21, 22, 23]}, 16, skew=True, ring=False,
                                                   window=2)
    pool = blk.executor.pool
    for step in range(8):
        y = blk.executor(blk, x, ids, w, sh)
        tier.step_done()
        torch.cuda.synchronize()
        ok, err = _close(y, ref)
        assert ok, (step, err)
    pool.flush()
    assert pool.swaps_in > 0
    sm = pool.slotmap.cpu()
    for s, e in enumerate(pool.expert_of):
        assert sm[e].item() == s
    assert (sm >= 0).sum().item() == 4
    assert 0 in pool.expert_of            # the hottest expert of the skewed routing moved in


@pytest.mark.gpu
def test_hybrid_path_graph_replay_matches_eager():
    tier, blk, x, ids, w, sh, ref = _executor_case("fp8", {1: [0, 1, 2, 3, 4, 5]}, 4, ring=False)
    eager = blk.executor(blk, x, ids, w, sh).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        blk.executor(blk, x, ids, w, sh)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = blk.executor(blk, x, ids, w, sh)
    for _ in range(3):
        out.zero_()
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert blk.executor.bridge.stats()["runs"] >= 5
    del g


def test_tiny_mixtral_on_cpu_engine_greedy_matches_eager():
    """The tiny Mixtral workload with every expert on the C++ CPU engine (no GPU): 2
    layers, hidden 256, 4 heads / 2 KV heads at head_dim 64, 8 experts top-2, SwiGLU
    intermediate 512, vocab 1024, bf16 weights N(0, 0.02) seed 0; two 64-token prompts,
    32 greedy tokens, token for token against the PyTorch eager model."""
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    cfg = get_preset("tiny-mixtral")
    ref = build_model(cfg, device="cpu", seed=0, std=0.02)
    tier = TieredExperts(cfg, device="cpu", resident_layers=set())
    m = build_model(cfg, device="cpu", seed=0, std=0.02, expert_sink=tier.expert_sink)
    tier.attach(m)
    assert all(l.mlp.experts is None and l.mlp.executor is not None for l in m.layers)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 1024, (64,), generator=g).tolist() for _ in range(2)]
    sp = SamplingParams(max_tokens=32)

    def rc():
        return RunnerConfig(block_size=16, max_seqs=2, max_model_len=128, max_batched_tokens=256,
                            use_cuda_graph=False)
    want = [o.token_ids for o in LLM(ref, device="cpu", runner_config=rc()).generate(prompts, sp)]
    got = [o.token_ids for o in LLM(m, device="cpu", runner_config=rc()).generate(prompts, sp)]
    tier.shutdown()
    assert got == want


# ----------------------------------------------------------------------------- async bridge + expert deferral
def _defer_case(device, fmt="bf16", layers=3, T=4, pool=None, defer=True):
    from vllm_xtu_moe_b200.config import EngineConfig
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    E, H, I, K = 32, 512, 256, 4
    cfg = _mini(fmt).replace(num_experts=E, top_k=K, hidden_size=H, moe_intermediate=I, num_layers=layers)
    ec = EngineConfig(moe_defer=defer, moe_async=True, moe_async_timeout_ms=5000)
    tier = TieredExperts(cfg, device=device, engine_config=ec, resident_layers=set(), pool_experts=pool or {},
                         ring=False, max_tokens=1024)
    _live.append(tier)
    raws = [_raw_gpu(fmt, E, H, I, 5 + l) for l in range(layers)]
    for l in range(layers):
        assert tier.expert_sink(l, raws[l]) is None

    def blk():
        b = type("Blk", (), {"experts": None, "executor": None, "cfg": cfg})()
        return b

    blocks = [blk() for _ in range(layers)]

    class Mdl:
        pass

    Mdl.layers = [type("L", (), {"mlp": b})() for b in blocks]
    Mdl.mtp = []
    tier.attach(Mdl)
    g = torch.Generator().manual_seed(9)
    xs = [(torch.randn(T, H, generator=g) * 0.5).to(torch.bfloat16) for _ in range(layers)]
    shs = [(torch.randn(T, H, generator=g) * 0.1).to(torch.bfloat16) for _ in range(layers)]
    routes = [_routes(T, E, K, 20 + l) for l in range(layers)]
    return tier, cfg, raws, blocks, xs, shs, routes


def _deferred_expectation(routed, shs):
    """out_0 = sh_0; out_l = sh_l + routed_{l-1}; the last also adds its own routed part."""
    L = len(routed)
    exp = []
    for l in range(L):
        e = shs[l].float() + (routed[l - 1] if l > 0 else 0)
        if l == L - 1:
            e = e + routed[l]
        exp.append(e)
    return exp


def test_deferral_on_host_tensors_follows_the_layer_shift():
    """Host-tensor path of expert deferral: layer l's CPU-expert result lands in layer l+1."""
    tier, cfg, raws, blocks, xs, shs, routes = _defer_case("cpu")
    outs = [b.executor(b, xs[l], routes[l][0], routes[l][1], shs[l]) for l, b in enumerate(blocks)]
    routed = [tier.executors[l].engine.forward(xs[l], routes[l][0], routes[l][1]) for l in range(len(blocks))]
    for l, (o, e) in enumerate(zip(outs, _deferred_expectation(routed, shs))):
        ok, err = _close(o, e)
        assert ok, (l, err)
    assert tier.cpu_pending is None


@pytest.mark.gpu
@pytest.mark.parametrize("defer", [False, True])
def test_async_bridge_layers_match_resident(defer):
    """The asynchronous bridge (post kernel -> worker thread -> bounded wait kernel) over
    three layers, with and without deferral, against all-GPU MoE layers."""
    tier, cfg, raws, blocks, xs, shs, routes = _defer_case("cuda", defer=defer)
    xs = [x.cuda() for x in xs]
    shs = [s.cuda() for s in shs]
    routes = [(i.cuda(), w.cuda()) for i, w in routes]
    outs = [b.executor(b, xs[l], *routes[l], shs[l]) for l, b in enumerate(blocks)]
    torch.cuda.synchronize()
    N.check_status()
    routed = []
    for l, r in enumerate(raws):
        res = M.prepare_experts(r["fmt"], r["w13"].cuda(), r["w2"].cuda())
        routed.append(M.fused_moe(xs[l], *routes[l], res).float())
    exp = (_deferred_expectation(routed, shs) if defer else [shs[l].float() + routed[l] for l in range(len(raws))])
    for l, (o, e) in enumerate(zip(outs, exp)):
        ok, err = _close(o, e)
        assert ok, (l, err)
    st = tier.stats()
    assert st["deferred"] == (2 if defer else 0) and st["async"] == (1 if defer else 3)
    assert tier.defer_pending is None
    bs = tier._async_bridge.stats()
    assert bs["runs"] == 3 and bs["req"] == 3 and bs["done"] == 3


@pytest.mark.gpu
def test_async_bridge_with_pool_and_graph_replay():
    """Deferral with a hot-expert pool in every layer, captured once and replayed: the
    request numbers live on the device, so replays equal the eager run bit for bit."""
    pool = {l: [0, 3, 5, 7, 11] for l in range(3)}
    tier, cfg, raws, blocks, xs, shs, routes = _defer_case("cuda", fmt="fp8", pool=pool)
    xs = [x.cuda() for x in xs]
    shs = [s.cuda() for s in shs]
    routes = [(i.cuda(), w.cuda()) for i, w in routes]

    def run():
        return [b.executor(b, xs[l], *routes[l], shs[l]) for l, b in enumerate(blocks)]

    eager = [o.clone() for o in run()]
    torch.cuda.synchronize()
    N.check_status()
    # pool pairs run in their own layer, only the CPU pairs are deferred; the MoE output
    # is linear in the routing weights, so each part is the layer with the other's zeroed
    cpu_part, pool_part = [], []
    for l, r in enumerate(raws):
        res = M.prepare_experts("fp8", r["w13"].cuda(), r["w2"].cuda(), r["s13"].cuda(), r["s2"].cuda())
        ids, w = routes[l]
        in_pool = torch.isin(ids, torch.tensor(pool[l], device=ids.device))
        pool_part.append(M.fused_moe(xs[l], ids, torch.where(in_pool, w, 0.0), res).float())
        cpu_part.append(M.fused_moe(xs[l], ids, torch.where(in_pool, 0.0, w), res).float())
    exp = _deferred_expectation(cpu_part, [shs[l].float() + pool_part[l] for l in range(3)])
    for l, (o, e) in enumerate(zip(eager, exp)):
        ok, err = _close(o, e)
        assert ok, (l, err)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        outs = run()
    for _ in range(3):
        for o in outs:
            o.zero_()
        g.replay()
    torch.cuda.synchronize()
    N.check_status()
    for o, e in zip(outs, eager):
        assert torch.equal(o, e)
    assert tier._async_bridge.stats()["done"] == 3 + 3 + 3 * 3   # eager, warm-up, three replays
    del g


@pytest.mark.gpu
def test_async_bridge_wait_times_out_and_recovers():
    """A wait whose request nobody computes (worker paused) ends after its time limit with
    a host-timeout status, the context stays usable, and a reset brings the bridge back."""
    tier, cfg, raws, blocks, xs, shs, routes = _defer_case("cuda", layers=1, defer=False)
    ex = tier.executors[0]
    br = tier.async_bridge(cfg.top_k)
    x, (ids, w) = xs[0].cuda(), routes[0]
    ids, w = ids.cuda(), w.cuda()
    out = torch.zeros(x.shape[0], cfg.hidden_size, device="cuda")
    br.pause(True)
    br.timeout_ns = 200_000_000
    br.post(x, ids, w, engine=ex.engine_index)
    br.wait(out)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="host flag wait timed out"):
        N.check_status()
    br.reset()
    br.timeout_ns = 5_000_000_000
    br.post(x, ids, w, engine=ex.engine_index)
    br.wait(out)
    torch.cuda.synchronize()
    N.check_status()
    ref = ex.engine.forward(x.cpu(), ids.cpu(), w.cpu())
    ok, err = _close(out.cpu(), ref)
    assert ok, err


def _tiny_tiered_llm_tokens(ec, graphs: bool):
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    cfg = get_preset("tiny-mixtral")
    tier = TieredExperts(cfg, device="cuda", engine_config=ec, resident_layers=set(), ring=False)
    _live.append(tier)
    m = build_model(cfg, device="cuda", seed=0, std=0.02, expert_sink=tier.expert_sink)
    tier.attach(m)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 1024, (64,), generator=g).tolist() for _ in range(2)]
    rc = RunnerConfig(block_size=64, max_seqs=2, max_model_len=256, max_batched_tokens=256, use_cuda_graph=graphs,
                      graph_batch_sizes=(1, 2))
    llm = LLM(m, device="cuda", runner_config=rc)
    toks = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=24))]
    N.check_status()
    llm.shutdown()
    return toks, tier.stats()


@pytest.mark.gpu
def test_tiny_mixtral_async_bridge_matches_host_function_bridge():
    """Every expert on the CPU engine, decode in CUDA graphs: the asynchronous bridge gives
    the same greedy tokens as the host-function bridge (same engine, same numerics)."""
    from vllm_xtu_moe_b200.config import EngineConfig
    want, st0 = _tiny_tiered_llm_tokens(EngineConfig(), True)
    got, st1 = _tiny_tiered_llm_tokens(EngineConfig(moe_async=True), True)
    assert got == want
    assert st0["async"] == 0 and st1["async"] > 0 and st1["cpu"] == 0


@pytest.mark.gpu
def test_tiny_mixtral_deferral_graphs_match_eager():
    """Expert deferral through the engine: decode replayed from CUDA graphs gives the same
    tokens as eager decode with deferral, and decode steps defer every layer but the last."""
    from vllm_xtu_moe_b200.config import EngineConfig
    eager, st_e = _tiny_tiered_llm_tokens(EngineConfig(moe_defer=True), False)
    graph, st_g = _tiny_tiered_llm_tokens(EngineConfig(moe_defer=True), True)
    assert graph == eager
    assert st_e["deferred"] > 0 and st_e["async"] > st_e["deferred"]   # 2 layers: the last never defers


# ----------------------------------------------------------------------------- host-side fault injection
def test_damaged_pin_tables_are_rejected(tmp_path):
    """A corrupt XTUP table raises a clear error instead of pinning the wrong experts."""
    good = tmp_path / "good.xtup"
    save_pin_table(good, {0: [3, 1], 1: [2]}, n_experts=8)
    assert load_pin_table(good) == {0: [3, 1], 1: [2]}
    raw = good.read_bytes()
    cases = {
        "magic": b"XTUQ" + raw[4:],
        "short header": raw[:10],
        "truncated": raw[:-2],
        "expert range": raw[:-4] + struct.pack("<HH", 1, 9),
        "layer range": raw[:-4] + struct.pack("<HH", 7, 2),
        "duplicate": raw[:-4] + struct.pack("<HH", 0, 3),
    }
    for name, data in cases.items():
        p = tmp_path / f"{name.replace(' ', '_')}.xtup"
        p.write_bytes(data)
        with pytest.raises(ValueError):
            load_pin_table(p)


def test_failing_host_copy_raises(monkeypatch):
    """A host-to-device copy that fails (the copy layer returns an error code, injected by a
    fake) surfaces as an exception from the expert copy, never as a silently stale slot."""
    from vllm_xtu_moe_b200.tiering import host as H
    from vllm_xtu_moe_b200.tiering.cpu_engine import CpuExpertEngine
    E, Hd, I = 4, 256, 128
    g = torch.Generator().manual_seed(1)
    eng = CpuExpertEngine("bf16", (torch.randn(E, 2 * I, Hd, generator=g) / 16).to(torch.bfloat16),
                          (torch.randn(E, Hd, I, generator=g) / 16).to(torch.bfloat16), threads=2)
    hx = H.HostExperts(eng, None, register=False)
    calls = []

    def fake_copy(dst, src, nbytes, stream):
        calls.append(nbytes)
        return -719                      # the error code of a failed cudaMemcpyAsync

    monkeypatch.setattr(H, "_h2d", lambda: fake_copy)

    class _Stream:
        cuda_stream = 0

    dst13 = torch.empty(2 * I, Hd, dtype=torch.bfloat16)
    dst2 = torch.empty(Hd, I, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="cudaMemcpyAsync failed"):
        hx.copy_expert(1, dst13, dst2, None, None, _Stream())
    assert len(calls) == 1
    eng.close()


def test_planner_counts_window_layers_once_per_sequence():
    """MiMo-V2's sliding-window layers hold one window per sequence, so the planned KV grows
    with the context only through its 9 global layers."""
    cfg = get_preset("mimo-v2-flash")
    a = PL.kv_bytes(cfg, 16384, 4)
    b = PL.kv_bytes(cfg, 32768, 4)
    per_tok_full = PL.kv_bytes_per_token(cfg)
    assert per_tok_full == 9 * 4 * (192 + 128) * 2
    assert b - a == per_tok_full * 16384 * 4
    p = PL.plan(cfg, max_model_len=131072, max_seqs=1)
    assert p.kv < 20 * (1 << 30)


def test_pool_hit_share():
    from vllm_xtu_moe_b200.tiering.policy import pool_hits
    assert pool_hits({0: 5, 3: 2, 7: 3}, [3, 7]) == (5, 10)
    assert pool_hits([1, 0, 4, 0], [2]) == (4, 5)
    assert pool_hits({}, [1]) == (0, 0)


@pytest.mark.gpu
@pytest.mark.parametrize("path", ["hybrid", "cpu", "async", "ring"])
def test_expert_parallel_share_on_tiers(path):
    """One expert-parallel rank's share (global experts 16..31 of 32) on the tiers: pairs
    routed to other ranks' experts are skipped by every path (pool split, CPU engine through
    either bridge, streamed ring), and the rank's partial equals the GPU-resident share's."""
    from vllm_xtu_moe_b200.config import EngineConfig
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    fmt, E, H, I, K, lo = "fp8", 32, 512, 256, 4, 16
    cfg = _mini(fmt).replace(num_experts=E, top_k=K, hidden_size=H, moe_intermediate=I)
    raw = _raw_gpu(fmt, E, H, I, 5)
    share = {k: (v[lo:].contiguous() if isinstance(v, torch.Tensor) else v) for k, v in raw.items()}
    ec = EngineConfig(stage_tile_e=6, stage_nslots=2, moe_async=path == "async")
    pool = {1: [3, 17, 20, 29]} if path in ("hybrid", "async") else {}
    tier = TieredExperts(cfg, device="cuda", engine_config=ec, resident_layers=set(), pool_experts=pool,
                         ring=path == "ring", gpu_prefill_min_tokens=32, max_tokens=1024)
    _live.append(tier)
    assert tier.expert_sink(1, share, lo=lo) is None
    cu = lambda k: share[k].cuda() if k in share else None
    res = M.prepare_experts(fmt, cu("w13"), cu("w2"), cu("s13"), cu("s2"))

    class Blk:
        experts = None
        executor = None
        expert_lo = lo

    Blk.cfg = cfg
    blk = Blk()

    class Mdl:
        layers = [type("L", (), {"mlp": blk})()]
        mtp = []

    tier.attach(Mdl)
    T = 48 if path == "ring" else 6
    ids, w = _routes(T, E, K, 9)
    x = (torch.randn(T, H, generator=torch.Generator().manual_seed(4)) * 0.5).to(torch.bfloat16).cuda()
    ids, w = ids.cuda(), w.cuda()
    ref = M.fused_moe(x, ids, w, res, lo=lo).float()
    y = blk.executor(blk, x, ids, w, None)
    torch.cuda.synchronize()
    ok, err = _close(y, ref)
    assert ok, err
    if path == "hybrid":
        assert blk.executor.pool.nslots == 3          # global 17, 20, 29 -> local 1, 4, 13
    assert tier.stats()[path] >= 1


def test_zipf_router_bias_skews_selection():
    """The benchmark's Zipf(1.1) router bias: seeded per-layer popularity order, the hottest
    quarter of the experts takes most routed pairs, selection weights stay the router's."""
    from vllm_xtu_moe_b200.models.model import build_model
    from vllm_xtu_moe_b200.tiering.skew import apply_zipf_router_bias, zipf_order
    cfg = _mini("bf16").replace(num_experts=32, top_k=4)
    m = build_model(cfg, device="cpu", seed=2)
    blk = m.layers[1].mlp
    x = torch.randn(512, cfg.hidden_size).to(torch.bfloat16)
    ids0, _ = blk.route(x)
    order = zipf_order(32, [1], seed=5)
    assert order == zipf_order(32, [1], seed=5) and sorted(order[1]) == list(range(32))
    apply_zipf_router_bias(m, order, s=1.1)
    ids1, w1 = blk.route(x)
    hot = torch.tensor(order[1][:8])
    share = lambda ids: torch.isin(ids, hot).float().mean().item()
    assert share(ids0) < 0.45 and share(ids1) > 0.6, (share(ids0), share(ids1))
    assert torch.allclose(w1.sum(1), torch.ones(512), atol=1e-4) or not cfg.norm_topk_prob
