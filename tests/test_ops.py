"""sm_100a hot-op kernels vs PyTorch fp32 restatements of the same ops."""
import math

import pytest
import torch

from vllm_xtu_moe_b200.ops import basic as B
from vllm_xtu_moe_b200.ops import moe as M
from vllm_xtu_moe_b200.ops import _native as N
from vllm_xtu_moe_b200.ops.attention import AttnMetadata, paged_attention, paged_attention_ref, num_split_workspace
from vllm_xtu_moe_b200.ops.router import router_topk, router_topk_ref, zipf_bias
from vllm_xtu_moe_b200.ops.quant import quant_fp8_block


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).abs().max() / (b.abs().max() + 1e-6)).item()


# ---------------------------------------------------------------- CPU-only checks
def test_router_ref_group_limited():
    torch.manual_seed(0)
    logits = torch.randn(5, 64)
    bias = torch.randn(64) * 0.1
    ids, w = router_topk_ref(logits, 8, "sigmoid", bias, n_group=8, topk_group=4, renorm=True, scale=2.5)
    assert ids.shape == (5, 8)
    assert torch.allclose(w.sum(-1), torch.full((5,), 2.5), atol=1e-5)
    # every chosen expert lies in one of at most 4 groups
    for t in range(5):
        assert len(set((ids[t] // 8).tolist())) <= 4


def test_router_ref_top_k_beyond_kept_groups():
    """top_k larger than the kept groups' experts (8 experts, 4 groups of 2, 2 kept, top 8):
    the kept experts by score, then the others in index order, never an expert twice."""
    torch.manual_seed(1)
    logits = torch.randn(6, 8)
    ids, w = router_topk_ref(logits, 8, "sigmoid", None, n_group=4, topk_group=2, renorm=True)
    for t in range(6):
        assert sorted(ids[t].tolist()) == list(range(8))
        kept = ids[t, :4].tolist()
        assert len(set(e // 2 for e in kept)) == 2
        rest = ids[t, 4:].tolist()
        assert rest == sorted(rest) and not set(rest) & set(kept)


def test_zipf_bias_is_seeded_and_skewed():
    a, b = zipf_bias(256, 1.1, seed=3), zipf_bias(256, 1.1, seed=3)
    assert torch.equal(a, b)
    assert a.max() - a.min() > 3.0


def test_rope_cache_shapes_yarn():
    cs = B.rope_cache(64, 128, 10000.0, scaling={"type": "yarn", "factor": 40, "original_max_position_embeddings": 4096,
                                                  "beta_fast": 32, "beta_slow": 1, "mscale": 1.0,
                                                  "mscale_all_dim": 1.0})
    assert cs.shape == (128, 64) and torch.isfinite(cs).all()


# ---------------------------------------------------------------- GPU kernels
@pytest.mark.gpu
@pytest.mark.parametrize("H", [256, 4096, 7168])
def test_rmsnorm(H):
    torch.manual_seed(0)
    x = torch.randn(37, H, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(37, H, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(H, device="cuda", dtype=torch.bfloat16)
    y, ro = B.rmsnorm(x, w, 1e-6, residual=r)
    yr, rr = B.rmsnorm_ref(x.cpu(), w.cpu(), 1e-6, residual=r.cpu())
    assert torch.equal(ro.cpu(), rr)
    assert rel_err(y.cpu(), yr) < 1e-2
    y2 = B.rmsnorm(x, w, 1e-6, add_one=True)
    assert rel_err(y2.cpu(), B.rmsnorm_ref(x.cpu(), w.cpu(), 1e-6, add_one=True)[0]) < 1e-2


@pytest.mark.gpu
@pytest.mark.parametrize("D,rot,neox,qknorm", [(128, 64, True, False), (64, 64, True, False), (256, 64, True, True),
                                               (64, 64, False, False)])
def test_rope_and_cache(D, rot, neox, qknorm):
    torch.manual_seed(1)
    T, Hq, Hk, bs = 19, 8, 2, 64
    qkv = torch.randn(T, (Hq + 2 * Hk) * D, device="cuda", dtype=torch.bfloat16)
    q = qkv[:, :Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hk) * D].view(T, Hk, D)
    v = qkv[:, (Hq + Hk) * D:].view(T, Hk, D)
    pos = torch.randint(0, 1000, (T,), device="cuda", dtype=torch.int32)
    cs = B.rope_cache(rot, 1024, 10000.0, "cuda")
    kc = torch.zeros(4, Hk, bs, D, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(4 * bs, device="cuda")[:T].int()
    qn = torch.randn(D, device="cuda", dtype=torch.bfloat16) if qknorm else None
    kn = torch.randn(D, device="cuda", dtype=torch.bfloat16) if qknorm else None
    q_ref, k_ref, v_ref = q.clone().cpu(), k.clone().cpu(), v.clone().cpu()
    kc_ref, vc_ref = kc.clone().cpu(), vc.clone().cpu()
    B.rope_and_cache(q, k, v, pos, cs, rot, neox, slot_mapping=slots, k_cache=kc, v_cache=vc, q_norm_w=qn,
                     k_norm_w=kn)
    B.rope_and_cache(q_ref, k_ref, v_ref, pos.cpu(), cs.cpu(), rot, neox, slot_mapping=slots.cpu(), k_cache=kc_ref,
                     v_cache=vc_ref, q_norm_w=qn.cpu() if qn is not None else None,
                     k_norm_w=kn.cpu() if kn is not None else None)
    assert rel_err(q.cpu(), q_ref) < 2e-2
    assert rel_err(k.cpu(), k_ref) < 2e-2
    assert rel_err(kc.cpu(), kc_ref) < 2e-2
    assert torch.equal(vc.cpu(), vc_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("E,K,scoring,ng,tg", [(8, 2, "softmax", 1, 1), (128, 8, "sigmoid", 1, 1),
                                               (256, 8, "sigmoid", 8, 4), (512, 10, "softmax", 1, 1),
                                               (8, 8, "sigmoid", 4, 2)])   # top_k beyond the kept groups
def test_router(E, K, scoring, ng, tg):
    torch.manual_seed(2)
    logits = torch.randn(300, E, device="cuda") + zipf_bias(E).cuda()
    bias = torch.randn(E, device="cuda") * 0.05 if scoring == "sigmoid" else None
    ids, w = router_topk(logits, K, scoring, bias, ng, tg, True, 2.5)
    ids_r, w_r = router_topk_ref(logits.cpu(), K, scoring, bias.cpu() if bias is not None else None, ng, tg, True, 2.5)
    # same expert sets and weights (order within the set may differ)
    s1, o1 = ids.cpu().sort(-1)
    s2, o2 = ids_r.sort(-1)
    assert torch.equal(s1, s2)
    assert torch.allclose(w.cpu().gather(1, o1), w_r.gather(1, o2), atol=1e-4)


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["bf16", "fp8"])
@pytest.mark.parametrize("T,E,K,H,I", [(1, 8, 2, 256, 512), (200, 16, 4, 512, 256), (33, 64, 8, 1024, 384),
                                       (4, 128, 8, 4096, 1408), (16, 128, 8, 1024, 256), (5, 16, 8, 512, 384),
                                       # verification-size batches: the gathered grouped GEMV (17..64 rows)
                                       (20, 128, 8, 4096, 1408), (40, 16, 8, 1024, 256), (64, 8, 8, 512, 384)])
def test_fused_moe(fmt, T, E, K, H, I):
    torch.manual_seed(3)
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device="cuda") / H ** 0.5
    w2 = torch.randn(E, H, I, device="cuda") / I ** 0.5
    if fmt == "fp8":
        q13, s13 = quant_fp8_block(w13)
        q2, s2 = quant_fp8_block(w2)
        ex = M.prepare_experts("fp8", q13, q2, s13, s2)
    else:
        ex = M.prepare_experts("bf16", w13.to(torch.bfloat16), w2.to(torch.bfloat16))
    logits = torch.randn(T, E, device="cuda")
    ids, w = router_topk(logits, K, "softmax")
    shared = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    y = M.fused_moe(x, ids, w, ex, shared=shared, act_limit=7.0)
    torch.cuda.synchronize()
    N.check_status()
    ref = M.moe_ref(x, ids, w, ex, act_limit=7.0) + shared.float()
    assert rel_err(y, ref) < 2e-2
    # shared expert fused into the routed decode GEMV launches (expert 0's weights serve as
    # the shared MLP) vs the same MLP run on its own and added in the combine
    if T <= 16 and H % 128 == 0 and I % 128 == 0:
        from vllm_xtu_moe_b200.models.layers import DenseMLP, Linear
        mlp = DenseMLP(Linear(ex.w13[0], ex.s13[0] if fmt == "fp8" else None),
                       Linear(ex.w2[0], ex.s2[0] if fmt == "fp8" else None), interleaved=True, limit=7.0)
        assert M.shared_fusable(mlp, ex, 7.0)
        ws = M.MoEWorkspace(T, K, E, H, I, x.device)
        for _ in range(2):   # repeated calls reuse the workspace rows of the shared expert
            yf = M.fused_moe(x, ids, w, ex, ws, act_limit=7.0, shared_mlp=mlp)
            ys = M.fused_moe(x, ids, w, ex, ws, act_limit=7.0, shared=mlp(x))
            torch.cuda.synchronize()
            N.check_status()
            assert rel_err(yf, ys.float()) < 1e-2
        sh_ref = M.moe_ref(x, torch.zeros_like(ids[:, :1]), torch.ones_like(w[:, :1]), ex, act_limit=7.0)
        assert rel_err(yf, M.moe_ref(x, ids, w, ex, act_limit=7.0) + sh_ref) < 2e-2
    # tier split: experts [E/2, E) elsewhere -> only [0, E/2) pairs computed here
    half = M.prepare_experts(ex.fmt, *(_slice_raw(ex, fmt, 0, E // 2)))
    y2 = M.fused_moe(x, ids, w, half, lo=0)
    ref2 = M.moe_ref(x, ids, w, half, lo=0, hi=E // 2)
    assert rel_err(y2, ref2) < 2e-2


def _slice_raw(ex, fmt, a, b):
    # rebuild checkpoint layout (gate, up) from the interleaved kernel layout
    if ex.interleaved:
        I = ex.inter
        w = ex.w13[a:b].view(torch.uint8) if fmt == "fp8" else ex.w13[a:b]
        blk = w.reshape(b - a, I // 128, 2, 128, -1)
        w13 = torch.cat([blk[:, :, 0].reshape(b - a, I, -1), blk[:, :, 1].reshape(b - a, I, -1)], dim=1)
        if fmt == "fp8":
            w13 = w13.view(torch.float8_e4m3fn)
            s = ex.s13[a:b]
            nb = s.shape[1]
            sb = s.reshape(b - a, nb // 2, 2, -1)
            s13 = torch.cat([sb[:, :, 0], sb[:, :, 1]], dim=1)
            return w13.contiguous(), ex.w2[a:b].contiguous(), s13.contiguous(), ex.s2[a:b].contiguous()
        return (w13.contiguous(), ex.w2[a:b].contiguous())
    if fmt == "fp8":
        return ex.w13[a:b], ex.w2[a:b], ex.s13[a:b], ex.s2[a:b]
    return ex.w13[a:b], ex.w2[a:b]


@pytest.mark.gpu
def test_embed_from_pinned_host_table():
    tab = torch.randn(5000, 512).to(torch.bfloat16).pin_memory()
    ids = torch.randint(0, 5000, (37,), dtype=torch.int32, device="cuda")
    y = B.embed(ids, tab)
    torch.cuda.synchronize()
    assert y.is_cuda and torch.equal(y.cpu(), tab[ids.long().cpu()])
    with pytest.raises(ValueError):
        B.embed(ids, torch.randn(10, 512).to(torch.bfloat16))     # not pinned


@pytest.mark.gpu
def test_argmax_embed():
    torch.manual_seed(4)
    lg = torch.randn(7, 151552, device="cuda")
    assert torch.equal(B.argmax(lg).cpu(), lg.argmax(-1).int().cpu())
    tab = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (9,), device="cuda", dtype=torch.int32)
    assert torch.equal(B.embed(ids, tab), tab[ids.long()])


def _make_paged(seqs, Hkv, D, Dv, bs=64, device="cuda"):
    """seqs: list of (q_len, kv_len). Returns caches, metadata, q."""
    nblk = sum((kl + bs - 1) // bs for _, kl in seqs) + 2
    kc = torch.randn(nblk, Hkv, bs, D, device=device, dtype=torch.bfloat16)
    vc = torch.randn(nblk, Hkv, bs, Dv, device=device, dtype=torch.bfloat16)
    perm = torch.randperm(nblk).tolist()
    tables, q_start, kv_len = [], [0], []
    for ql, kl in seqs:
        nb = (kl + bs - 1) // bs
        tables.append([perm.pop() for _ in range(nb)])
        q_start.append(q_start[-1] + ql)
        kv_len.append(kl)
    mb = max(len(t) for t in tables)
    bt = torch.zeros(len(seqs), mb, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t)
    T = q_start[-1]
    meta = AttnMetadata(num_seqs=len(seqs), q_start=torch.tensor(q_start, dtype=torch.int32, device=device),
                        kv_len=torch.tensor(kv_len, dtype=torch.int32, device=device), block_table=bt.to(device),
                        slot_mapping=torch.zeros(T, dtype=torch.int32, device=device),
                        positions=torch.zeros(T, dtype=torch.int32, device=device),
                        max_q_len=max(q for q, _ in seqs), max_kv_len=max(kv_len), is_decode=False,
                        q_start_host=q_start, kv_len_host=kv_len)
    return kc, vc, meta, T


@pytest.mark.gpu
@pytest.mark.parametrize("Hq,Hkv,D", [(96, 8, 128), (4, 2, 64), (16, 2, 256), (8, 8, 128), (12, 1, 128)])
@pytest.mark.parametrize("mode", ["prefill", "decode", "decode_split", "spec", "spec_split", "spec2"])
def test_paged_attention(Hq, Hkv, D, mode):
    torch.manual_seed(5)
    if mode == "prefill":
        seqs = [(300, 300), (77, 590), (1, 1), (130, 130)]
    elif mode in ("spec", "spec_split"):
        seqs = [(5, 700), (5, 129), (5, 64)]
    elif mode == "spec2":          # 2 query positions: up to 32 rows per KV head (two 16-row tiles)
        seqs = [(2, 700), (2, 129), (2, 64), (2, 2)]
    else:
        seqs = [(1, 1000), (1, 63), (1, 4097)]
    kc, vc, meta, T = _make_paged(seqs, Hkv, D, D)
    if mode == "decode_split":
        meta.num_splits = 8
    elif mode == "spec_split":
        meta.num_splits = 4
    q = torch.randn(T, Hq, D, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o = paged_attention(q, kc, vc, meta, scale)
    torch.cuda.synchronize()
    N.check_status()
    ref = paged_attention_ref(q.float(), kc.float(), vc.float(), meta, scale)
    err = (o.float() - ref.float()).abs().max().item()
    assert err < 3e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("Hq,Hkv,D,Dv", [(64, 8, 192, 128), (16, 2, 128, 128), (8, 2, 64, 64)])
@pytest.mark.parametrize("mode", ["prefill", "decode", "decode_split", "spec"])
@pytest.mark.parametrize("window,sinks", [(128, True), (200, False), (0, True)])
def test_paged_attention_window_and_sinks(Hq, Hkv, D, Dv, mode, window, sinks):
    """Sliding-window attention with learned per-head sinks (MiMo-style SWA layers; 192/128
    q-k/v head dims) in the prefill, decode, split-decode and multi-token decode forms."""
    torch.manual_seed(11)
    seqs = {"prefill": [(300, 300), (77, 590), (1, 1), (130, 700)], "decode": [(1, 1000), (1, 63), (1, 4097)],
            "decode_split": [(1, 1000), (1, 63), (1, 4097)], "spec": [(3, 700), (3, 129), (3, 64)]}[mode]
    kc, vc, meta, T = _make_paged(seqs, Hkv, D, Dv)
    if mode == "decode_split":
        meta.num_splits = 8
    elif mode == "spec_split":
        meta.num_splits = 4
    q = torch.randn(T, Hq, D, device="cuda", dtype=torch.bfloat16)
    sk = (torch.randn(Hq, device="cuda") * 2.0).float() if sinks else None
    scale = 1.0 / math.sqrt(D)
    o = paged_attention(q, kc, vc, meta, scale, window=window, sinks=sk)
    torch.cuda.synchronize()
    N.check_status()
    ref = paged_attention_ref(q.float(), kc.float(), vc.float(), meta, scale, window=window, sinks=sk)
    err = (o.float() - ref.float()).abs().max().item()
    assert err < 3e-2, err


def test_attention_ref_window_and_sinks_semantics():
    """The restatement itself: a window of 1 returns each query's own value row; a huge
    sink drives the output to zero; window >= context equals full causal attention."""
    torch.manual_seed(2)
    kc, vc, meta, T = _make_paged([(5, 9), (3, 3)], 1, 16, 16, bs=16, device="cpu")
    q = torch.randn(T, 2, 16)
    own = paged_attention_ref(q, kc.float(), vc.float(), meta, 0.25, window=1)
    for b, (ql, kl) in enumerate([(5, 9), (3, 3)]):
        s0 = meta.q_start_host[b]
        for i in range(ql):
            p = kl - ql + i
            blk = int(meta.block_table[b, p // 16])
            assert torch.allclose(own[s0 + i, 0], vc[blk, 0, p % 16].float(), atol=1e-5)
    zero = paged_attention_ref(q, kc.float(), vc.float(), meta, 0.25, sinks=torch.full((2,), 80.0))
    assert zero.abs().max().item() < 1e-6
    full = paged_attention_ref(q, kc.float(), vc.float(), meta, 0.25)
    wide = paged_attention_ref(q, kc.float(), vc.float(), meta, 0.25, window=64)
    assert torch.allclose(full, wide)


@pytest.mark.gpu
def test_paged_attention_long_prefill():
    """4K-token prompts, GQA group 12 (GLM-Air heads), two chunks of one sequence."""
    torch.manual_seed(7)
    seqs = [(4000, 4000), (1500, 6000)]
    kc, vc, meta, T = _make_paged(seqs, 8, 128, 128)
    q = torch.randn(T, 96, 128, device="cuda", dtype=torch.bfloat16)
    o = paged_attention(q, kc, vc, meta, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    N.check_status()
    ref = paged_attention_ref(q, kc, vc, meta, 1 / math.sqrt(128))   # torch on the GPU, fp32 math
    assert (o.float() - ref.float()).abs().max().item() < 3e-2


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["prefill", "decode", "decode1"])
def test_paged_attention_running_max_rescale(mode):
    """Scores that grow along the keys for some heads and shrink for others, so that
    within one warp some rows must rescale O and others must not."""
    torch.manual_seed(8)
    Hq, Hkv, D = 96, 8, 128
    seqs = {"prefill": [(700, 700), (300, 1000)], "decode": [(1, 3000), (4, 900)],
            "decode1": [(1, 3000), (1, 900), (1, 65)]}[mode]
    kc, vc, meta, T = _make_paged(seqs, Hkv, D, D)
    # k[t] = 0.02 * pos(t) * ones + noise  ->  q.k grows (or shrinks) linearly with the key position
    bs = kc.shape[2]
    pos = torch.arange(bs, device="cuda").float()
    for blk_row, (ql, kl) in zip(meta.block_table.tolist(), seqs):
        for j, b in enumerate(blk_row[:(kl + bs - 1) // bs]):
            ramp = (j * bs + pos)[None, :, None] * 0.02
            kc[b] = (ramp + 0.1 * torch.randn(Hkv, bs, D, device="cuda")).to(torch.bfloat16)
    sign = torch.where(torch.arange(Hq, device="cuda") % 3 == 0, -1.0, 1.0)
    q = (sign[None, :, None] * torch.ones(T, Hq, D, device="cuda") + 0.1 * torch.randn(T, Hq, D, device="cuda"))
    q = q.to(torch.bfloat16)
    scale = 1 / math.sqrt(D)
    o = paged_attention(q, kc, vc, meta, scale)
    torch.cuda.synchronize()
    N.check_status()
    ref = paged_attention_ref(q, kc, vc, meta, scale)
    assert (o.float() - ref.float()).abs().max().item() < 3e-2


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 4, 16, 40])
def test_dense_mlp_paths(T):
    """Shared-expert / dense MLP: GEMV path (T <= 16) and tensor-core path vs fp32 reference."""
    from vllm_xtu_moe_b200.models.layers import DenseMLP, Linear
    from vllm_xtu_moe_b200.ops import gemm as G
    torch.manual_seed(10)
    H, I = 1024, 1408
    w13 = torch.randn(2 * I, H, device="cuda") / H ** 0.5
    w2 = torch.randn(H, I, device="cuda") / I ** 0.5
    q13, s13 = quant_fp8_block(w13)
    q2, s2 = quant_fp8_block(w2)
    mlp = DenseMLP(Linear(G.interleave_gate_up(q13.view(torch.uint8)).view(torch.float8_e4m3fn),
                          G.interleave_gate_up_scale(s13)), Linear(q2, s2), True)
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    y = mlp(x)
    torch.cuda.synchronize()
    from vllm_xtu_moe_b200.ops.quant import dequant_fp8_block
    w13d = dequant_fp8_block(q13, s13).to(torch.bfloat16).float()
    w2d = dequant_fp8_block(q2, s2).to(torch.bfloat16).float()
    g = x.float() @ w13d.t()
    h = G.silu_and_mul_clamped(g[:, :I], g[:, I:]).to(torch.bfloat16).float()
    ref = h @ w2d.t()
    assert rel_err(y, ref) < 2e-2


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 4, 16, 20, 32])
@pytest.mark.parametrize("E,K,scoring,ng,tg", [(128, 8, "sigmoid", 1, 1), (256, 8, "sigmoid", 8, 4),
                                               (64, 4, "softmax", 1, 1)])
def test_route_decode_matches_separate_router(T, E, K, scoring, ng, tg):
    """Router + permute in one launch vs logits GEMV -> router_topk -> permute."""
    from vllm_xtu_moe_b200.ops import gemm as G
    torch.manual_seed(11)
    H, I = 1024, 256
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    gate = (torch.randn(E, H, device="cuda") * 0.2).to(torch.bfloat16)   # well-separated scores
    bias = torch.randn(E, device="cuda") * 0.05 if scoring == "sigmoid" else None
    ex = M.prepare_experts("bf16", torch.zeros(E, 2 * I, H, device="cuda", dtype=torch.bfloat16),
                           torch.zeros(E, H, I, device="cuda", dtype=torch.bfloat16))
    assert M.decode_route_ok(x, gate, ex, K, ng)
    ws = M.MoEWorkspace(32, K, E, H, I, x.device)
    for lo, n_local in [(0, E), (E // 4, E // 2)]:
        for _ in range(2):   # the launch counter must be left zeroed
            ids, w = M.route_decode(x, gate, bias, K, scoring, ng, tg, True, 2.5, ws, lo, n_local)
            torch.cuda.synchronize()
            N.check_status()
            logits = G.linear(x, gate, out_dtype=torch.float32)
            ids_r, w_r = router_topk(logits, K, scoring, bias, ng, tg, True, 2.5)
            s1, o1 = ids.sort(-1)
            s2, o2 = ids_r.sort(-1)
            assert torch.equal(s1, s2)
            assert torch.allclose(w.gather(1, o1), w_r.gather(1, o2), atol=1e-4)
            # the permutation: each local pair lands in its expert's segment, once
            seg = ws.seg[: n_local + 1].cpu()
            cnt = torch.bincount((ids.flatten() - lo).clamp(0, n_local)[(ids.flatten() >= lo) &
                                 (ids.flatten() < lo + n_local)].long().cpu(), minlength=n_local)
            assert torch.equal(seg[1:] - seg[:-1], cnt.int())
            rows = ws.perm_slot[: int(seg[-1])].cpu()
            assert sorted(rows.tolist()) == [p for p in range(T * K)
                                             if lo <= int(ids.flatten()[p]) < lo + n_local]
            act = ws.active.cpu()
            assert act[0].item() == int((cnt > 0).sum()) and torch.equal(act[1:1 + act[0]],
                                                                          torch.nonzero(cnt).flatten().int())


@pytest.mark.gpu
@pytest.mark.parametrize("fmt", ["fp8", "bf16"])
@pytest.mark.parametrize("T", [17, 20, 32])
def test_verification_moe_fused_router_gather_shared(fmt, T):
    """A verification-size MoE step (16 < T <= 32 rows): router + permute in one launch, the
    row gather (with the shared expert's token rows appended) and the grouped GEMV with the
    shared expert as one more grid row, against the fp32 reference of routed + shared; also
    the expert-parallel slice (local experts [E/4, 3E/4))."""
    from vllm_xtu_moe_b200.models.layers import DenseMLP, Linear
    torch.manual_seed(12)
    E, K, H, I = 64, 8, 1024, 256
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    gate = (torch.randn(E, H, device="cuda") * 0.2).to(torch.bfloat16)
    w13 = torch.randn(E, 2 * I, H, device="cuda") / H ** 0.5
    w2 = torch.randn(E, H, I, device="cuda") / I ** 0.5
    if fmt == "fp8":
        q13, s13 = quant_fp8_block(w13)
        q2, s2 = quant_fp8_block(w2)
        ex = M.prepare_experts("fp8", q13, q2, s13, s2)
    else:
        ex = M.prepare_experts("bf16", w13.to(torch.bfloat16), w2.to(torch.bfloat16))
    mlp = DenseMLP(Linear(ex.w13[0], ex.s13[0] if fmt == "fp8" else None),
                   Linear(ex.w2[0], ex.s2[0] if fmt == "fp8" else None), interleaved=True, limit=7.0)
    assert M.shared_fusable(mlp, ex, 7.0) and M.decode_route_ok(x, gate, ex, K, 1)
    sh_ref = M.moe_ref(x, torch.zeros(T, 1, dtype=torch.int32, device="cuda"),
                       torch.ones(T, 1, device="cuda"), ex, act_limit=7.0)
    ws = M.MoEWorkspace(32, K, E, H, I, x.device)
    for _ in range(2):   # repeated calls reuse the workspace (rows, counters, shared rows)
        ids, w = M.route_decode(x, gate, None, K, "softmax", 1, 1, True, 1.0, ws, 0, E)
        y = M.fused_moe(x, ids, w, ex, ws, act_limit=7.0, shared_mlp=mlp, permuted=True)
        torch.cuda.synchronize()
        N.check_status()
        assert rel_err(y, M.moe_ref(x, ids, w, ex, act_limit=7.0) + sh_ref) < 2e-2
    # the DenseMLP on its own at this size (one-expert gathered GEMV, two 16-row passes)
    assert rel_err(mlp(x), sh_ref) < 2e-2
    # expert-parallel slice: only pairs of experts [lo, lo + E/2) computed here
    lo, nl = E // 4, E // 2
    half = M.prepare_experts(ex.fmt, *(_slice_raw(ex, fmt, lo, lo + nl)))
    ws2 = M.MoEWorkspace(32, K, nl, H, I, x.device)
    ids, w = M.route_decode(x, gate, None, K, "softmax", 1, 1, True, 1.0, ws2, lo, nl)
    y2 = M.fused_moe(x, ids, w, half, ws2, lo=lo, act_limit=7.0, permuted=True)
    torch.cuda.synchronize()
    N.check_status()
    assert rel_err(y2, M.moe_ref(x, ids, w, half, lo=lo, hi=lo + nl, act_limit=7.0)) < 2e-2


@pytest.mark.gpu
def test_sigmoid_gate_kernels():
    """gate_mul_ (strided gated-GQA output gate) and shared_gate_ (per-token sigmoid of a
    dot product) against fp32 torch."""
    from vllm_xtu_moe_b200.ops.basic import gate_mul_, shared_gate_
    torch.manual_seed(9)
    T, nh, hd = 37, 8, 256
    qg = torch.randn(T, nh, 2 * hd, device="cuda").to(torch.bfloat16)
    o = torch.randn(T, nh, hd, device="cuda").to(torch.bfloat16)
    ref = (o.float() * torch.sigmoid(qg[:, :, hd:].float()))
    gate_mul_(o, qg[:, :, hd:])
    torch.cuda.synchronize()
    assert (o.float() - ref).abs().max().item() < 2e-2
    H = 2048
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    w = (torch.randn(1, H, device="cuda") * 0.02).to(torch.bfloat16)
    y = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    ref = y.float() * torch.sigmoid(x.float() @ w.float().t())
    shared_gate_(y, x, w)
    torch.cuda.synchronize()
    assert (y.float() - ref).abs().max().item() < 2e-2
