"""DeepSeek sparse attention (DSA): the lightning indexer's selection and the absorbed
sparse MLA against an fp32 restatement (expanded K / V, dense attention masked to the
selected tokens); the GPU kernels against the CPU paths; a DSA model end to end."""
import math

import pytest
import torch

from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
from vllm_xtu_moe_b200.models.model import build_model
from vllm_xtu_moe_b200.ops import basic as B
from vllm_xtu_moe_b200.ops import _native as N
from vllm_xtu_moe_b200.ops import dsa as D
from vllm_xtu_moe_b200.ops.attention import AttnMetadata


def _cfg(topk=16):
    return scaled_down(get_preset("deepseek-v3.2"), layers=2, hidden=256, experts=8).replace(
        num_heads=4, q_lora_rank=64, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=32, v_head_dim=32,
        head_dim=64, index_topk=topk, index_n_heads=8, index_head_dim=128, moe_intermediate=128,
        shared_intermediate=128, dense_intermediate=256, rotary_dim=32, rope_scaling=None)


def _meta(T, device="cpu", bs=64, nblocks=None):
    nb = (T + bs - 1) // bs
    perm = torch.randperm(nblocks or nb + 3)[:nb].to(torch.int32)
    return AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T], dtype=torch.int32, device=device),
                        kv_len=torch.tensor([T], dtype=torch.int32, device=device),
                        block_table=perm[None].to(device),
                        slot_mapping=torch.tensor([int(perm[t // bs]) * bs + t % bs for t in range(T)],
                                                  dtype=torch.int32, device=device),
                        positions=torch.arange(T, dtype=torch.int32, device=device), max_q_len=T, max_kv_len=T,
                        is_decode=False, q_start_host=[0, T], kv_len_host=[T]), (nblocks or nb + 3)


def _layer_vs_oracle(device, cfg, T, seed=3, decode=False):
    """Run layer 0 of a DSA model on a T-token prompt and the fp32 oracle (expanded K / V,
    dense attention masked to each query's top-k selection); returns the relative error.
    decode: the prompt's first T - 1 tokens as a prefill step, then token T - 1 alone as a
    decode step (the oracle's last row)."""
    torch.manual_seed(0)
    m = build_model(cfg, device=device, seed=seed)
    if device == "cpu":
        m.act_dtype = torch.float32
    layer = m.layers[0].attn
    meta, nbl = _meta(T)
    to = lambda mt: AttnMetadata(**{k: (v.to(device) if isinstance(v, torch.Tensor) else v)
                                    for k, v in mt.__dict__.items()})
    x = (torch.randn(T, cfg.hidden_size) * 0.5).to(torch.bfloat16).to(device)
    kv = m._attn_cache(0, nbl, 64, torch.bfloat16, device)
    if decode:
        bt = meta.block_table
        pre = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T - 1], dtype=torch.int32),
                           kv_len=torch.tensor([T - 1], dtype=torch.int32), block_table=bt,
                           slot_mapping=meta.slot_mapping[:T - 1], positions=meta.positions[:T - 1],
                           max_q_len=T - 1, max_kv_len=T - 1, is_decode=False, q_start_host=[0, T - 1],
                           kv_len_host=[T - 1])
        dec = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, 1], dtype=torch.int32),
                           kv_len=torch.tensor([T], dtype=torch.int32), block_table=bt,
                           slot_mapping=meta.slot_mapping[T - 1:], positions=meta.positions[T - 1:], max_q_len=1,
                           max_kv_len=T, is_decode=True, q_start_host=[0, 1], kv_len_host=[T])
        layer(x[:T - 1], to(pre) if device != "cpu" else pre, kv, m.rope)
        last = layer(x[T - 1:], to(dec) if device != "cpu" else dec, kv, m.rope).float()
    if device != "cpu":
        meta = to(meta)
    kv_o = m._attn_cache(0, nbl, 64, torch.bfloat16, device)
    out = layer(x, meta, kv_o, m.rope).float()
    if decode:
        out = torch.cat([out[:T - 1], last])
    c, ix = cfg, layer.indexer
    nh, dn, dr, dv, dc = layer.nh, layer.dn, layer.dr, layer.dv, layer.dc
    K_ = ix.topk
    qa = B.rmsnorm(layer.q_a(x), layer.q_a_norm, c.norm_eps)
    qi, wi = ix.keys_and_queries(x, qa, meta, torch.zeros_like(kv_o[1]), m.rope)
    ki = kv_o[1][meta.block_table[0].long()].reshape(-1, 128)[:T].float()
    I = torch.einsum("th,thj->tj", wi.float(), torch.relu(torch.einsum("thd,jd->thj", qi.float(), ki)))
    q = layer.q_b(qa).view(T, nh, dn + dr).float()
    ckv = layer.kv_a(x).float()
    lat = B.rmsnorm(ckv[:, :dc].to(torch.bfloat16), layer.kv_a_norm, c.norm_eps).float()
    pos_c = meta.positions.cpu()
    rope_c = m.rope.cpu()
    kr = B.apply_rope_ref(ckv[:, dc:].view(T, 1, dr).cpu(), pos_c, rope_c, dr, c.rope_neox).to(x.device)
    qr = B.apply_rope_ref(q[:, :, dn:].cpu(), pos_c, rope_c, dr, c.rope_neox).to(x.device)
    kvb = (lat @ layer.kv_b.dense_weight().float().t()).view(T, nh, dn + dv)
    Kf = torch.cat([kvb[:, :, :dn], kr.float().expand(T, nh, dr)], -1)
    Qf = torch.cat([q[:, :, :dn], qr.float()], -1)
    s = torch.einsum("thd,jhd->htj", Qf, Kf) * layer.scale
    allow = torch.zeros(T, T, dtype=torch.bool, device=x.device)
    for t in range(T):
        sel = torch.arange(t + 1, device=x.device) if t < K_ else torch.topk(I[t, :t + 1], K_).indices
        allow[t, sel] = True
    p = torch.softmax(s.masked_fill(~allow[None], float("-inf")), -1)
    o = torch.einsum("htj,jhv->thv", p, kvb[:, :, dn:]).to(torch.bfloat16)
    ref = layer.o(o.reshape(T, nh * dv)).float()
    if decode:
        out, ref = out[T - 1:], ref[T - 1:]
    return (out - ref).abs().max().item() / ref.abs().max().item()


def test_dsa_layer_matches_masked_dense_reference_cpu():
    """A 90-token prompt with index_topk 16: every query past position 15 attends to its 16
    best-scored tokens.  The oracle expands K / V with kv_b and masks dense attention."""
    err = _layer_vs_oracle("cpu", _cfg(16), 90)
    assert err < 3e-2, err
    err = _layer_vs_oracle("cpu", _cfg(16), 90, decode=True)
    assert err < 3e-2, err


def test_dsa_short_context_is_dense_cpu():
    """Contexts within index_topk take the dense MLA path (the selection is everything)."""
    torch.manual_seed(1)
    cfg = _cfg(128)
    m = build_model(cfg, device="cpu", seed=3)
    m.act_dtype = torch.float32
    dense = build_model(cfg.replace(index_topk=0), device="cpu", seed=3)
    dense.act_dtype = torch.float32
    T = 40
    meta, nbl = _meta(T)
    x = (torch.randn(T, cfg.hidden_size) * 0.5).to(torch.bfloat16)
    a = m.layers[0].attn(x, meta, m._attn_cache(0, nbl, 64, torch.bfloat16, "cpu"), m.rope)
    b = dense.layers[0].attn(x, meta, dense._attn_cache(0, nbl, 64, torch.bfloat16, "cpu"), dense.rope)
    assert torch.allclose(a.float(), b.float(), atol=1e-3)


# ----------------------------------------------------------------------------- GPU kernels
@pytest.mark.gpu
@pytest.mark.parametrize("nh,T,L", [(64, 3, 1000), (8, 5, 70), (32, 2, 4097)])
def test_index_scores_kernel(nh, T, L):
    torch.manual_seed(2)
    nb = (L + 63) // 64 + 2
    kc = torch.randn(nb, 1, 64, 128).to(torch.bfloat16)
    bt = torch.randperm(nb)[:(L + 63) // 64].to(torch.int32)[None]
    pos = torch.tensor(sorted(torch.randint(0, L, (T,)).tolist()), dtype=torch.int32)
    pos[-1] = L - 1
    meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T], dtype=torch.int32), kv_len=torch.tensor([L]),
                        block_table=bt, slot_mapping=torch.zeros(T), positions=pos, max_q_len=T, max_kv_len=L,
                        is_decode=False)
    q = torch.randn(T, nh, 128).to(torch.bfloat16)
    w = torch.randn(T, nh) * 0.1
    seq = torch.zeros(T, dtype=torch.int32)
    ref = D.index_scores(q, w, kc, meta, seq, L)
    mg = AttnMetadata(num_seqs=1, q_start=meta.q_start.cuda(), kv_len=meta.kv_len.cuda(), block_table=bt.cuda(),
                      slot_mapping=meta.slot_mapping.cuda(), positions=pos.cuda(), max_q_len=T, max_kv_len=L,
                      is_decode=False)
    got = D.index_scores(q.cuda(), w.cuda(), kc.cuda(), mg, seq.cuda(), (L + 63) // 64 * 64).cpu()
    for t in range(T):
        p = int(pos[t]) + 1
        err = (got[t, :p] - ref[t, :p]).abs().max().item() / (ref[t, :p].abs().max().item() + 1e-6)
        assert err < 1e-2, (t, err)


@pytest.mark.gpu
@pytest.mark.parametrize("L,K", [(5000, 2048), (300, 64), (40, 64), (2049, 2048)])
def test_topk_kernel(L, K):
    """Top-K positions (as flat cache rows, in position order) of each row's prefix; fewer
    context tokens than K: all of them."""
    torch.manual_seed(3)
    T = 4
    nb = (L + 63) // 64
    bt = torch.randperm(nb + 2)[:nb].to(torch.int32)[None]
    pos = torch.tensor([L - 1, L // 2, min(L - 1, K + 3), 0], dtype=torch.int32)
    scores = torch.randn(T, (L + 63) // 64 * 64)
    meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T], dtype=torch.int32), kv_len=torch.tensor([L]),
                        block_table=bt, slot_mapping=torch.zeros(T), positions=pos, max_q_len=T, max_kv_len=L,
                        is_decode=False)
    seq = torch.zeros(T, dtype=torch.int32)
    r_ref, l_ref = D.topk_rows(scores, meta, seq, K)
    mg = AttnMetadata(num_seqs=1, q_start=meta.q_start.cuda(), kv_len=meta.kv_len.cuda(), block_table=bt.cuda(),
                      slot_mapping=meta.slot_mapping.cuda(), positions=pos.cuda(), max_q_len=T, max_kv_len=L,
                      is_decode=False)
    r, l = D.topk_rows(scores.cuda(), mg, seq.cuda(), K)
    torch.cuda.synchronize()
    assert torch.equal(l.cpu(), l_ref)
    for t in range(T):
        n = int(l_ref[t])
        assert torch.equal(r[t, :n].cpu(), r_ref[t, :n]), t


@pytest.mark.gpu
def test_sparse_mla_gather_attention():
    """Gather + latent decode kernel over per-query selections vs the dense oracle."""
    torch.manual_seed(4)
    T, nh, D_, K = 6, 16, 576, 256
    nb = 40
    kc = (torch.randn(nb, 1, 64, D_) * 0.5).to(torch.bfloat16)
    rows = torch.stack([torch.randperm(nb * 64)[:K] for _ in range(T)]).to(torch.int32)
    lens = torch.tensor([K, 17, 1, 200, 64, 130], dtype=torch.int32)
    q = (torch.randn(T, nh, D_) * 0.3).to(torch.bfloat16)
    ref = D.sparse_mla_dense_ref(q, kc, rows, lens, 1 / math.sqrt(192), 512)
    got = D.sparse_mla(q.cuda(), kc.cuda(), rows.cuda(), lens.cuda(), 1 / math.sqrt(192), 512).float().cpu()
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-2, err


def _gpu_cfg():
    """DeepSeek-V3 head geometry (latent 512 + rope 64, 16 heads) at a small width."""
    return _cfg(64).replace(num_heads=16, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
                            kv_lora_rank=512, q_lora_rank=128, head_dim=192, rotary_dim=64, num_mtp_layers=0)


@pytest.mark.gpu
def test_dsa_layer_matches_masked_dense_reference_gpu():
    """The GPU path (indexer kernels, top-k kernel, gathered latent attention with the
    absorbed projections) against the fp32 oracle on a 150-token prompt, index_topk 64."""
    err = _layer_vs_oracle("cuda", _gpu_cfg(), 150)
    assert err < 3e-2, err
    err = _layer_vs_oracle("cuda", _gpu_cfg(), 150, decode=True)
    assert err < 3e-2, err


@pytest.mark.gpu
def test_dsa_model_generation_eager_and_graph_gpu():
    """A tiny DSA model generates past index_topk (prompts up to 150 tokens, sparse decode)
    eagerly and from captured decode graphs with the same tokens."""
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    m = build_model(_gpu_cfg(), device="cuda", seed=5)
    prompts = [list(range(3, 153)), list(range(200, 260))]
    outs = {}
    for graph in (False, True):
        rc = RunnerConfig(block_size=64, max_seqs=2, max_model_len=512, max_batched_tokens=256, use_cuda_graph=graph)
        llm = LLM(m, device="cuda", runner_config=rc)
        outs[graph] = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=12))]
        llm.shutdown()
    torch.cuda.synchronize()
    N.check_status()
    assert all(len(o) == 12 for o in outs[True])
    assert outs[False] == outs[True]
