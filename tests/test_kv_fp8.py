"""fp8 (e4m3) KV cache: the cache-write kernel's layout and rounding, the fp8 decode
attention kernel (direct read, f16 MMAs), the dequantise-then-attend path of other step
shapes, and a whole model served with an fp8 cache against the bf16 one."""
import math

import pytest
import torch

from vllm_xtu_moe_b200.ops import _native as N
from vllm_xtu_moe_b200.ops.attention import AttnMetadata, dequant_fp8_cache, paged_attention, paged_attention_ref
from vllm_xtu_moe_b200.ops.basic import rope_and_cache, to_e4m3, write_kv_ref


def _paged_fp8(seqs, Hkv, D, Dv, k_scale, v_scale, bs=64, device="cuda"):
    nblk = sum((kl + bs - 1) // bs for _, kl in seqs) + 2
    kf = torch.randn(nblk, Hkv, bs, D, device=device) * 2
    vf = torch.randn(nblk, Hkv, bs, Dv, device=device) * 2
    kc = to_e4m3(kf, 1 / k_scale)
    vc = to_e4m3(vf.transpose(2, 3).contiguous(), 1 / v_scale)
    perm = torch.randperm(nblk).tolist()
    tables, q_start, kv_len = [], [0], []
    for ql, kl in seqs:
        tables.append([perm.pop() for _ in range((kl + bs - 1) // bs)])
        q_start.append(q_start[-1] + ql)
        kv_len.append(kl)
    bt = torch.zeros(len(seqs), max(len(t) for t in tables), dtype=torch.int32)
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


def test_fp8_cache_reference_write_and_dequant():
    """CPU: the reference write stores k / k_scale and v / v_scale (V transposed per block)
    saturated at 448, and the dequantisation restores them within e4m3 rounding."""
    torch.manual_seed(0)
    T, Hk, D, Dv, bs = 7, 2, 32, 16, 8
    k = torch.randn(T, Hk, D) * 3
    v = torch.randn(T, Hk, Dv) * 3
    v[0, 0, 0] = 1e4                      # saturates
    kc = torch.zeros(4, Hk, bs, D, dtype=torch.float8_e4m3fn)
    vc = torch.zeros(4, Hk, Dv, bs, dtype=torch.float8_e4m3fn)
    slots = torch.tensor([0, 1, 9, 10, 17, 30, -1])
    write_kv_ref(k, v, slots, kc, vc, k_scale=0.5, v_scale=2.0)
    kd, vd = dequant_fp8_cache(kc, vc, 0.5, 2.0)
    for t, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        kk, vv = kd[s // bs, :, s % bs].float(), vd[s // bs, :, s % bs].float()
        assert torch.allclose(kk, k[t], rtol=0.07, atol=0.02)
        want = v[t].clone()
        if t == 0:
            want[0, 0] = 448 * 2.0
        assert torch.allclose(vv, want, rtol=0.07, atol=0.05), t


@pytest.mark.gpu
@pytest.mark.parametrize("Hq,Hkv,D", [(96, 8, 128), (16, 2, 128), (8, 2, 64)])
@pytest.mark.parametrize("mode", ["decode", "decode_split", "spec2", "spec5", "prefill"])
def test_fp8_paged_attention_matches_dequantised_reference(Hq, Hkv, D, mode):
    torch.manual_seed(3)
    seqs = {"decode": [(1, 1000), (1, 63), (1, 4097)], "decode_split": [(1, 1000), (1, 63), (1, 4097)],
            "spec2": [(2, 700), (2, 129), (2, 64)], "spec5": [(5, 700), (5, 130), (5, 64)],
            "prefill": [(300, 300), (77, 590), (1, 1)]}[mode]
    ks, vs = 0.75, 1.5
    kc, vc, meta, T = _paged_fp8(seqs, Hkv, D, D, ks, vs)
    if mode == "decode_split":
        meta.num_splits = 8
    q = torch.randn(T, Hq, D, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(D)
    o = paged_attention(q, kc, vc, meta, scale, k_scale=ks, v_scale=vs)
    torch.cuda.synchronize()
    N.check_status()
    ref = paged_attention_ref(q.float(), kc, vc, meta, scale, k_scale=ks, v_scale=vs)
    err = (o.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
    assert err < 2e-2, (mode, err)


@pytest.mark.gpu
def test_fp8_cache_write_kernel_matches_reference():
    """The rope/KV kernel's e4m3 write (K rows, V transposed per block) equals the reference
    write of the same rotated k and v byte for byte."""
    torch.manual_seed(4)
    T, Hq, Hk, D, bs = 70, 4, 2, 128, 64
    q = torch.randn(T, Hq, D, device="cuda").to(torch.bfloat16)
    k = (torch.randn(T, Hk, D, device="cuda") * 4).to(torch.bfloat16)
    v = (torch.randn(T, Hk, D, device="cuda") * 4).to(torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int32, device="cuda")
    inv = 1.0 / (10000 ** (torch.arange(0, 64, 2, device="cuda").float() / 64))
    ang = torch.arange(4096, device="cuda").float()[:, None] * inv[None]
    cos_sin = torch.cat([ang.cos(), ang.sin()], -1).contiguous()
    slots = torch.randperm(3 * bs, device="cuda")[:T].int()
    kc = torch.zeros(3, Hk, bs, D, dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros(3, Hk, D, bs, dtype=torch.float8_e4m3fn, device="cuda")
    q2, k2 = q.clone(), k.clone()
    rope_and_cache(q2, k2, v, pos, cos_sin, 64, True, slot_mapping=slots, k_cache=kc, v_cache=vc, k_scale=0.5,
                   v_scale=2.0)
    torch.cuda.synchronize()
    kr = torch.zeros_like(kc)
    vr = torch.zeros_like(vc)
    write_kv_ref(k2, v, slots, kr, vr, 0.5, 2.0)
    assert torch.equal(kc.view(torch.uint8), kr.view(torch.uint8))
    assert torch.equal(vc.view(torch.uint8), vr.view(torch.uint8))


def _tiny_glm():
    from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
    return scaled_down(get_preset("glm-4.5-air"), layers=2, hidden=512, experts=8).replace(
        num_heads=8, num_kv_heads=2, head_dim=64, moe_intermediate=256, shared_intermediate=256,
        dense_intermediate=512, dense_fmt="bf16", expert_fmt="bf16", num_mtp_layers=0)


def _logits(model, device, kv_dtype):
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    llm = LLM(model, device=device, runner_config=RunnerConfig(block_size=64 if device != "cpu" else 16, max_seqs=2,
                                                                max_model_len=256, max_batched_tokens=128,
                                                                use_cuda_graph=False, kv_cache_dtype=kv_dtype))
    for p in ([3, 4, 5, 6, 7, 8, 9, 10, 11], list(range(20, 60))):
        llm.add_request(p, SamplingParams(max_tokens=1))
    plan = llm.scheduler.schedule()
    ids, meta = llm.runner.build_meta(plan)
    rows = torch.tensor([meta.q_start_host[i + 1] - 1 for i in range(meta.num_seqs)], device=model.device)
    _, _, _, logits = llm.runner.forward(ids, meta, rows)
    return logits.float().cpu()


def test_model_with_fp8_cache_close_to_bf16_cpu():
    from vllm_xtu_moe_b200.models.model import build_model
    m = build_model(_tiny_glm(), device="cpu", seed=3)
    a, b = _logits(m, "cpu", "bf16"), _logits(m, "cpu", "fp8")
    err = (a - b).abs().max().item() / a.abs().max().item()
    assert err < 5e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("graph", [False, True])
def test_generation_with_fp8_cache_gpu(graph):
    """Greedy generation (prefill through the dequantised blocks, decode on the fp8 kernel,
    eager or CUDA-graph) stays close to the bf16 cache's tokens."""
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    m = build_model(_tiny_glm(), device="cuda", seed=3)
    prompts = [[3, 4, 5, 6, 7, 8, 9], list(range(20, 160))]
    out = {}
    for kv in ("bf16", "fp8"):
        rc = RunnerConfig(block_size=64, max_seqs=2, max_model_len=512, max_batched_tokens=256, use_cuda_graph=graph,
                          kv_cache_dtype=kv)
        llm = LLM(m, device="cuda", runner_config=rc)
        out[kv] = [r.token_ids for r in llm.generate(prompts, SamplingParams(max_tokens=12))]
        torch.cuda.synchronize()
        N.check_status()
        llm.shutdown()
    same = sum(x == y for a, b in zip(out["bf16"], out["fp8"]) for x, y in zip(a, b))
    assert same >= 0.6 * sum(len(a) for a in out["bf16"]), out


# ----------------------------------------------------------------------------- MLA latent
def _tiny_dsv3():
    from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
    return scaled_down(get_preset("deepseek-v3"), layers=2, hidden=512, experts=16).replace(
        num_heads=8, q_lora_rank=256, moe_intermediate=256, shared_intermediate=256, dense_intermediate=1024,
        expert_fmt="bf16", dense_fmt="bf16", num_mtp_layers=0)


def test_mla_fp8_latent_cache_write_and_dequant_cpu():
    """The fp8 latent write rounds latent / scale to e4m3 at each slot; the dequantising
    gather lays the step's blocks out in sequence order (b * maxb + j) times the scale."""
    from vllm_xtu_moe_b200.models.mla import dequant_latent_cache, write_latent_fp8
    torch.manual_seed(0)
    D, bs, nb = 96, 64, 6
    cache = torch.zeros(nb, 1, bs, D, dtype=torch.float8_e4m3fn)
    T = 70
    x = (torch.randn(T, 1, D) * 3).to(torch.bfloat16)
    bt = torch.tensor([[4, 1]], dtype=torch.int32)
    slots = torch.tensor([int(bt[0, t // bs]) * bs + t % bs for t in range(T)], dtype=torch.int32)
    write_latent_fp8(x, slots, cache, 0.5)
    meta = AttnMetadata(num_seqs=1, q_start=torch.tensor([0, T]), kv_len=torch.tensor([T]), block_table=bt,
                        slot_mapping=slots, positions=torch.arange(T), max_q_len=T, max_kv_len=T, is_decode=False,
                        q_start_host=[0, T], kv_len_host=[T])
    out, m2 = dequant_latent_cache(cache, meta, 0.5)
    assert torch.equal(m2.block_table, torch.tensor([[0, 1]], dtype=torch.int32))
    flat = out.view(-1, D)[:T].float()
    want = (to_e4m3(x[:, 0].float(), 2.0).float() * 0.5).to(torch.bfloat16).float()
    assert torch.equal(flat, want)


def test_mla_model_with_fp8_latent_cache_close_to_bf16_cpu():
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    m = build_model(_tiny_dsv3(), device="cpu", seed=2)
    prompts = [list(range(3, 90)), list(range(7, 30))]
    out = {}
    for kv in ("bf16", "fp8"):
        rc = RunnerConfig(block_size=64, max_seqs=2, max_model_len=256, max_batched_tokens=128,
                          use_cuda_graph=False, kv_cache_dtype=kv)
        out[kv] = [r.token_ids for r in LLM(m, device="cpu", runner_config=rc).generate(
            prompts, SamplingParams(max_tokens=6))]
    same = sum(x == y for a, b in zip(out["bf16"], out["fp8"]) for x, y in zip(a, b))
    assert same >= 0.6 * 12, out


@pytest.mark.gpu
def test_mla_fp8_latent_kernels_match_reference():
    """xtu_mla_latent_write_fp8 / xtu_mla_latent_dequant_gather against the CPU path, bit
    for bit (e4m3 rounding with saturation, then e4m3 x scale rounded to bf16)."""
    from vllm_xtu_moe_b200.models.mla import dequant_latent_cache, write_latent_fp8
    torch.manual_seed(1)
    D, bs, nb = 576, 64, 12
    T = [150, 40]
    x = (torch.randn(sum(T), 1, D) * 40).to(torch.bfloat16)   # some values past 448 x scale saturate
    bt = torch.tensor([[7, 2, 9], [5, 0, 0]], dtype=torch.int32)
    slots, q_start, pos = [], [0], []
    for b, n in enumerate(T):
        slots += [int(bt[b, t // bs]) * bs + t % bs for t in range(n)]
        q_start.append(q_start[-1] + n)
        pos += list(range(n))
    slots = torch.tensor(slots, dtype=torch.int32)
    meta = AttnMetadata(num_seqs=2, q_start=torch.tensor(q_start, dtype=torch.int32),
                        kv_len=torch.tensor(T, dtype=torch.int32), block_table=bt, slot_mapping=slots,
                        positions=torch.tensor(pos, dtype=torch.int32), max_q_len=150, max_kv_len=150,
                        is_decode=False, q_start_host=q_start, kv_len_host=T)
    ref_cache = torch.zeros(nb, 1, bs, D, dtype=torch.float8_e4m3fn)
    write_latent_fp8(x, slots, ref_cache, 0.25)
    ref, _ = dequant_latent_cache(ref_cache, meta, 0.25)
    gmeta = AttnMetadata(**{k: (v.cuda() if isinstance(v, torch.Tensor) else v) for k, v in meta.__dict__.items()})
    cache = torch.zeros(nb, 1, bs, D, dtype=torch.float8_e4m3fn, device="cuda")
    write_latent_fp8(x.cuda(), gmeta.slot_mapping, cache, 0.25)
    got, _ = dequant_latent_cache(cache, gmeta, 0.25)
    torch.cuda.synchronize()
    N.check_status()
    assert torch.equal(cache.cpu().view(torch.uint8), ref_cache.view(torch.uint8))
    for b, n in enumerate(T):   # blocks past a sequence's length are not written
        nbk = (n + bs - 1) // bs
        assert torch.equal(got.view(2, 3, bs, D)[b, :nbk].cpu(), ref.view(2, 3, bs, D)[b, :nbk])


@pytest.mark.gpu
def test_mla_generation_with_fp8_latent_cache_gpu():
    """DeepSeek-V3-shaped MLA with an fp8 latent cache: CUDA-graph decode equals eager decode
    token for token, and both stay close to the bf16 cache's tokens."""
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.model import build_model
    m = build_model(_tiny_dsv3(), device="cuda", seed=4)
    prompts = [list(range(1, 150)), list(range(9, 70))]
    out = {}
    for kv, graph in (("bf16", False), ("fp8", False), ("fp8", True)):
        rc = RunnerConfig(block_size=64, max_seqs=2, max_model_len=512, max_batched_tokens=256,
                          use_cuda_graph=graph, kv_cache_dtype=kv)
        llm = LLM(m, device="cuda", runner_config=rc)
        out[(kv, graph)] = [r.token_ids for r in llm.generate(prompts, SamplingParams(max_tokens=10))]
        torch.cuda.synchronize()
        N.check_status()
        llm.shutdown()
    assert out[("fp8", False)] == out[("fp8", True)]
    same = sum(x == y for a, b in zip(out[("bf16", False)], out[("fp8", False)]) for x, y in zip(a, b))
    assert same >= 0.6 * 20, out
