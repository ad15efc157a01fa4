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
