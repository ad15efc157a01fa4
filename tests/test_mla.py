"""MLA (DeepSeek-V3 attention) on the GPU: the latent-cache decode kernel (576-wide keys,
V = latent, two CTAs per 512 output columns) and the flash prefill over expanded K/V,
both against the PyTorch restatement."""
import math

import pytest
import torch

from vllm_xtu_moe_b200.ops.attention import AttnMetadata, choose_splits, paged_attention, paged_attention_ref


def _latent_cache(seqs, Hq=128, D=576, bs=64, seed=0):
    g = torch.Generator().manual_seed(seed)
    nb_per = [(kv + bs - 1) // bs for _, kv in seqs]
    nb = sum(nb_per) + 3
    kc = (torch.randn(nb, 1, bs, D, generator=g) * 0.5).to(torch.bfloat16)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(len(seqs), max(nb_per), dtype=torch.int32)
    i = 0
    for b, n in enumerate(nb_per):
        bt[b, :n] = perm[i:i + n].int()
        i += n
    qs = [0]
    for ql, _ in seqs:
        qs.append(qs[-1] + ql)
    d = "cuda"
    meta = AttnMetadata(num_seqs=len(seqs), q_start=torch.tensor(qs, dtype=torch.int32, device=d),
                        kv_len=torch.tensor([kv for _, kv in seqs], dtype=torch.int32, device=d),
                        block_table=bt.to(d), slot_mapping=torch.zeros(qs[-1], dtype=torch.int32, device=d),
                        positions=torch.zeros(qs[-1], dtype=torch.int32, device=d),
                        max_q_len=max(q for q, _ in seqs), max_kv_len=max(kv for _, kv in seqs),
                        is_decode=True, q_start_host=qs, kv_len_host=[kv for _, kv in seqs])
    q = (torch.randn(qs[-1], Hq, D, generator=g) * 0.5).to(torch.bfloat16).to(d)
    return q, kc.to(d), meta


@pytest.mark.gpu
@pytest.mark.parametrize("seqs,splits", [([(1, 1000), (1, 77), (1, 4097)], 1), ([(1, 1000), (1, 77), (1, 4097)], 8),
                                         ([(2, 300), (3, 64)], 1)])
def test_mla_latent_decode_matches_reference(seqs, splits):
    q, kc, meta = _latent_cache(seqs)
    meta.num_splits = splits
    scale = 1.0 / math.sqrt(192)
    o = paged_attention(q, kc, None, meta, scale, v_dim=512)
    ref = paged_attention_ref(q.float(), kc.float(), None, meta, scale, v_dim=512)
    torch.cuda.synchronize()
    err = (o.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
    assert err < 2e-2, err


@pytest.mark.gpu
def test_mla_model_prefill_and_decode_gpu_vs_cpu():
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
    from vllm_xtu_moe_b200.models.model import build_model
    cfg = scaled_down(get_preset("deepseek-v3"), layers=2, hidden=512, experts=16).replace(
        num_heads=16, moe_intermediate=256, shared_intermediate=256, dense_intermediate=1024, q_lora_rank=256,
        kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128, head_dim=192,
        num_mtp_layers=0)
    cpu = build_model(cfg, device="cpu", seed=5)
    gpu = cpu.to("cuda")
    outs = {}
    for name, m in (("cpu", cpu), ("gpu", gpu)):
        llm = LLM(m, device=str(m.device), runner_config=RunnerConfig(block_size=64, max_seqs=2, max_model_len=1024,
                                                                      max_batched_tokens=512, use_cuda_graph=False))
        outs[name] = [o.token_ids for o in llm.generate([list(range(3, 300)), list(range(7, 90))],
                                                        SamplingParams(max_tokens=4))]
        llm.shutdown()
    same = sum(a == b for x, y in zip(outs["cpu"], outs["gpu"]) for a, b in zip(x, y))
    assert same >= 6, outs
