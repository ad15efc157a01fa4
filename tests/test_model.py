"""Whole-model checks: the GPU kernels path vs the CPU PyTorch path on identical weights."""
import pytest
import torch

from vllm_xtu_moe_b200.engine import LLM, SamplingParams
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
from vllm_xtu_moe_b200.models.model import build_model
from vllm_xtu_moe_b200.ops import _native as N


def _glm_mini():
    return scaled_down(get_preset("glm-4.5-air"), layers=2, hidden=1024, experts=16).replace(
        num_heads=16, num_kv_heads=2, moe_intermediate=256, shared_intermediate=256, dense_intermediate=1024,
        dense_fmt="fp8", expert_fmt="fp8")


def _rc(graph):
    return RunnerConfig(block_size=64, max_seqs=4, max_model_len=1024, max_batched_tokens=256, use_cuda_graph=graph)


def test_generate_cpu_all_families():
    for name in ["tiny-mixtral", "glm-4.5-air", "deepseek-v3", "qwen3-next-80b-a3b"]:
        cfg = get_preset(name)
        if name != "tiny-mixtral":
            cfg = scaled_down(cfg, layers=4 if "qwen" in name else 2, hidden=256, experts=16).replace(
                num_heads=4, num_kv_heads=2, head_dim=64 if not cfg.is_mla else cfg.head_dim, moe_intermediate=256,
                shared_intermediate=256, dense_intermediate=512, linear_num_key_heads=2, linear_num_value_heads=4,
                linear_key_head_dim=32, linear_value_head_dim=32, q_lora_rank=64 if cfg.is_mla else 0,
                kv_lora_rank=64 if cfg.is_mla else 0, qk_nope_head_dim=32 if cfg.is_mla else 0,
                v_head_dim=32 if cfg.is_mla else 0, rotary_dim=32 if cfg.rotary_dim else None)
        llm = LLM(cfg, device="cpu", runner_config=RunnerConfig(block_size=16, max_seqs=4, max_model_len=256,
                                                                max_batched_tokens=64, use_cuda_graph=False))
        outs = llm.generate([list(range(1, 40)), list(range(5, 90))], SamplingParams(max_tokens=6))
        assert all(len(o.token_ids) == 6 for o in outs)


def _prefill_logits(model, prompts):
    llm = LLM(model, runner_config=_rc(False))
    for p in prompts:
        llm.add_request(p, SamplingParams(max_tokens=1))
    plan = llm.scheduler.schedule()
    ids, meta = llm.runner.build_meta(plan)
    rows = torch.tensor([meta.q_start_host[i + 1] - 1 for i in range(meta.num_seqs)], device=model.device)
    _, _, _, logits = llm.runner.forward(ids, meta, rows)
    return logits.float().cpu()


@pytest.mark.gpu
@pytest.mark.parametrize("which", ["tiny-mixtral", "glm-mini"])
def test_gpu_matches_cpu_prefill(which):
    cfg = get_preset("tiny-mixtral") if which == "tiny-mixtral" else _glm_mini()
    cpu = build_model(cfg, device="cpu", seed=3)
    gpu = cpu.to("cuda")
    prompts = [list(range(3, 200)), list(range(50, 120))]
    lc = _prefill_logits(cpu, prompts)
    lg = _prefill_logits(gpu, prompts)
    torch.cuda.synchronize()
    N.check_status()
    err = (lc - lg).abs().max().item() / lc.abs().max().item()
    assert err < 5e-2, err


@pytest.mark.gpu
def test_gpu_decode_graph_matches_eager():
    cfg = _glm_mini()
    m = build_model(cfg, device="cuda", seed=4)
    prompts = [list(range(1, 150)), list(range(9, 70)), list(range(100, 400))]
    outs = {}
    for graph in (False, True):
        llm = LLM(m, runner_config=_rc(graph))
        outs[graph] = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10))]
        llm.shutdown()
    torch.cuda.synchronize()
    N.check_status()
    assert outs[False] == outs[True]
