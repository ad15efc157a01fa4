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


def _mimo_mini(head_dim=192, v_dim=128, window=32):
    """MiMo-V2 structure at test size: full, swa, swa, swa layers (the full layer with 2 KV
    heads, the sliding-window layers with 4 and learned sinks), 192-wide q/k, 128-wide v."""
    return scaled_down(get_preset("mimo-v2-flash"), layers=4, hidden=512, experts=16).replace(
        num_heads=8, num_kv_heads=2, swa_num_kv_heads=4, head_dim=head_dim, v_head_dim=v_dim, rotary_dim=64,
        sliding_window=window, moe_intermediate=256, dense_intermediate=1024, expert_fmt="bf16", dense_fmt="bf16",
        num_mtp_layers=0)


def _kimi_mini():
    """Kimi-Linear structure at test size: 3 KDA layers (2 heads x 128, so the GPU kernels run)
    and one MLA layer without rotary embedding."""
    return scaled_down(get_preset("kimi-linear-48b-a3b"), layers=4, hidden=512, experts=16).replace(
        num_heads=8, linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=128,
        linear_value_head_dim=128, kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64, v_head_dim=128,
        head_dim=192, moe_intermediate=256, shared_intermediate=256, dense_intermediate=1024)


def _qwen_mini():
    """Qwen3-Next structure at test size: 3 gated-DeltaNet layers (128-wide heads, so the GPU
    kernels run) and one gated GQA layer."""
    return scaled_down(get_preset("qwen3-next-80b-a3b"), layers=4, hidden=512, experts=16).replace(
        num_heads=4, num_kv_heads=2, head_dim=128, rotary_dim=32, linear_num_key_heads=2, linear_num_value_heads=4,
        linear_key_head_dim=128, linear_value_head_dim=128, moe_intermediate=256, shared_intermediate=256,
        expert_fmt="bf16")


def _dsv3_mini():
    """DeepSeek-V3 structure at test size (MLA with kv_lora 512 + rope 64, so the latent
    decode kernel runs)."""
    return scaled_down(get_preset("deepseek-v3"), layers=2, hidden=512, experts=16).replace(
        num_heads=8, q_lora_rank=256, moe_intermediate=256, shared_intermediate=256, dense_intermediate=1024,
        expert_fmt="bf16", dense_fmt="bf16", num_mtp_layers=0)


def _rc(graph, max_model_len=1024):
    return RunnerConfig(block_size=64, max_seqs=4, max_model_len=max_model_len, max_batched_tokens=256,
                        use_cuda_graph=graph)


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


def test_mimo_structure_on_cpu():
    """MiMo-V2 layers: per-layer KV-head counts and value width in the caches, the window and
    sinks on the sliding-window layers only, and generation through the engine."""
    cfg = _mimo_mini(head_dim=64, v_dim=32, window=16)
    m = build_model(cfg, device="cpu", seed=1)
    kinds = [cfg.layer_type(i) for i in range(cfg.num_layers)]
    assert kinds == ["full", "swa", "swa", "swa"]
    caches = m.allocate_caches(8, 16, 2)
    assert caches[0][0].shape == (8, 2, 16, 64) and caches[0][1].shape == (8, 2, 16, 32)
    assert caches[1][0].shape == (8, 4, 16, 64) and caches[1][1].shape == (8, 4, 16, 32)
    a0, a1 = m.layers[0].attn, m.layers[1].attn
    assert a0.window == 0 and a0.sinks is None and a1.window == 16 and a1.sinks.shape == (8,)
    assert m.kv_bytes_per_token() == (2 * 96 + 3 * 4 * 96) * 2
    llm = LLM(m, device="cpu", runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=256,
                                                          max_batched_tokens=64, use_cuda_graph=False))
    outs = llm.generate([list(range(1, 70)), list(range(5, 40))], SamplingParams(max_tokens=5))
    assert all(len(o.token_ids) == 5 for o in outs)


def test_kimi_linear_on_cpu_and_config_mapping():
    from vllm_xtu_moe_b200.models.config import from_hf_config
    from vllm_xtu_moe_b200.models.deltanet import KimiDeltaAttention
    cfg = _kimi_mini().replace(hidden_size=256, linear_key_head_dim=32, linear_value_head_dim=32, kv_lora_rank=64,
                               qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32, head_dim=48)
    m = build_model(cfg, device="cpu", seed=2)
    assert [type(l.attn).__name__ for l in m.layers] == ["KimiDeltaAttention"] * 3 + ["MLAAttention"]
    assert isinstance(m.layers[0].attn, KimiDeltaAttention)
    llm = LLM(m, device="cpu", runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=256,
                                                          max_batched_tokens=64, use_cuda_graph=False))
    outs = llm.generate([list(range(1, 70)), list(range(5, 40))], SamplingParams(max_tokens=5))
    assert all(len(o.token_ids) == 5 for o in outs)
    hf = {"architectures": ["KimiLinearForCausalLM"], "hidden_size": 2304, "num_attention_heads": 32,
          "num_hidden_layers": 8, "vocab_size": 1000, "kv_lora_rank": 512, "q_lora_rank": None,
          "qk_nope_head_dim": 128, "qk_rope_head_dim": 64, "v_head_dim": 128, "mla_use_nope": True,
          "linear_attn_config": {"full_attn_layers": [4, 8], "kda_layers": [1, 2, 3, 5, 6, 7], "num_heads": 32,
                                 "head_dim": 128, "short_conv_kernel_size": 4},
          "num_experts": 256, "num_experts_per_token": 8, "num_shared_experts": 1, "moe_intermediate_size": 1024,
          "intermediate_size": 9216, "first_k_dense_replace": 1, "routed_scaling_factor": 2.446}
    c = from_hf_config(hf)
    assert c.arch == "kimi_linear" and c.linear_kind == "kda" and not c.mla_rope and c.is_mla
    assert c.layer_types == ["linear"] * 3 + ["full"] + ["linear"] * 3 + ["full"]
    assert (c.linear_num_key_heads, c.linear_key_head_dim, c.q_lora_rank) == (32, 128, 0)


def test_mimo_hf_config_mapping():
    from vllm_xtu_moe_b200.models.config import from_hf_config
    hf = {"architectures": ["MiMoV2FlashForCausalLM"], "hidden_size": 4096, "num_attention_heads": 64,
          "num_key_value_heads": 4, "head_dim": 192, "v_head_dim": 128, "num_hidden_layers": 4,
          "vocab_size": 1000, "hybrid_layer_pattern": [0, 1, 1, 1], "sliding_window": 128,
          "swa_num_key_value_heads": 8, "add_swa_attention_sink_bias": True, "partial_rotary_factor": 0.334,
          "n_routed_experts": 256, "num_experts_per_tok": 8, "moe_intermediate_size": 2048,
          "intermediate_size": 16384, "first_k_dense_replace": 1}
    c = from_hf_config(hf)
    assert c.arch == "mimo_v2" and c.layer_types == ["full", "swa", "swa", "swa"]
    assert (c.kv_heads(0), c.kv_heads(1), c.window(0), c.window(2)) == (4, 8, 0, 128)
    assert c.has_sinks(1) and not c.has_sinks(0) and c.gqa_v_dim == 128 and c.rot_dim == 64


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
@pytest.mark.parametrize("which", ["tiny-mixtral", "glm-mini", "mimo-mini", "kimi-mini", "qwen-mini"])
def test_gpu_matches_cpu_prefill(which):
    cfg = {"tiny-mixtral": lambda: get_preset("tiny-mixtral"), "glm-mini": _glm_mini, "mimo-mini": _mimo_mini,
           "kimi-mini": _kimi_mini, "qwen-mini": _qwen_mini}[which]()
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
@pytest.mark.parametrize("which", ["glm-mini", "mimo-mini", "kimi-mini", "qwen-mini", "dsv3-mini"])
def test_gpu_decode_graph_matches_eager(which):
    """Decode replayed from CUDA graphs equals eager decode token for token; for the
    linear-attention families this also checks that capturing a graph (whose warm-up passes
    execute) leaves the sequences' recurrent state alone, and that padding rows of a graph
    batch own no state."""
    cfg = {"glm-mini": _glm_mini, "mimo-mini": _mimo_mini, "kimi-mini": _kimi_mini, "qwen-mini": _qwen_mini,
           "dsv3-mini": _dsv3_mini}[which]()
    m = build_model(cfg, device="cuda", seed=4)
    prompts = [list(range(1, 150)), list(range(9, 70)), list(range(100, 400))]
    outs = {}
    for graph in (False, True):
        # graphs size their split-KV factor for max_model_len, eager steps for the current
        # context; with max_model_len 512 both use one split, so the runs are bit-identical
        # (with different split counts a rounding difference can flip a near-tied greedy pick)
        llm = LLM(m, runner_config=_rc(graph, 512))
        outs[graph] = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=10))]
        llm.shutdown()
    torch.cuda.synchronize()
    N.check_status()
    assert outs[False] == outs[True]


@pytest.mark.gpu
def test_embedding_offloaded_to_pinned_host_memory():
    """The token-embedding table kept in pinned host memory (read by the lookup kernel over
    the host link) gives the same logits as the device-resident table, and frees its HBM."""
    cfg = _glm_mini()
    m = build_model(cfg, device="cuda", seed=6)
    prompts = [list(range(3, 90)), list(range(40, 75))]
    want = _prefill_logits(m, prompts)
    freed = m.offload_embedding()
    assert freed == cfg.vocab_size * cfg.hidden_size * 2
    assert not m.embed_tokens.is_cuda and m.embed_tokens.is_pinned()
    got = _prefill_logits(m, prompts)
    torch.cuda.synchronize()
    N.check_status()
    assert torch.equal(got, want)


def _mimo_generate(device, bounded, graphs=False, bs=16, window=16, max_tokens=8):
    cfg = _mimo_mini(head_dim=64 if device == "cpu" else 192, v_dim=32 if device == "cpu" else 128, window=window)
    m = build_model(cfg, device=device, seed=3)
    rc = RunnerConfig(block_size=bs, max_seqs=2, max_model_len=512, max_batched_tokens=64, use_cuda_graph=graphs,
                      graph_batch_sizes=(1, 2), swa_bounded=bounded)
    llm = LLM(m, device=device, runner_config=rc)
    prompts = [list(range(1, 71)), list(range(9, 44))]
    held = []
    orig = llm.blocks.ensure

    def ensure(req, upto):          # record how many window-pool blocks a request holds
        ok = orig(req, upto)
        held.append(len(req.swa_blocks))
        return ok

    llm.blocks.ensure = ensure
    toks = [o.token_ids for o in llm.generate(prompts, SamplingParams(max_tokens=max_tokens))]
    return toks, held, rc.swa_blocks, llm.blocks


def test_bounded_sliding_window_pool_matches_full_context_cpu():
    """Sliding-window layers keeping only their window in a pool of their own give the same
    tokens as keeping the whole context, across chunked prefill and decode, while a request
    never holds more than window / block_size + 2 + its chunk's blocks of that pool."""
    want, _, nb0, _ = _mimo_generate("cpu", bounded=False)
    got, held, nb, bm = _mimo_generate("cpu", bounded=True)
    assert nb0 == 0 and nb > 0
    assert got == want
    assert max(held) <= 16 // 16 + 2 + 64 // 16
    assert len(bm.swa_free) == nb           # everything returned at the end


@pytest.mark.gpu
def test_bounded_sliding_window_pool_matches_full_context_gpu():
    want, _, _, _ = _mimo_generate("cuda", bounded=False, graphs=True, bs=64, window=32, max_tokens=10)
    got, _, nb, _ = _mimo_generate("cuda", bounded=True, graphs=True, bs=64, window=32, max_tokens=10)
    torch.cuda.synchronize()
    N.check_status()
    assert nb > 0 and got == want
