"""Checkpoint IO: safetensors round trip, and HF-named checkpoints of each family loaded
back into an identical model (export -> load -> same logits)."""
import json

import pytest
import torch

from vllm_xtu_moe_b200.engine import LLM, SamplingParams
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.models.config import get_preset, scaled_down
from vllm_xtu_moe_b200.models.loader import CheckpointSource, export_hf, load_model
from vllm_xtu_moe_b200.models.model import build_model
from vllm_xtu_moe_b200.utils.safetensors import SafetensorsFile, save_file


def test_safetensors_round_trip(tmp_path):
    ts = {"a": torch.randn(3, 5), "b": torch.arange(7, dtype=torch.int32),
          "c": torch.randn(4, 8).to(torch.float8_e4m3fn), "d": torch.randn(2, 2).to(torch.bfloat16),
          "e": torch.randint(0, 255, (6,), dtype=torch.uint8)}
    save_file(ts, tmp_path / "x.safetensors", {"format": "pt"})
    f = SafetensorsFile(tmp_path / "x.safetensors")
    for k, v in ts.items():
        got = f.get(k)
        assert got.dtype == v.dtype and got.shape == v.shape
        assert torch.equal(got.view(torch.uint8), v.view(torch.uint8))
    assert f.meta == {"format": "pt"}
    f.close()


def _cfg(name):
    cfg = get_preset(name)
    if name == "tiny-mixtral":
        return cfg
    if name == "kimi-linear-48b-a3b":
        return scaled_down(cfg, layers=4, hidden=256, experts=8).replace(
            num_heads=4, linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=32,
            linear_value_head_dim=32, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16, v_head_dim=32,
            head_dim=48, moe_intermediate=128, shared_intermediate=128, dense_intermediate=256)
    if name == "mimo-v2-flash":
        return scaled_down(cfg, layers=4, hidden=256, experts=8).replace(
            num_heads=4, num_kv_heads=1, swa_num_kv_heads=2, head_dim=64, v_head_dim=32, rotary_dim=32,
            sliding_window=8, moe_intermediate=256, dense_intermediate=512, expert_fmt="bf16", dense_fmt="bf16")
    return scaled_down(cfg, layers=4 if "qwen" in name else 2, hidden=256, experts=8).replace(
        num_heads=4, num_kv_heads=2, head_dim=64 if not cfg.is_mla else cfg.head_dim, moe_intermediate=256,
        shared_intermediate=256, dense_intermediate=512, linear_num_key_heads=2, linear_num_value_heads=4,
        linear_key_head_dim=32, linear_value_head_dim=32, q_lora_rank=128 if cfg.is_mla else 0,
        kv_lora_rank=128 if cfg.is_mla else 0, qk_nope_head_dim=32 if cfg.is_mla else 0,
        v_head_dim=32 if cfg.is_mla else 0, rotary_dim=32 if cfg.rotary_dim else None)


def _logits(model):
    llm = LLM(model, device="cpu", runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=256,
                                                              max_batched_tokens=128, use_cuda_graph=False))
    for p in ([3, 4, 5, 6, 7, 8, 9, 10, 11], list(range(20, 60))):
        llm.add_request(p, SamplingParams(max_tokens=1))
    plan = llm.scheduler.schedule()
    ids, meta = llm.runner.build_meta(plan)
    rows = torch.tensor([meta.q_start_host[i + 1] - 1 for i in range(meta.num_seqs)])
    _, _, _, logits = llm.runner.forward(ids, meta, rows)
    return logits.float()


@pytest.mark.parametrize("name", ["tiny-mixtral", "glm-4.5-air", "deepseek-v3", "qwen3-next-80b-a3b",
                                  "mimo-v2-flash", "kimi-linear-48b-a3b"])
def test_hf_checkpoint_round_trip(tmp_path, name):
    cfg = _cfg(name)
    m = build_model(cfg, device="cpu", seed=11)
    export_hf(m, cfg, tmp_path / "model.safetensors")
    m2, src = load_model(tmp_path, device="cpu", cfg=cfg)
    # every tensor of the checkpoint was consumed by the builder
    assert src.used == set(src.ckpt.keys()), set(src.ckpt.keys()) - src.used
    a, b = _logits(m), _logits(m2)
    assert torch.equal(a, b)
    src.close()


def test_loader_streams_experts_into_sink(tmp_path):
    """The expert sink receives checkpoint-layout experts per layer (e.g. for the CPU engine)."""
    cfg = _cfg("glm-4.5-air")
    m = build_model(cfg, device="cpu", seed=3)
    export_hf(m, cfg, tmp_path / "model.safetensors")
    seen = []

    def sink(layer, raw):
        seen.append((layer, raw["fmt"], tuple(raw["w13"].shape), tuple(raw["s13"].shape)))
        from vllm_xtu_moe_b200.ops.moe import prepare_experts
        return prepare_experts(raw["fmt"], raw["w13"], raw["w2"], raw.get("s13"), raw.get("s2"))

    m2, src = load_model(tmp_path, device="cpu", cfg=cfg, expert_sink=sink)
    I, H, E = cfg.moe_intermediate, cfg.hidden_size, cfg.num_experts
    moe_layers = [i for i in range(cfg.num_layers) if cfg.is_moe_layer(i)] + [cfg.num_layers - 1] * cfg.num_mtp_layers
    assert [s[0] for s in seen] == moe_layers
    assert all(s[1] == "fp8" and s[2] == (E, 2 * I, H) and s[3] == (E, 2 * I // 128, H // 128) for s in seen)
    src.close()


def _gptq_pack(w: torch.Tensor, group: int = 32):
    """Test-side GPTQ packer (AutoGPTQ "gptq" format) of a weight [out, in]: returns the
    checkpoint tensors and the exact dequantized weight they stand for."""
    N, K = w.shape
    G = K // group
    wt = w.t().float()                                             # [in, out]
    wg = wt.view(G, group, N)
    scale = (wg.abs().amax(1) / 7.0).clamp(min=1e-4).half()       # [G, out]
    zero = torch.full((G, N), 8, dtype=torch.int64)
    q = (torch.round(wg / scale.float()[:, None, :]) + 8).clamp(0, 15).to(torch.int64).view(K, N)
    qw = torch.zeros(K // 8, N, dtype=torch.int64)
    for i in range(8):
        qw |= q[i::8] << (4 * i)
    qz = torch.zeros(G, N // 8, dtype=torch.int64)
    for i in range(8):
        qz |= (zero[:, i::8] - 1) << (4 * i)
    deq = ((q.view(G, group, N) - zero[:, None, :]).float() * scale.float()[:, None, :]).view(K, N).t()
    def to32(t):       # the uint32 words as the int32 tensors checkpoints store
        return torch.tensor(((t + 2 ** 31) % 2 ** 32 - 2 ** 31).tolist(), dtype=torch.int32)
    return {"qweight": to32(qw), "qzeros": to32(qz), "scales": scale}, deq


def test_gptq_dequant_matches_packing():
    from vllm_xtu_moe_b200.ops.quant import dequant_gptq
    torch.manual_seed(0)
    w = torch.randn(64, 128) * 0.05
    t, deq = _gptq_pack(w)
    got = dequant_gptq(t["qweight"], t["scales"], t["qzeros"])
    assert torch.equal(got, deq)
    assert (got - w).abs().max().item() < 0.02


def test_gptq_checkpoint_loads(tmp_path):
    """Experts and attention projections stored as GPTQ INT4: the loaded model equals one
    loaded from the same weights dequantized to bf16."""
    from vllm_xtu_moe_b200.utils.safetensors import SafetensorsFile, save_file
    cfg = _cfg("tiny-mixtral")
    m = build_model(cfg, device="cpu", seed=5)
    export_hf(m, cfg, tmp_path / "model.safetensors")
    f = SafetensorsFile(tmp_path / "model.safetensors")
    tensors = {k: f.get(k).clone() for k in f.keys()}
    f.close()
    gptq, plain = dict(tensors), dict(tensors)
    for k in list(tensors):
        if k.endswith(".weight") and (".experts." in k or ".self_attn.q_proj" in k):
            pre = k[:-len(".weight")]
            packed, deq = _gptq_pack(tensors[k].float())
            del gptq[k]
            gptq.update({f"{pre}.{s}": v for s, v in packed.items()})
            plain[k] = deq.to(torch.bfloat16)
    (tmp_path / "g").mkdir()
    (tmp_path / "p").mkdir()
    save_file(gptq, tmp_path / "g" / "model.safetensors", {"format": "pt"})
    save_file(plain, tmp_path / "p" / "model.safetensors", {"format": "pt"})
    mg, sg = load_model(tmp_path / "g", device="cpu", cfg=cfg)
    mp_, sp_ = load_model(tmp_path / "p", device="cpu", cfg=cfg)
    assert sg.used == set(sg.ckpt.keys())
    assert torch.equal(_logits(mg), _logits(mp_))
    sg.close()
    sp_.close()


def test_gptq_v2_zero_points_and_unsupported_formats(tmp_path):
    """gptq_v2 stores zero points as they are (v1: minus one); 3-bit weights and unknown
    checkpoint formats are refused instead of being dequantized wrongly."""
    import json
    from vllm_xtu_moe_b200.models.loader import CheckpointSource
    from vllm_xtu_moe_b200.ops.quant import dequant_gptq
    torch.manual_seed(1)
    t, deq = _gptq_pack(torch.randn(64, 128) * 0.05)
    qz = t["qzeros"].to(torch.int64) & 0xFFFFFFFF
    v2 = torch.zeros_like(qz)
    for i in range(8):                 # every packed zero point + 1 (no carries: v1 stores 7)
        v2 |= (((qz >> (4 * i)) & 0xF) + 1) << (4 * i)
    v2 = torch.tensor(((v2 + 2 ** 31) % 2 ** 32 - 2 ** 31).tolist(), dtype=torch.int32)
    assert torch.equal(dequant_gptq(t["qweight"], t["scales"], v2, zero_offset=0), deq)
    with pytest.raises(ValueError, match="3-bit"):
        dequant_gptq(t["qweight"], t["scales"], t["qzeros"], bits=3)
    for qc, ok in [({"quant_method": "gptq", "bits": 4, "checkpoint_format": "gptq_v2"}, (4, 0)),
                   ({"quant_method": "gptq", "bits": 8}, (8, 1)),
                   ({"quant_method": "gptq", "bits": 3}, None),
                   ({"quant_method": "gptq", "bits": 4, "checkpoint_format": "marlin"}, None)]:
        d = tmp_path / f"c{len(list(tmp_path.iterdir()))}"
        d.mkdir()
        (d / "config.json").write_text(json.dumps({"quantization_config": qc}))
        if ok is None:
            with pytest.raises(ValueError):
                CheckpointSource._gptq_format(d)
        else:
            assert CheckpointSource._gptq_format(d) == ok


def test_gptq_int4_rows_match_dequant():
    """4-bit, 128-grouped GPTQ weights repacked as INT4 rows (kept at 4 bits) stand for the
    same weight as the dequantized checkpoint; other group sizes are left to dequantization."""
    from vllm_xtu_moe_b200.ops.quant import dequant_gptq, dequant_int4_rows, gptq_to_int4_rows
    torch.manual_seed(2)
    t, deq = _gptq_pack(torch.randn(96, 256) * 0.05, group=128)
    packed, sz = gptq_to_int4_rows(t["qweight"], t["scales"], t["qzeros"])
    assert packed.shape == (96, 128) and packed.dtype == torch.uint8 and sz.shape == (96, 2, 2)
    assert torch.equal(dequant_int4_rows(packed, sz), dequant_gptq(t["qweight"], t["scales"], t["qzeros"]))
    t32, _ = _gptq_pack(torch.randn(96, 256) * 0.05, group=32)
    assert gptq_to_int4_rows(t32["qweight"], t32["scales"], t32["qzeros"]) is None


def test_gptq_int4_experts_stay_4bit_on_the_cpu_tier(tmp_path):
    """A GPTQ expert checkpoint (4-bit, group 128) served with the experts on the CPU tier:
    the engine holds INT4 rows (a quarter of bf16's bytes) and the logits match the model
    loaded from the dequantized weights."""
    from vllm_xtu_moe_b200.tiering.executor import TieredExperts
    from vllm_xtu_moe_b200.utils.safetensors import SafetensorsFile, save_file
    cfg = _cfg("tiny-mixtral")
    m = build_model(cfg, device="cpu", seed=6)
    export_hf(m, cfg, tmp_path / "model.safetensors")
    f = SafetensorsFile(tmp_path / "model.safetensors")
    tensors = {k: f.get(k).clone() for k in f.keys()}
    f.close()
    gptq, plain = dict(tensors), dict(tensors)
    for k in list(tensors):
        if k.endswith(".weight") and ".experts." in k:
            pre = k[:-len(".weight")]
            packed, deq = _gptq_pack(tensors[k].float(), group=128)
            del gptq[k]
            gptq.update({f"{pre}.{s}": v for s, v in packed.items()})
            plain[k] = deq.to(torch.bfloat16)
    for d, ts in (("g", gptq), ("p", plain)):
        (tmp_path / d).mkdir()
        save_file(ts, tmp_path / d / "model.safetensors", {"format": "pt"})
    tier = TieredExperts(cfg, device="cpu", resident_layers=set(), threads=2)
    mg, sg = load_model(tmp_path / "g", device="cpu", cfg=cfg, expert_sink=tier.expert_sink)
    tier.attach(mg)
    mp_, sp_ = load_model(tmp_path / "p", device="cpu", cfg=cfg)
    engines = [ex.engine for ex in tier.executors]
    assert engines and all(e.fmt == "int4" for e in engines)
    E, I, H = cfg.num_experts, cfg.moe_intermediate, cfg.hidden_size
    assert engines[0].info()["bytes"] <= E * 3 * I * H // 2 * 1.2          # ~4 bits per weight
    a, b = _logits(mp_), _logits(mg)
    assert (a - b).abs().max().item() <= 3e-2 * a.abs().max().item(), (a - b).abs().max().item()
    tier.shutdown()
    sg.close()
    sp_.close()
