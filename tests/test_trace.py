"""Observability hooks: routing dump -> XTUP table, per-layer timing, config registry."""
import json

import torch

from vllm_xtu_moe_b200.config import EngineConfig
from vllm_xtu_moe_b200.engine import LLM, SamplingParams
from vllm_xtu_moe_b200.engine.runner import RunnerConfig
from vllm_xtu_moe_b200.models.config import get_preset
from vllm_xtu_moe_b200.tiering.policy import load_pin_table
from vllm_xtu_moe_b200.utils.trace import load_dump, to_xtup


def test_routing_dump_and_pin_table(tmp_path):
    dump = tmp_path / "route.json"
    ec = EngineConfig(routing_dump=str(dump))
    cfg = get_preset("tiny-mixtral")
    llm = LLM(cfg, device="cpu", engine_config=ec,
              runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=256, max_batched_tokens=64,
                                         use_cuda_graph=False))
    outs = llm.generate([list(range(1, 30)), list(range(40, 51))], SamplingParams(max_tokens=5))
    llm.shutdown()
    E, counts = load_dump(str(dump))
    assert E == cfg.num_experts and set(counts) == set(range(cfg.num_layers))
    # every forwarded token routed top-k times per layer: prompt tokens + decode steps
    tokens = 29 + 11 + sum(len(o.token_ids) - 1 for o in outs)
    assert all(sum(c) == tokens * cfg.top_k for c in counts.values())
    stats = to_xtup(str(dump), str(tmp_path / "t.xtup"), per_layer=3)
    table = load_pin_table(tmp_path / "t.xtup")
    assert len(table) == cfg.num_layers and all(len(v) == 3 for v in table.values())
    assert 0.0 < stats["mean_coverage"] <= 1.0


def test_engine_config_env_names():
    ec = EngineConfig.from_env({"XIAOTU_PIN": "1", "XIAOTU_GPF_STAGE_TILE_E": "32", "XIAOTU_MOE_INT8": "off",
                                "XIAOTU_MOE_GPU_RESIDENT_LAYERS": "0-4,10", "VLLM_EXPERTS_LOAD_DEVICE": "cpu"})
    assert ec.pin is True and ec.stage_tile_e == 32 and ec.moe_int8 == "off"
    assert ec.resident_layers == "0-4,10" and ec.experts_load_device == "cpu"
