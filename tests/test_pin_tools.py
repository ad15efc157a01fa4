"""PIN-table tooling: coverage, held-out hit rate, LRU probe, budget-sized seed tables,
and a routing dump with per-window counts from a real (CPU) engine run."""
import json
import math

import pytest

from vllm_xtu_moe_b200.tiering import pin_tools as T
from vllm_xtu_moe_b200.tiering.host import expert_slot_bytes
from vllm_xtu_moe_b200.tiering.policy import load_pin_table


def _windows(n, E=8, hot=(1, 5), seed=0):
    import random
    rnd = random.Random(seed)
    wins = []
    for _ in range(n):
        w = {}
        for l in (0, 1):
            c = [0] * E
            for _ in range(40):
                e = rnd.choice(hot) if rnd.random() < 0.8 else rnd.randrange(E)
                c[(e + l) % E] += 1
            w[l] = c
        wins.append(w)
    return wins


def test_coverage_and_heldout_hit_rate():
    wins = _windows(20)
    counts = {l: [sum(w[l][e] for w in wins) for e in range(8)] for l in (0, 1)}
    cov = T.coverage(counts, 2)
    assert 0.75 < cov["coverage"] <= 1.0
    h = T.heldout_hit_rate(wins, 2, folds=10)
    assert 0.7 < h <= cov["coverage"] + 1e-9          # held out never beats in-sample here
    assert math.isnan(T.heldout_hit_rate(wins[:5], 2, folds=10))
    assert T.heldout_hit_rate(wins, 8, folds=10) == pytest.approx(1.0)
    assert T.lru_hit_rate(wins, 0) == 0.0 and T.lru_hit_rate(wins, 16) > 0.95


def test_seed_table_sizing_and_fill(tmp_path):
    slot = expert_slot_bytes("fp8", 4096, 1408)
    assert slot == 3 * 4096 * 1408 + (2 * 1408 // 128) * (4096 // 128) * 4 + (4096 // 128) * (1408 // 128) * 4
    n = T.slots_for_budget(20.0, "fp8", 4096, 1408, 45)
    assert n * 45 * slot <= 20 * 2 ** 30 < (n + 1) * 45 * slot
    counts = {3: [0, 5, 0, 9, 1, 0, 0, 0]}
    tab = T.seed_table([3, 4], 8, 3, counts)
    assert tab == {3: [3, 1, 4], 4: [0, 1, 2]}
    out = tmp_path / "seed.xtup"
    T.main(["seed", str(out), "--model", "glm-4.5-air", "--slots-per-layer", "4"])
    t = load_pin_table(out)
    assert len(t) == 45 and all(v == [0, 1, 2, 3] for v in t.values())


def test_routing_dump_windows_from_an_engine_run(tmp_path, monkeypatch, capsys):
    from vllm_xtu_moe_b200.config import get_engine_config
    from vllm_xtu_moe_b200.engine import LLM, SamplingParams
    from vllm_xtu_moe_b200.engine.runner import RunnerConfig
    from vllm_xtu_moe_b200.models.config import get_preset
    dump = tmp_path / "route.json"
    monkeypatch.setenv("XIAOTU_ROUTING_DUMP", str(dump))
    monkeypatch.setenv("XIAOTU_ROUTING_DUMP_WINDOW", "2")
    ec = get_engine_config(refresh=True)
    try:
        llm = LLM(get_preset("tiny-mixtral"), device="cpu", engine_config=ec,
                  runner_config=RunnerConfig(block_size=16, max_seqs=2, max_model_len=128, max_batched_tokens=64,
                                             use_cuda_graph=False))
        llm.generate([list(range(1, 30)), list(range(40, 50))], SamplingParams(max_tokens=9))
        llm.shutdown()
    finally:
        monkeypatch.delenv("XIAOTU_ROUTING_DUMP")
        get_engine_config(refresh=True)
    d = json.loads(dump.read_text())
    assert d["window_steps"] == 2 and len(d["windows"]) >= 4
    # windows add up to the totals
    for l, row in d["counts"].items():
        assert [sum(w.get(l, [0] * len(row))[e] for w in d["windows"]) for e in range(len(row))] == row
    T.main(["profile", str(dump), "--slots", "2,4", "--folds", "2"])
    rep = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert rep["windows"] == len(d["windows"]) and len(rep["by_slots"]) == 2
    assert 0 < rep["by_slots"][0]["hit_rate_heldout"] <= 1
